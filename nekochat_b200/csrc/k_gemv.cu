// Dequantising GEMV / skinny matmul over the engine's packed weight rows: the MatmulQ8, MatmulQ4 and Matmul
// kernels (app/architecture/shared/cpp/gpu/shaders/matmul_q8.comp, matmul_q4.comp, matmul.comp) and
// cpu::matmul (cpu_ops.cpp:462-481), written for sm_100a.
//
// Shape of the work: y[m][n] = sum_k x[m][k] * deq(W[n])[k] for M <= a few rows (decode) and N up to 152K rows
// of K <= 10K weights. Every weight byte is read once per step, so the kernel is bound by HBM bandwidth.
//
// Design
//  * Persistent CTAs, one contiguous range of weight rows each (rows are self-contained, quant.h:34-36).
//  * A producer warp streams the range into a ring of shared-memory stages with cp.async.bulk (the TMA
//    engine, no registers or LSU involved), each stage completing on an mbarrier; 8 consumer warps compute.
//  * Programmatic dependent launch: the producer issues its first stages BEFORE griddepcontrol.wait, so the
//    next kernel's weights stream in while the previous kernel (attention, another GEMV) is still running.
//    Only activations depend on the predecessor; consumers wait for it before staging x.
//  * Activations are staged once per CTA in shared memory, optionally normalised on the way (RMSNorm or
//    LayerNorm prologue: the norm of the reference's preceding LayerNorm dispatch is fused here).
//  * Consumers: warp w owns R consecutive rows of each stage; lane l reads 4 code bytes per 128-byte segment
//    (conflict-free), decodes them in registers with the engine's own bit layout (exact), multiplies with
//    fp32 activations and applies the f16 block scale per 32 weights; fp32 warp-shuffle reduction per row.
//  * Fused epilogues: bias, GELU, residual accumulate, and the SwiGLU pair (gate row n with up row n + F).
#include "neko_common.cuh"
#include "neko_internal.h"

namespace neko {

namespace {

constexpr int kConsumerWarps = 8;
constexpr int kThreads = (kConsumerWarps + 1) * 32;

// Physical float index of logical activation k in the staged x row. FP4 reads x in two 4-float groups 16 apart
// per lane; flipping bit 4 for odd 32-blocks keeps those reads bank-conflict free.
template <int FMT>
__device__ __forceinline__ int xphys(int k) {
    return FMT == kFP4 ? (k ^ (((k >> 5) & 1) << 4)) : k;
}

struct XSrc {
    const float* base;  // smem (staged) or global
    int64_t stride;     // floats between rows
    bool smem;
};

template <int FMT>
__device__ __forceinline__ float4 load_x4(const XSrc& xs, int m, int k) {
    const float* p = xs.base + int64_t(m) * xs.stride + (xs.smem ? xphys<FMT>(k) : k);
    return *reinterpret_cast<const float4*>(p);
}

// Stages activation rows [0, M) into shared memory, applying the norm prologue.
// RMSNorm: y = x * rsqrt(mean(x^2) + eps) * gamma; LayerNorm: (x - mean) * rstd * gamma + beta
// (cpu_ops.cpp:483-511: sums accumulated in double like the CPU reference).
template <int FMT>
__device__ void stage_x(const GemvArgs& a, float* xs, int warp, int lane) {
    for (int m = warp; m < a.M; m += kConsumerWarps) {
        const float* src = a.x + int64_t(m) * a.x_stride;
        float* dst = xs + int64_t(m) * a.K;
        double s1 = 0.0, s2 = 0.0;
        for (int k = lane * 4; k < a.K; k += 128) {
            float4 v = *reinterpret_cast<const float4*>(src + k);
            *reinterpret_cast<float4*>(dst + xphys<FMT>(k)) = v;
            s1 += double(v.x) + double(v.y) + double(v.z) + double(v.w);
            s2 += double(v.x) * v.x + double(v.y) * v.y + double(v.z) * v.z + double(v.w) * v.w;
        }
        if (a.norm == kNormNone) continue;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            s1 += __shfl_xor_sync(0xffffffffu, s1, o);
            s2 += __shfl_xor_sync(0xffffffffu, s2, o);
        }
        float r, mean = 0.0f;
        if (a.norm == kNormRms) {
            r = float(1.0 / sqrt(s2 / a.K + double(a.eps)));
        } else {
            const double mu = s1 / a.K;
            double var = 0.0;
            __syncwarp();
            for (int k = lane * 4; k < a.K; k += 128) {
                float4 v = *reinterpret_cast<const float4*>(dst + xphys<FMT>(k));
                double d0 = v.x - mu, d1 = v.y - mu, d2 = v.z - mu, d3 = v.w - mu;
                var += d0 * d0 + d1 * d1 + d2 * d2 + d3 * d3;
            }
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) var += __shfl_xor_sync(0xffffffffu, var, o);
            r = float(1.0 / sqrt(var / a.K + double(a.eps)));
            mean = float(mu);
        }
        __syncwarp();
        for (int k = lane * 4; k < a.K; k += 128) {
            float4* p = reinterpret_cast<float4*>(dst + xphys<FMT>(k));
            float4 v = *p;
            float4 g = *reinterpret_cast<const float4*>(a.gamma + k);
            if (a.norm == kNormRms) {
                v.x = __fmul_rn(__fmul_rn(v.x, r), g.x);
                v.y = __fmul_rn(__fmul_rn(v.y, r), g.y);
                v.z = __fmul_rn(__fmul_rn(v.z, r), g.z);
                v.w = __fmul_rn(__fmul_rn(v.w, r), g.w);
            } else {
                float4 b = *reinterpret_cast<const float4*>(a.beta + k);
                v.x = __fadd_rn(__fmul_rn(__fmul_rn(__fsub_rn(v.x, mean), r), g.x), b.x);
                v.y = __fadd_rn(__fmul_rn(__fmul_rn(__fsub_rn(v.y, mean), r), g.y), b.y);
                v.z = __fadd_rn(__fmul_rn(__fmul_rn(__fsub_rn(v.z, mean), r), g.z), b.z);
                v.w = __fadd_rn(__fmul_rn(__fmul_rn(__fsub_rn(v.w, mean), r), g.w), b.w);
            }
            *p = v;
        }
    }
}

// Partial dot product of one lane's slice of one row with MT activation rows.
// FP8: 4 codes at byte k0 (weights k0..k0+3) of block k0/32.
template <int MT>
__device__ __forceinline__ void dot_fp8(const uint8_t* row, int K, int k0, const float4 (&xv)[MT], float (&acc)[MT]) {
    const uint32_t q = *reinterpret_cast<const uint32_t*>(row + k0);
    const float s = half_bits_to_float(*reinterpret_cast<const uint16_t*>(row + K + 2 * (k0 >> 5)));
    __half2 e, o;
    fp8x4_to_half2(q, e, o);
    const float2 fe = __half22float2(e), fo = __half22float2(o);
#pragma unroll
    for (int m = 0; m < MT; m++) {
        float p = xv[m].x * fe.x;
        p = fmaf(xv[m].y, fo.x, p);
        p = fmaf(xv[m].z, fe.y, p);
        p = fmaf(xv[m].w, fo.y, p);
        acc[m] = fmaf(s, p, acc[m]);
    }
}

// FP4: 4 code bytes at byte b0 of the row's code area; byte j of block blk holds weight j (low nibble) and
// weight 16 + j (high nibble). xl/xh are activations 32*blk + j0 .. +3 and 32*blk + 16 + j0 .. +3.
template <int MT>
__device__ __forceinline__ void dot_fp4(const uint8_t* row, int K, int b0, const float4 (&xl)[MT],
                                        const float4 (&xh)[MT], float (&acc)[MT]) {
    const uint32_t q = *reinterpret_cast<const uint32_t*>(row + b0);
    const float s = half_bits_to_float(*reinterpret_cast<const uint16_t*>(row + (K >> 1) + 2 * (b0 >> 4)));
    const float2 le = __half22float2(fp4x2_to_half2(q & 0x000F000Fu));
    const float2 lo = __half22float2(fp4x2_to_half2((q >> 8) & 0x000F000Fu));
    const float2 he = __half22float2(fp4x2_to_half2((q >> 4) & 0x000F000Fu));
    const float2 ho = __half22float2(fp4x2_to_half2((q >> 12) & 0x000F000Fu));
#pragma unroll
    for (int m = 0; m < MT; m++) {
        float p = xl[m].x * le.x;
        p = fmaf(xl[m].y, lo.x, p);
        p = fmaf(xl[m].z, le.y, p);
        p = fmaf(xl[m].w, lo.y, p);
        p = fmaf(xh[m].x, he.x, p);
        p = fmaf(xh[m].y, ho.x, p);
        p = fmaf(xh[m].z, he.y, p);
        p = fmaf(xh[m].w, ho.y, p);
        acc[m] = fmaf(s, p, acc[m]);
    }
}

// F16: 4 halves at element k0.
template <int MT>
__device__ __forceinline__ void dot_f16(const uint8_t* row, int k0, const float4 (&xv)[MT], float (&acc)[MT]) {
    const uint2 q = *reinterpret_cast<const uint2*>(row + 2 * k0);
    const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&q.x));
    const float2 b = __half22float2(*reinterpret_cast<const __half2*>(&q.y));
#pragma unroll
    for (int m = 0; m < MT; m++) {
        acc[m] = fmaf(xv[m].x, a.x, acc[m]);
        acc[m] = fmaf(xv[m].y, a.y, acc[m]);
        acc[m] = fmaf(xv[m].z, b.x, acc[m]);
        acc[m] = fmaf(xv[m].w, b.y, acc[m]);
    }
}

// Accumulates R rows (row stride rb inside the stage) x MT activation rows over the full K of the rows.
template <int FMT, int R, int MT>
__device__ __forceinline__ void row_block(const uint8_t* rows0, int64_t rb, int nr, int K, const XSrc& xs, int m0,
                                          int M, int lane, float (&acc)[R][MT]) {
#pragma unroll
    for (int r = 0; r < R; r++)
#pragma unroll
        for (int m = 0; m < MT; m++) acc[r][m] = 0.0f;
    if (FMT == kFP4) {
        for (int b0 = lane * 4; b0 < (K >> 1); b0 += 128) {
            const int blk = b0 >> 4, j0 = b0 & 15;
            float4 xl[MT], xh[MT];
#pragma unroll
            for (int m = 0; m < MT; m++) {
                const bool ok = m0 + m < M;
                xl[m] = ok ? load_x4<FMT>(xs, m0 + m, 32 * blk + j0) : make_float4(0, 0, 0, 0);
                xh[m] = ok ? load_x4<FMT>(xs, m0 + m, 32 * blk + 16 + j0) : make_float4(0, 0, 0, 0);
            }
#pragma unroll
            for (int r = 0; r < R; r++)
                if (r < nr) dot_fp4<MT>(rows0 + r * rb, K, b0, xl, xh, acc[r]);
        }
    } else {
        for (int k0 = lane * 4; k0 < K; k0 += 128) {
            float4 xv[MT];
#pragma unroll
            for (int m = 0; m < MT; m++)
                xv[m] = m0 + m < M ? load_x4<FMT>(xs, m0 + m, k0) : make_float4(0, 0, 0, 0);
#pragma unroll
            for (int r = 0; r < R; r++) {
                if (r >= nr) continue;
                if (FMT == kFP8) dot_fp8<MT>(rows0 + r * rb, K, k0, xv, acc[r]);
                else dot_f16<MT>(rows0 + r * rb, k0, xv, acc[r]);
            }
        }
    }
}

template <int FMT, int R, int MT>
__global__ void __launch_bounds__(kThreads, 2) gemv_kernel(const GemvArgs a) {
    extern __shared__ __align__(128) uint8_t smem[];
    constexpr float kFactor = FMT == kFP8 ? kFp8Factor : FMT == kFP4 ? kFp4Factor : 1.0f;
    uint64_t* full = reinterpret_cast<uint64_t*>(smem);
    uint64_t* empty = full + a.nstage;
    float* xs = reinterpret_cast<float*>(smem + a.xs_off);
    uint8_t* ring = smem + a.ring_off;
    const bool paired = a.pair_off != 0;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

    const int r0 = blockIdx.x * a.rows_per_cta;
    const int r1 = min(a.rows, r0 + a.rows_per_cta);
    const int SR = a.stage_rows;
    pdl_trigger();
    if (r0 >= r1) return;
    const int nst = (r1 - r0 + SR - 1) / SR;

    if (threadIdx.x == 0) {
        for (int s = 0; s < a.nstage; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], kConsumerWarps);
        }
        fence_barrier_init();
    }
    __syncthreads();

    if (warp == kConsumerWarps) {
        // ---------------- producer: weights only, so it never waits for the previous kernel
        if (lane == 0) {
            for (int st = 0; st < nst; st++) {
                const int slot = st % a.nstage;
                if (st >= a.nstage && !mbar_wait(&empty[slot], ((st / a.nstage) - 1) & 1)) break;
                const int row = r0 + st * SR;
                const int n = min(SR, r1 - row);
                const uint32_t bytes = uint32_t(n * a.row_bytes);
                uint8_t* dst = ring + slot * a.stage_stride;
                mbar_arrive_expect_tx(&full[slot], paired ? 2 * bytes : bytes);
                bulk_g2s(dst, a.W + int64_t(row) * a.row_bytes, bytes, &full[slot]);
                if (paired)
                    bulk_g2s(dst + SR * a.row_bytes, a.W + (int64_t(row) + a.pair_off) * a.row_bytes, bytes,
                             &full[slot]);
            }
        }
        return;
    }

    // ---------------- consumers
    pdl_wait();
    XSrc src;
    if (a.x_smem) {
        stage_x<FMT>(a, xs, warp, lane);
        asm volatile("bar.sync 1, %0;" ::"n"(kConsumerWarps * 32) : "memory");
        src = XSrc{xs, a.K, true};
    } else {
        src = XSrc{a.x, a.x_stride, false};
    }

    for (int st = 0; st < nst; st++) {
        const int slot = st % a.nstage;
        if (!mbar_wait(&full[slot], (st / a.nstage) & 1)) return;
        const int row0 = r0 + st * SR;
        const int nrows = min(SR, r1 - row0);
        const int my0 = warp * R;
        const int nr = min(R, nrows - my0);
        if (nr > 0) {
            const uint8_t* stage = ring + slot * a.stage_stride + my0 * a.row_bytes;
            for (int m0 = 0; m0 < a.M; m0 += MT) {
                float acc[R][MT];
                row_block<FMT, R, MT>(stage, a.row_bytes, nr, a.K, src, m0, a.M, lane, acc);
                float accu[R][MT];
                if (paired) row_block<FMT, R, MT>(stage + SR * a.row_bytes, a.row_bytes, nr, a.K, src, m0, a.M, lane,
                                                  accu);
#pragma unroll
                for (int r = 0; r < R; r++) {
#pragma unroll
                    for (int m = 0; m < MT; m++) {
                        const float g = warp_sum(acc[r][m]) * kFactor;
                        const float u = paired ? warp_sum(accu[r][m]) * kFactor : 0.0f;
                        if (r >= nr || m0 + m >= a.M || lane != ((r * MT + m) & 31)) continue;
                        const int n = row0 + my0 + r;
                        float* dst = a.y + int64_t(m0 + m) * a.y_stride + a.n_off + n;
                        float v;
                        if (paired) {
                            v = g / (1.0f + expf(-g)) * u;  // cpu::siluMul (cpu_ops.cpp:526-533)
                        } else {
                            v = g;
                            if (a.flags & kBias) v += a.bias[n];
                            if (a.flags & kGelu) v = gelu(v);
                            if (a.flags & kAccumulate) v += *dst;
                        }
                        *dst = v;
                    }
                }
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[slot]);
    }
}

using KernelFn = void (*)(const GemvArgs);

template <int FMT>
KernelFn pick_mt(int R, int MT) {
#define NEKO_PICK(RR, MM) \
    if (R == RR && MT == MM) return &gemv_kernel<FMT, RR, MM>;
    NEKO_PICK(1, 1) NEKO_PICK(1, 2) NEKO_PICK(1, 4)
    NEKO_PICK(2, 1) NEKO_PICK(2, 2) NEKO_PICK(2, 4)
    NEKO_PICK(4, 1) NEKO_PICK(4, 2) NEKO_PICK(4, 4)
#undef NEKO_PICK
    return nullptr;
}

KernelFn pick(int fmt, int R, int MT) {
    return fmt == kFP8 ? pick_mt<kFP8>(R, MT) : fmt == kFP4 ? pick_mt<kFP4>(R, MT) : pick_mt<kF16>(R, MT);
}

// Opt every instantiation into the large dynamic shared memory budget once per device.
cudaError_t ensure_smem_attr() {
    static int done_mask = 0;
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 31 && (done_mask >> dev) & 1) return cudaSuccess;
    for (int f : {kF16, kFP8, kFP4})
        for (int R : {1, 2, 4})
            for (int MT : {1, 2, 4}) {
                cudaError_t e = cudaFuncSetAttribute(pick(f, R, MT), cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                     kGemvSmemBudget);
                if (e != cudaSuccess) return e;
            }
    if (dev < 31) done_mask |= 1 << dev;
    return cudaSuccess;
}

}  // namespace

int gemv_launch_count() { return 1; }

cudaError_t launch_gemv(GemvArgs a, cudaStream_t st, bool pdl, int max_ctas) {
    if (a.rows <= 0 || a.M <= 0) return cudaSuccess;
    if (cudaError_t e = ensure_smem_attr(); e != cudaSuccess) return e;
    const bool paired = a.pair_off != 0;
    const int sms = num_sms();
    // CTAs: one per SM, fewer when there are too few rows to give each at least 4.
    int ctas = max_ctas > 0 ? max_ctas : sms;
    ctas = std::max(1, std::min(ctas, (a.rows + 3) / 4));
    a.rows_per_cta = (a.rows + ctas - 1) / ctas;
    ctas = (a.rows + a.rows_per_cta - 1) / a.rows_per_cta;

    // Activations staged in shared memory when they fit (required for the norm prologue).
    const int64_t x_bytes = int64_t(a.M) * a.K * 4;
    a.x_smem = (x_bytes <= kGemvXSmemMax) ? 1 : 0;
    if (!a.x_smem && a.norm != kNormNone) return cudaErrorInvalidValue;
    if (!a.x_smem && (a.x_stride % 4 != 0 || (reinterpret_cast<uintptr_t>(a.x) & 15) != 0))
        return cudaErrorInvalidValue;

    // Rows per warp per stage: enough that one stage is ~16-32 KB, but not more than the CTA's share.
    const int64_t rb = a.row_bytes * (paired ? 2 : 1);
    int R = int(std::max<int64_t>(1, 24576 / (kConsumerWarps * rb)));
    const int per_warp = (a.rows_per_cta + kConsumerWarps - 1) / kConsumerWarps;
    R = std::min(R, per_warp);
    R = R >= 4 ? 4 : R >= 2 ? 2 : 1;
    // activation rows per pass over a stage (more rows loop; 4 x 4 accumulators keep the kernel spill-free)
    const int MT = a.M >= 4 ? 4 : a.M >= 2 ? 2 : 1;

    a.xs_off = 128 * ((2 * 8 * 8 + 127) / 128);  // room for up to 8 stages of (full, empty) barriers
    const int x_alloc = a.x_smem ? int((x_bytes + 127) / 128 * 128) : 0;
    a.ring_off = a.xs_off + x_alloc;
    const int64_t room = kGemvSmemBudget - a.ring_off;
    // Rows per stage: one row block per warp, fewer when very wide rows would leave room for less than two stages.
    int64_t sr = int64_t(kConsumerWarps) * R;
    if (2 * sr * rb > room) sr = std::max<int64_t>(1, room / (2 * rb));
    if (sr * rb > room) sr = room / rb;
    if (sr < 1) return cudaErrorInvalidValue;  // a single row does not fit next to the staged activations
    a.stage_rows = int(sr);
    a.stage_stride = (sr * rb + 127) / 128 * 128;
    const int stages_needed = int((a.rows_per_cta + sr - 1) / sr);
    a.nstage = int(std::min<int64_t>(std::min(8, stages_needed), room / a.stage_stride));
    if (a.nstage < 1) return cudaErrorInvalidValue;
    const size_t smem = size_t(a.ring_off + a.nstage * a.stage_stride);
    return launch_ex(pick(a.fmt, R, MT), dim3(ctas), dim3(kThreads), smem, st, pdl, a);
}

}  // namespace neko
