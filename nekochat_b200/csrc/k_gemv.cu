// Dequantising GEMV / skinny matmul over the engine's packed weight rows: the MatmulQ8, MatmulQ4 and Matmul
// kernels (app/architecture/shared/cpp/gpu/shaders/matmul_q8.comp, matmul_q4.comp, matmul.comp) and
// cpu::matmul (cpu_ops.cpp:462-481), written for sm_100a.
//
// Shape of the work: y[m][n] = sum_k x[m][k] * deq(W[n])[k] for M <= a few rows (decode) and N up to 152K rows
// of K <= 10K weights. Every weight byte is read once per step, so the kernel is bound by HBM bandwidth and, for
// the small per-layer matrices of a decode step, by latency.
//
// Design
//  * Persistent CTAs, one contiguous range of weight rows each (rows are self-contained, quant.h:34-36).
//  * A producer warp streams the range into a ring of shared-memory stages with cp.async.bulk (the TMA engine),
//    in chunks of at most 4 KB issued by all its lanes, each stage completing on an mbarrier; 8 consumer warps
//    compute. With programmatic dependent launch the producer issues its first stages BEFORE
//    griddepcontrol.wait, so the weights stream in while the previous kernel is still running; only the
//    activations depend on the predecessor.
//  * Activations are staged once per CTA by all consumer threads into a permuted shared-memory layout in which
//    each lane's 16-weight slice reads its activations as bank-conflict-free float4s; an RMSNorm / LayerNorm
//    prologue (the engine's preceding LayerNorm dispatch) is applied on the way.
//  * Consumers: a row is walked in 512-byte segments; lane l takes bytes [16 l, 16 l + 16) of each segment with
//    one 128-bit shared load (16 FP8 codes, one 32-weight FP4 block, or 8 halves), decodes them in registers
//    with the engine's own bit layout (exact), multiplies with fp32 activations in two independent chains,
//    applies the f16 block scale and reduces each row with warp shuffles.
//  * Fused epilogues: bias, GELU, residual accumulate, the SwiGLU pair (gate row n with up row n + F), and a
//    greedy argmax (max of (value, ~index) keys) for the LM head.
#include "neko_common.cuh"
#include "neko_internal.h"
#include "gemv_core.cuh"

namespace neko {

namespace {

constexpr int kConsumerWarps = 8;
constexpr int kThreads = (kConsumerWarps + 1) * 32;
constexpr int kMaxArgmaxRows = 64;
constexpr int kMaxStageVec = 10;  // float4 activations staged per consumer thread (40 KB / 256 threads)
constexpr int kStageRound = 6;    // float4 loads a thread keeps in flight while staging
constexpr int kMaxNormVec = 4;    // float4 per thread when a norm prologue is fused (M * K <= 4096)
constexpr int kChunkBytes = 4096;

__device__ __forceinline__ void consumer_sync() {
    asm volatile("bar.sync 1, %0;" ::"n"(kConsumerWarps * 32) : "memory");
}

// Stages activation rows [0, M) into the permuted layout (zero-padded to whole segments), applying the norm
// prologue: RMSNorm y = x * rsqrt(mean(x^2) + eps) * gamma, LayerNorm (x - mean) * rstd * gamma + beta
// (cpu_ops.cpp:483-511; sums in double like the CPU reference, the LayerNorm variance as E[x^2] - mean^2 in
// double). All activation (and gamma / beta) loads of a thread are issued before any is used, so staging costs
// one L2 round trip; the row sums go through per-warp partials in shared memory in a fixed order.
template <int FMT>
__device__ void stage_x(const GemvArgs& a, float* xs, double* part, int tid, int warp, int lane) {
    constexpr int NT = kConsumerWarps * 32;
    const int K4 = a.K / 4, total = a.M * K4, padded = seg_count(FMT, a.K) * Seg<FMT>::W;
    const bool norm = a.norm != kNormNone;
    for (int m = 0; m < a.M; m++) {
        float* row = xs + m * padded;
        for (int k = a.K + tid; k < padded; k += NT) row[xperm<FMT>(k)] = 0.0f;
    }
    if (!norm) {
        // rounds of kStageRound float4 per thread: all loads of a round are in flight together
        for (int base = 0; base < total; base += kStageRound * NT) {
            float4 v[kStageRound];
#pragma unroll
            for (int j = 0; j < kStageRound; j++) {
                const int i = base + tid + j * NT;
                if (i < total) v[j] = *reinterpret_cast<const float4*>(a.x + int64_t(i / K4) * a.x_stride + 4 * (i % K4));
            }
#pragma unroll
            for (int j = 0; j < kStageRound; j++) {
                const int i = base + tid + j * NT;
                if (i < total) *reinterpret_cast<float4*>(xs + (i / K4) * padded + xperm<FMT>(4 * (i % K4))) = v[j];
            }
        }
        consumer_sync();
        return;
    }
    float4 v[kMaxNormVec], g[kMaxNormVec], b[kMaxNormVec];
#pragma unroll
    for (int j = 0; j < kMaxNormVec; j++) {
        const int i = tid + j * NT;
        if (i < total) v[j] = *reinterpret_cast<const float4*>(a.x + int64_t(i / K4) * a.x_stride + 4 * (i % K4));
    }
    // norm: at most kMaxNormVec float4 per thread and K % 128 == 0 (a warp's 32 float4 lie in one row)
#pragma unroll
    for (int j = 0; j < kMaxNormVec; j++) {
        const int i = tid + j * NT;
        if (i < total) {
            g[j] = __ldg(reinterpret_cast<const float4*>(a.gamma + 4 * (i % K4)));
            if (a.norm == kNormLayer) b[j] = __ldg(reinterpret_cast<const float4*>(a.beta + 4 * (i % K4)));
        }
    }
#pragma unroll
    for (int j = 0; j < kMaxNormVec; j++) {
        const int i = tid + j * NT;
        double s1 = 0.0, s2 = 0.0;
        if (i < total) {
            s1 = double(v[j].x) + double(v[j].y) + double(v[j].z) + double(v[j].w);
            s2 = double(v[j].x) * v[j].x + double(v[j].y) * v[j].y + double(v[j].z) * v[j].z + double(v[j].w) * v[j].w;
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            s1 += __shfl_xor_sync(0xffffffffu, s1, o);
            s2 += __shfl_xor_sync(0xffffffffu, s2, o);
        }
        if (lane == 0) {
            part[2 * (j * kConsumerWarps + warp)] = s1;
            part[2 * (j * kConsumerWarps + warp) + 1] = s2;
        }
    }
    consumer_sync();
#pragma unroll
    for (int j = 0; j < kMaxNormVec; j++) {
        const int i = tid + j * NT;
        if (i >= total) continue;
        const int m = i / K4;
        double s1 = 0.0, s2 = 0.0;  // the row's partials, in a fixed order: slots (j', w') whose float4s are in row m
        for (int jj = 0; jj < kMaxNormVec; jj++)
            for (int w = 0; w < kConsumerWarps; w++) {
                const int i0 = jj * NT + w * 32;
                if (i0 < total && i0 / K4 == m) {
                    s1 += part[2 * (jj * kConsumerWarps + w)];
                    s2 += part[2 * (jj * kConsumerWarps + w) + 1];
                }
            }
        float r, mean = 0.0f;
        if (a.norm == kNormRms) {
            r = float(1.0 / sqrt(s2 / a.K + double(a.eps)));
        } else {
            const double mu = s1 / a.K;
            r = float(1.0 / sqrt(s2 / a.K - mu * mu + double(a.eps)));
            mean = float(mu);
        }
        float4 y = v[j];
        if (a.norm == kNormRms) {
            y.x = __fmul_rn(__fmul_rn(y.x, r), g[j].x);
            y.y = __fmul_rn(__fmul_rn(y.y, r), g[j].y);
            y.z = __fmul_rn(__fmul_rn(y.z, r), g[j].z);
            y.w = __fmul_rn(__fmul_rn(y.w, r), g[j].w);
        } else {
            y.x = __fadd_rn(__fmul_rn(__fmul_rn(__fsub_rn(y.x, mean), r), g[j].x), b[j].x);
            y.y = __fadd_rn(__fmul_rn(__fmul_rn(__fsub_rn(y.y, mean), r), g[j].y), b[j].y);
            y.z = __fadd_rn(__fmul_rn(__fmul_rn(__fsub_rn(y.z, mean), r), g[j].z), b[j].z);
            y.w = __fadd_rn(__fmul_rn(__fmul_rn(__fsub_rn(y.w, mean), r), g[j].w), b[j].w);
        }
        *reinterpret_cast<float4*>(xs + m * padded + xperm<FMT>(4 * (i % K4))) = y;
    }
    consumer_sync();
}

// Accumulates nr (<= R) rows (row stride rb inside the stage) x MT activation rows over the full K.
template <int FMT, int R, int MT>
__device__ __forceinline__ void row_block(const uint8_t* rows0, int64_t rb, int nr, const GemvArgs& a,
                                          const float* xs, int m0, int lane, float (&acc)[R][MT]) {
    constexpr int Q = Seg<FMT>::Q, W = Seg<FMT>::W;
    const int cbytes = code_bytes(FMT, a.K), nseg = seg_count(FMT, a.K);
#pragma unroll
    for (int r = 0; r < R; r++)
#pragma unroll
        for (int m = 0; m < MT; m++) acc[r][m] = 0.0f;
    for (int s = 0; s < nseg; s++) {
        if (s * kSegBytes + 16 * lane >= cbytes) continue;  // lanes past the end of a partial last segment
        float4 xv[MT][Q];
#pragma unroll
        for (int m = 0; m < MT; m++) {
#pragma unroll
            for (int q = 0; q < Q; q++) {
                if (m0 + m >= a.M) {
                    xv[m][q] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
                } else if (xs) {  // permuted staging: float4 index ((s * Q + q) * 32 + lane) of row m
                    xv[m][q] =
                        reinterpret_cast<const float4*>(xs)[(m0 + m) * (nseg * Q * 32) + (s * Q + q) * 32 + lane];
                } else {  // activations read straight from global memory
                    const int k = s * W + lane * (W / 32) + 4 * q;
                    xv[m][q] = k < a.K ? __ldg(reinterpret_cast<const float4*>(a.x + int64_t(m0 + m) * a.x_stride + k))
                                       : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
                }
            }
        }
#pragma unroll
        for (int r = 0; r < R; r++)
            if (r < nr) seg_dot<FMT, MT>(rows0 + r * rb, cbytes, s, lane, xv, acc[r]);
    }
}

template <int FMT, int R, int MT>
__global__ void __launch_bounds__(kThreads, 2) gemv_kernel(const GemvArgs a) {
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ unsigned long long skey[kMaxArgmaxRows];  // fused greedy argmax: this CTA's best key per row
    __shared__ double part[2 * kMaxNormVec * kConsumerWarps];  // norm prologue: per-warp partial sums
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
    if (threadIdx.x < kMaxArgmaxRows) skey[threadIdx.x] = 0;
    __syncthreads();

    if (warp == kConsumerWarps) {
        // ---------------- producer warp: weights only, so it never waits for the previous kernel
        for (int st = 0; st < nst; st++) {
            const int slot = st % a.nstage;
            int ok = 1;
            if (st >= a.nstage && lane == 0) ok = mbar_wait(&empty[slot], ((st / a.nstage) - 1) & 1);
            if (!__shfl_sync(0xffffffffu, ok, 0)) break;
            const int row = r0 + st * SR;
            const int n = min(SR, r1 - row);
            const uint32_t bytes = uint32_t(n * a.row_bytes);
            uint8_t* dst = ring + slot * a.stage_stride;
            if (lane == 0) mbar_arrive_expect_tx(&full[slot], paired ? 2 * bytes : bytes);
            __syncwarp();
            const int nchunk = int((bytes + kChunkBytes - 1) / kChunkBytes);
            for (int c = lane; c < (paired ? 2 : 1) * nchunk; c += 32) {
                const int half = c / nchunk, cc = c % nchunk;
                const uint32_t off = uint32_t(cc) * kChunkBytes, sz = min(uint32_t(kChunkBytes), bytes - off);
                const uint8_t* src = a.W + (int64_t(row) + (half ? a.pair_off : 0)) * a.row_bytes + off;
                bulk_g2s(dst + (half ? SR * a.row_bytes : 0) + off, src, sz, &full[slot]);
            }
        }
        return;
    }

    // ---------------- consumers: activations depend on the previous kernel
    pdl_wait();
    if (a.x_smem) stage_x<FMT>(a, xs, part, threadIdx.x, warp, lane);

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
                row_block<FMT, R, MT>(stage, a.row_bytes, nr, a, a.x_smem ? xs : nullptr, m0, lane, acc);
                float accu[R][MT];
                if (paired)
                    row_block<FMT, R, MT>(stage + SR * a.row_bytes, a.row_bytes, nr, a, a.x_smem ? xs : nullptr, m0,
                                          lane, accu);
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
                        if (a.argmax) atomicMax(&skey[m0 + m], argmax_key(v, n));
                    }
                }
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[slot]);
    }
    if (a.argmax) {  // one global atomic per CTA and activation row
        consumer_sync();
        if (threadIdx.x < a.M) atomicMax(a.argmax + threadIdx.x, skey[threadIdx.x]);
    }
}

using KernelFn = void (*)(const GemvArgs);

template <int FMT>
KernelFn pick_mt(int R, int MT) {
#define NEKO_PICK(RR, MM) \
    if (R == RR && MT == MM) return &gemv_kernel<FMT, RR, MM>;
    NEKO_PICK(1, 1) NEKO_PICK(1, 2) NEKO_PICK(2, 1) NEKO_PICK(2, 2) NEKO_PICK(4, 1)
    if constexpr (FMT != kFP4) {  // FP4 tiles of 4 activation rows do not fit the register budget
        NEKO_PICK(1, 4)
    }
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
                KernelFn k = pick(f, R, MT);
                if (!k) continue;
                cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, kGemvSmemBudget);
                if (e != cudaSuccess) return e;
            }
    if (dev < 31) done_mask |= 1 << dev;
    return cudaSuccess;
}

}  // namespace

int gemv_launch_count() { return 1; }

cudaError_t launch_gemv(GemvArgs a, cudaStream_t st, bool pdl, int max_ctas) {
    if (a.rows <= 0 || a.M <= 0) return cudaSuccess;
    if (a.x_hi || a.in_ss || a.out_hi || a.out_ss) {  // matmul chaining: the tensor-core kernel or nothing
        const cudaError_t e = max_ctas <= 0 ? launch_gemm_tc(a, st, pdl) : cudaErrorNotSupported;
        return e == cudaErrorNotSupported ? cudaErrorInvalidValue : e;
    }
    if (max_ctas <= 0) {  // 1..4 activation rows: the streaming kernel; 5+: tensor cores (when the call fits)
        cudaError_t e = launch_gemv_stream(a, st, pdl);
        if (e != cudaErrorNotSupported) return e;
        e = launch_gemm_tc(a, st, pdl);
        if (e != cudaErrorNotSupported) return e;
    }
    if (cudaError_t e = ensure_smem_attr(); e != cudaSuccess) return e;
    const bool paired = a.pair_off != 0;
    const int sms = num_sms();
    // CTAs: one per SM, fewer when there are too few rows to give each at least 4.
    int ctas = max_ctas > 0 ? max_ctas : sms;
    ctas = std::max(1, std::min(ctas, (a.rows + 3) / 4));
    a.rows_per_cta = (a.rows + ctas - 1) / ctas;
    ctas = (a.rows + a.rows_per_cta - 1) / a.rows_per_cta;

    // Activations staged in shared memory (permuted, padded to whole segments) when they fit; the norm prologue
    // needs them there.
    static_assert(kGemvNormMaxElems == 4 * kConsumerWarps * 32 * kMaxNormVec, "norm prologue register budget");
    const int64_t x_bytes = gemv_x_bytes(a.fmt, a.M, a.K);
    a.x_smem = (x_bytes <= kGemvXSmemMax && int64_t(a.M) * a.K <= 4 * kConsumerWarps * 32 * kMaxStageVec) ? 1 : 0;
    if (a.norm != kNormNone && !gemv_norm_fusable(a.fmt, a.M, a.K)) return cudaErrorInvalidValue;
    if (a.x_stride % 4 != 0 || (reinterpret_cast<uintptr_t>(a.x) & 15) != 0 || a.K % 4 != 0)
        return cudaErrorInvalidValue;  // float4 activation loads
    if (a.norm != kNormNone && ((reinterpret_cast<uintptr_t>(a.gamma) & 15) ||
                                (a.norm == kNormLayer && (reinterpret_cast<uintptr_t>(a.beta) & 15))))
        return cudaErrorInvalidValue;
    if (a.argmax && (a.M > kMaxArgmaxRows || a.pair_off != 0)) return cudaErrorInvalidValue;

    // Rows per warp per stage: enough that one stage is ~16-32 KB, but not more than the CTA's share.
    const int64_t rb = a.row_bytes * (paired ? 2 : 1);
    int R = int(std::max<int64_t>(1, 24576 / (kConsumerWarps * rb)));
    const int per_warp = (a.rows_per_cta + kConsumerWarps - 1) / kConsumerWarps;
    R = std::min(R, per_warp);
    R = R >= 4 ? 4 : R >= 2 ? 2 : 1;
    // activation rows per pass over a stage (more rows loop); R x MT <= 4 (MT <= 2 for FP4) keeps the register
    // tiles spill-free
    int MT = a.M >= 4 ? 4 : a.M >= 2 ? 2 : 1;
    MT = std::min(MT, 4 / R);
    if (a.fmt == kFP4) MT = std::min(MT, 2);

    a.xs_off = 256;  // up to 8 stages of (full, empty) barriers
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
