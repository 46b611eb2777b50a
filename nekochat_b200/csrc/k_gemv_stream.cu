// Streaming dequant GEMV for 1..4 activation rows: the MatmulQ8 / MatmulQ4 dispatch (matmul_q8.comp,
// matmul_q4.comp; cpu::matmul, cpu_ops.cpp:462-481) when the weights are the whole cost.
//
// At M <= 4 every weight byte is used for at most 4 multiply-adds, so the kernel's job is to move the packed
// rows from HBM at full bandwidth and keep the decode arithmetic off the critical path:
//  * one CTA per SM, a contiguous range of rows each; a producer warp streams the range through a ring of
//    stages of up to 52 KB with cp.async.bulk (TMA), 8 KB per copy (large stages: fewer producer / consumer
//    hand-offs, which is what limits a TMA ring's rate);
//  * 16 consumer warps work stage by stage: a stage holds 16 x rpw rows (rpw <= 4, the rows per warp), warp w
//    takes rows w, w + 16, ... of it with all their 128-bit weight loads issued before the math (SwiGLU: gate
//    and up rows together); one lane waits for the stage and releases it; FP8 codes are decoded by the
//    hardware e4m3 -> f16 conversion (the engine's FP8 code is e4m3, see gemv_core.cuh), FP4 by bit arithmetic;
//  * four rows are reduced across the warp together (6 shuffles instead of 20) before the stores;
//  * activations (with the optional RMSNorm / LayerNorm prologue) are staged once per CTA with cp.async.
// The per-row arithmetic is seg_dot_rows, the same as the single-kernel decode step's, so the two agree.
#include <algorithm>

#include "gemv_core.cuh"
#include "mma_frag.cuh"
#include "neko_common.cuh"
#include "neko_internal.h"

namespace neko {

namespace {

constexpr int kSW = 16;              // consumer warps
constexpr int kSNT = kSW * 32;       // consumer threads
constexpr int kSThr = kSNT + 32;     // + the producer warp
constexpr int kSMaxSlots = 16;
constexpr int kSChunk = 8192;        // bytes per bulk copy
constexpr int kSMaxStat = 64;        // norm partial slots (M * K / 128 <= 4096 / 128)

// Dynamic shared memory: full[16] | empty[16] | TShared | activations | ring. The small per-CTA arrays live in
// the dynamic region too: file-scope __shared__ arrays are placed by the device linker in one window shared
// with the other files' and would make this kernel's static shared memory depend on them.
extern __shared__ __align__(128) uint8_t gsm[];
struct TShared {
    double part[2 * kSMaxStat];                // norm partial sums
    unsigned long long key[kDecodeMaxSeqs];    // the CTA's greedy argmax keys
};
constexpr int kSHdr = 256 + int(sizeof(TShared) + 127) / 128 * 128;  // bytes before the activations
__device__ __forceinline__ TShared& tsh() { return *reinterpret_cast<TShared*>(gsm + 256); }

template <int NM>
constexpr int kSRows = NM == 1 ? 4 : 2;  // rows per warp pass

__device__ __forceinline__ void ssync() { asm volatile("bar.sync 1, %0;" ::"n"(kSNT) : "memory"); }
__device__ __forceinline__ double wsum_d(double v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// The M activation rows into the permuted layout of seg_dot_rows, with the norm prologue (sums in double,
// cpu_ops.cpp:483-511).
template <int FMT>
__device__ void stage_act(const GemvArgs& a, float* xs, int warp, int lane) {
    const int tid = threadIdx.x, K4 = a.K / 4, total = a.M * K4, xrow = seg_count(FMT, a.K) * Seg<FMT>::W;
    for (int i = tid; i < total; i += kSNT) {
        const int m = i / K4, k = 4 * (i - m * K4);
        asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(xs + m * xrow + xperm<FMT>(k))),
                     "l"(a.x + int64_t(m) * a.x_stride + k)
                     : "memory");
    }
    asm volatile("cp.async.wait_all;" ::: "memory");
    if (a.norm == kNormNone) {
        ssync();
        return;
    }
    for (int base = 0; base < total; base += kSNT) {  // K % 128 == 0: a warp's 32 float4 share a row
        const int i = base + tid;
        double s1 = 0.0, s2 = 0.0;
        if (i < total) {
            const int m = i / K4;
            const float4 v = *reinterpret_cast<const float4*>(xs + m * xrow + xperm<FMT>(4 * (i - m * K4)));
            s1 = double(v.x) + double(v.y) + double(v.z) + double(v.w);
            s2 = double(v.x) * v.x + double(v.y) * v.y + double(v.z) * v.z + double(v.w) * v.w;
        }
        if (base + warp * 32 < total) {
            s1 = wsum_d(s1);
            s2 = wsum_d(s2);
            if (lane == 0) {
                tsh().part[2 * (base / 32 + warp)] = s1;
                tsh().part[2 * (base / 32 + warp) + 1] = s2;
            }
        }
    }
    ssync();
    const int gpr = K4 / 32;  // partial slots per row
    for (int i = tid; i < total; i += kSNT) {
        const int m = i / K4, k = 4 * (i - m * K4);
        double a1 = 0.0, a2 = 0.0;
        for (int q = m * gpr; q < (m + 1) * gpr; q++) {
            a1 += tsh().part[2 * q];
            a2 += tsh().part[2 * q + 1];
        }
        float mean = 0.0f, r;
        if (a.norm == kNormRms) {
            r = float(1.0 / sqrt(a2 / a.K + double(a.eps)));
        } else {
            const double mu = a1 / a.K;
            mean = float(mu);
            r = float(1.0 / sqrt(a2 / a.K - mu * mu + double(a.eps)));
        }
        float4* px = reinterpret_cast<float4*>(xs + m * xrow + xperm<FMT>(k));
        float4 y = *px;
        const float4 ga = __ldg(reinterpret_cast<const float4*>(a.gamma + k));
        if (a.norm == kNormRms) {
            y.x = __fmul_rn(__fmul_rn(y.x, r), ga.x);
            y.y = __fmul_rn(__fmul_rn(y.y, r), ga.y);
            y.z = __fmul_rn(__fmul_rn(y.z, r), ga.z);
            y.w = __fmul_rn(__fmul_rn(y.w, r), ga.w);
        } else {
            const float4 be = __ldg(reinterpret_cast<const float4*>(a.beta + k));
            y.x = __fadd_rn(__fmul_rn(__fmul_rn(__fsub_rn(y.x, mean), r), ga.x), be.x);
            y.y = __fadd_rn(__fmul_rn(__fmul_rn(__fsub_rn(y.y, mean), r), ga.y), be.y);
            y.z = __fadd_rn(__fmul_rn(__fmul_rn(__fsub_rn(y.z, mean), r), ga.z), be.z);
            y.w = __fadd_rn(__fmul_rn(__fmul_rn(__fsub_rn(y.w, mean), r), ga.w), be.w);
        }
        *px = y;
    }
    ssync();
}

// The producer warp: every stage of this CTA's rows (rps rows per stage; SwiGLU: the gate rows, then the up
// rows) into the ring with cp.async.bulk, 8 KB per copy, waiting for a slot to be released before reusing it.
__device__ void stream_producer(const GemvArgs& a, int r0, int r1, int rps, int nslot, int slot_bytes, uint64_t* full,
                                uint64_t* empty, uint8_t* ring, int lane) {
    const bool pair = a.pair_off != 0;
    const int nst = (r1 - r0 + rps - 1) / rps;
    int st = 0;
    for (; st < nst; st++) {
        const int slot = st % nslot;
        if (st >= nslot) {
            int ok = 1;
            if (lane == 0) ok = mbar_wait(&empty[slot], ((st / nslot) - 1) & 1);
            if (!__shfl_sync(0xffffffffu, ok, 0)) break;
        }
        const int row = r0 + st * rps, cnt = min(rps, r1 - row);
        const uint32_t bytes = uint32_t(cnt) * uint32_t(a.row_bytes);
        uint8_t* dst = ring + size_t(slot) * slot_bytes;
        if (lane == 0) mbar_arrive_expect_tx(&full[slot], pair ? 2 * bytes : bytes);
        __syncwarp();
        const int nch = int((bytes + kSChunk - 1) / kSChunk);
        for (int c = lane; c < (pair ? 2 : 1) * nch; c += 32) {
            const int half = c >= nch ? 1 : 0, cc = c - half * nch;
            const uint32_t off = uint32_t(cc) * kSChunk, sz = min(uint32_t(kSChunk), bytes - off);
            bulk_g2s(dst + (half ? bytes : 0) + off, a.W + (int64_t(row) + (half ? a.pair_off : 0)) * a.row_bytes + off,
                     sz, &full[slot]);
        }
    }
    if (lane == 0)  // leave only when no copy of ours is still landing (a consumer may have given up)
        for (int s = st > nslot ? st - nslot : 0; s < st; s++) mbar_wait(&full[s % nslot], (s / nslot) & 1);
}

struct StreamPlan {
    int rows_per_cta;
    int rpw;         // rows per warp per stage (output rows; pairs for SwiGLU)
    int rps;         // rows per stage = kSW * rpw
    int nslot, slot_bytes, xs_bytes;
};

template <int FMT, int NM>
__global__ void __launch_bounds__(kSThr, 1) gemv_stream_kernel(const GemvArgs a, const StreamPlan sp) {
    constexpr int RR = kSRows<NM>;
    uint64_t* full = reinterpret_cast<uint64_t*>(gsm);
    uint64_t* empty = full + kSMaxSlots;
    float* xs = reinterpret_cast<float*>(gsm + kSHdr);
    uint8_t* ring = gsm + kSHdr + sp.xs_bytes;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const bool pair = a.pair_off != 0;
    const int r0 = blockIdx.x * sp.rows_per_cta, r1 = min(a.rows, r0 + sp.rows_per_cta);
    pdl_trigger();
    if (r0 >= r1) return;
    const int n = r1 - r0, rps = sp.rps, nst = (n + rps - 1) / rps;
    if (threadIdx.x == 0) {
        for (int s = 0; s < sp.nslot; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], kSW);
        }
        fence_barrier_init();
    }
    if (threadIdx.x < kDecodeMaxSeqs) tsh().key[threadIdx.x] = 0ull;
    __syncthreads();

    if (warp == kSW) {  // producer: weights only, so it never waits for the previous kernel
        stream_producer(a, r0, r1, sp.rps, sp.nslot, sp.slot_bytes, full, empty, ring, lane);
        return;
    }

    // ---------------- consumers
    pdl_wait();  // the activations come from the previous kernel
    stage_act<FMT>(a, xs, warp, lane);
    constexpr float kF = FMT == kFP8 ? kFp8HwFactor : kFp4Factor;
    const int cbytes = code_bytes(FMT, a.K), nseg = seg_count(FMT, a.K), xrow = nseg * Seg<FMT>::W;
    const int rpp = pair ? RR / 2 : RR;  // output rows a pass can take
    unsigned long long best[NM];
#pragma unroll
    for (int m = 0; m < NM; m++) best[m] = 0ull;
    int slot = 0, par = 0;
    for (int st = 0; st < nst; st++) {
        int ok = 1;
        if (lane == 0) ok = mbar_wait(&full[slot], par);
        ok = __shfl_sync(0xffffffffu, ok, 0);  // a wait that gave up is a device error; the stage is skipped
        const int srow = st * rps, in_stage = min(rps, n - srow);
        const uint8_t* base = ring + size_t(slot) * sp.slot_bytes;
        for (int q0 = warp; ok && q0 < in_stage; q0 += kSW * rpp) {  // one pass unless rpw > rpp
            const uint8_t* wr[RR];
            int nr = 0;
#pragma unroll
            for (int r = 0; r < RR; r++) {
                if (r >= rpp) break;
                const int q = q0 + r * kSW;
                if (q < in_stage && r < sp.rpw) {
                    wr[r] = base + int64_t(q) * a.row_bytes;
                    if (pair) wr[rpp + r] = base + int64_t(in_stage + q) * a.row_bytes;
                    nr = r + 1;
                } else {  // no row: repeat row 0 (never used) so every load of the pass is unconditional
                    wr[r] = wr[0];
                    if (pair) wr[rpp + r] = wr[rpp];
                }
            }
            const int nrows = pair ? rpp + nr : nr;
            float acc[RR][NM];
            dot_rows<FMT, NM, RR>(wr, nrows, cbytes, nseg, xs, xrow, a.M, lane, acc);
            float red_[RR][NM];
            if constexpr (RR == 4 && NM == 1) {
                // four rows at once: halves exchange rows (0,1) / (2,3), then quarters, then three xor steps;
                // lane 8 q ends up with row q
                const bool h16 = lane & 16, h8 = lane & 8;
                float v0 = h16 ? acc[2][0] : acc[0][0], v1 = h16 ? acc[3][0] : acc[1][0];
                v0 += __shfl_xor_sync(0xffffffffu, h16 ? acc[0][0] : acc[2][0], 16);
                v1 += __shfl_xor_sync(0xffffffffu, h16 ? acc[1][0] : acc[3][0], 16);
                float t = h8 ? v1 : v0;
                t += __shfl_xor_sync(0xffffffffu, h8 ? v0 : v1, 8);
                t += __shfl_xor_sync(0xffffffffu, t, 4);
                t += __shfl_xor_sync(0xffffffffu, t, 2);
                t += __shfl_xor_sync(0xffffffffu, t, 1);
#pragma unroll
                for (int r = 0; r < 4; r++) red_[r][0] = __shfl_sync(0xffffffffu, t, 8 * r) * kF;
            } else {
#pragma unroll
                for (int r = 0; r < RR; r++)
#pragma unroll
                    for (int m = 0; m < NM; m++)
                        red_[r][m] = (r < nrows && m < a.M) ? warp_sum(acc[r][m]) * kF : 0.0f;
            }
#pragma unroll
            for (int r = 0; r < RR; r++) {
                if (r >= rpp) break;
#pragma unroll
                for (int m = 0; m < NM; m++) {
                    if (m >= a.M) break;
                    if (r >= nr || lane != ((r * NM + m) & 31)) continue;
                    const int row = r0 + srow + q0 + r * kSW;
                    float* dst = a.y + int64_t(m) * a.y_stride + a.n_off + row;
                    const float gs = red_[r][m];
                    float val;
                    if (pair) {
                        const float us = red_[rpp + r < RR ? rpp + r : 0][m];
                        val = gs / (1.0f + expf(-gs)) * us;  // cpu::siluMul (cpu_ops.cpp:526-533)
                    } else {
                        val = gs;
                        if (a.flags & kBias) val += a.bias[row];
                        if (a.flags & kGelu) val = gelu(val);
                        if (a.flags & kAccumulate) val += *dst;
                    }
                    *dst = val;
                    if (a.argmax) best[m] = max(best[m], argmax_key(val, row));
                }
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[slot]);
        if (++slot == sp.nslot) {
            slot = 0;
            par ^= 1;
        }
    }
    if (a.argmax) {  // per warp, then one global atomic per CTA and activation row
#pragma unroll
        for (int m = 0; m < NM; m++) {
            if (m >= a.M) break;
            unsigned long long k = best[m];
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) k = max(k, __shfl_xor_sync(0xffffffffu, k, o));
            if (lane == 0 && k) atomicMax(&tsh().key[m], k);
        }
        ssync();
        if (threadIdx.x < a.M && tsh().key[threadIdx.x]) atomicMax(a.argmax + threadIdx.x, tsh().key[threadIdx.x]);
    }
}

// ------------------------------------------------------------------------------------------------ tensor cores
// The same stream of weight rows with the dot products on mma.sync m16n8k16 (f16 operands, fp32 accumulation):
// D[m][n] = sum_k x[m][k] w[n][k] with the 1..4 activation rows as M (rows 4..15 zero) and 8 weight rows as N.
// K is permuted inside each 16-step so that lane (g, c) reads 4 contiguous code bytes of weight row g (bytes 4c..
// 4c+3 of the step, MMA k = 2c, 2c+1, 2c+8, 2c+9) and the same 4 activations: one 32-bit load and two hardware
// conversions feed two MMAs (the activations as hi + lo f16, about 22 bits). Codes are exact in f16; each 32-weight
// block's partial sums are scaled in fp32, as in the CUDA-core kernel.
//  * the producer copies each row into the stage at a pitch of rowBytes + 16, so the 8 rows' 4-byte loads of a
//    warp fall on 32 different banks (at the packed pitch, 1088 bytes for K = 1024, half the rows share banks);
//  * a stage holds T tiles of 8 rows; G groups of T consumer warps (G T <= 16) take stages round-robin, group q
//    stages q, q + G, ..., and warp w of a group a whole tile (all of K): no reduction across warps. The ring has
//    a multiple of G slots, so each slot belongs to one group, which waits on its phases in order (an mbarrier
//    parity wait is only unambiguous for a waiter at most one phase ahead of the barrier).
// About 0.09 warp instructions per FP8 weight against ~0.19 on CUDA cores; the per-row copies cost more than
// that saves at one activation row, so it takes 2..4.
struct MmaPlan {
    int rows_per_cta;
    int tiles;       // 8-row tiles per stage = warps per group
    int groups;      // warp groups taking stages (groups x tiles <= 16 consumer warps; the rest idle)
    int rps;         // rows per stage = 8 tiles
    int pitch;       // bytes per row in a stage (row_bytes + 16)
    int nslot, slot_bytes, xs_bytes;
};

// The M activation rows as f16 hi / lo ([M][K] each), with the norm prologue (sums in double, cpu_ops.cpp:
// 483-511), read straight from global memory (a few KB, L2-resident).
__device__ void stage_act_hilo(const GemvArgs& a, __half* xh, __half* xl, int warp, int lane) {
    const int tid = threadIdx.x, K4 = a.K / 4, total = a.M * K4;
    float r[kDecodeMaxSeqs], mean[kDecodeMaxSeqs];
    if (a.norm != kNormNone) {
        double s1[kDecodeMaxSeqs] = {0.0, 0.0, 0.0, 0.0}, s2[kDecodeMaxSeqs] = {0.0, 0.0, 0.0, 0.0};
        for (int i = tid; i < total; i += kSNT) {
            const int m = i / K4, k = 4 * (i - m * K4);
            const float4 v = *reinterpret_cast<const float4*>(a.x + int64_t(m) * a.x_stride + k);
#pragma unroll
            for (int mm = 0; mm < kDecodeMaxSeqs; mm++)
                if (mm == m) {
                    s1[mm] += double(v.x) + double(v.y) + double(v.z) + double(v.w);
                    s2[mm] += double(v.x) * v.x + double(v.y) * v.y + double(v.z) * v.z + double(v.w) * v.w;
                }
        }
#pragma unroll
        for (int m = 0; m < kDecodeMaxSeqs; m++) {
            const double t1 = wsum_d(s1[m]), t2 = wsum_d(s2[m]);
            if (lane == 0) {
                tsh().part[2 * (m * kSW + warp)] = t1;
                tsh().part[2 * (m * kSW + warp) + 1] = t2;
            }
        }
        ssync();
#pragma unroll
        for (int m = 0; m < kDecodeMaxSeqs; m++) {
            double a1 = 0.0, a2 = 0.0;
            for (int w = 0; w < kSW; w++) {
                a1 += tsh().part[2 * (m * kSW + w)];
                a2 += tsh().part[2 * (m * kSW + w) + 1];
            }
            mean[m] = 0.0f;
            if (a.norm == kNormRms) {
                r[m] = float(1.0 / sqrt(a2 / a.K + double(a.eps)));
            } else {
                const double mu = a1 / a.K;
                mean[m] = float(mu);
                r[m] = float(1.0 / sqrt(a2 / a.K - mu * mu + double(a.eps)));
            }
        }
    }
    for (int i = tid; i < total; i += kSNT) {
        const int m = i / K4, k = 4 * (i - m * K4);
        float4 y = *reinterpret_cast<const float4*>(a.x + int64_t(m) * a.x_stride + k);
        if (a.norm != kNormNone) {
            float rm = r[0], mm = mean[0];
#pragma unroll
            for (int q = 1; q < kDecodeMaxSeqs; q++)
                if (q == m) {
                    rm = r[q];
                    mm = mean[q];
                }
            const float4 ga = __ldg(reinterpret_cast<const float4*>(a.gamma + k));
            if (a.norm == kNormRms) {
                y.x = __fmul_rn(__fmul_rn(y.x, rm), ga.x);
                y.y = __fmul_rn(__fmul_rn(y.y, rm), ga.y);
                y.z = __fmul_rn(__fmul_rn(y.z, rm), ga.z);
                y.w = __fmul_rn(__fmul_rn(y.w, rm), ga.w);
            } else {
                const float4 be = __ldg(reinterpret_cast<const float4*>(a.beta + k));
                y.x = __fadd_rn(__fmul_rn(__fmul_rn(__fsub_rn(y.x, mm), rm), ga.x), be.x);
                y.y = __fadd_rn(__fmul_rn(__fmul_rn(__fsub_rn(y.y, mm), rm), ga.y), be.y);
                y.z = __fadd_rn(__fmul_rn(__fmul_rn(__fsub_rn(y.z, mm), rm), ga.z), be.z);
                y.w = __fadd_rn(__fmul_rn(__fmul_rn(__fsub_rn(y.w, mm), rm), ga.w), be.w);
            }
        }
        uint32_t h0, l0, h1, l1;
        split_hilo(y.x, y.y, h0, l0);
        split_hilo(y.z, y.w, h1, l1);
        *reinterpret_cast<uint2*>(xh + m * a.K + k) = make_uint2(h0, h1);
        *reinterpret_cast<uint2*>(xl + m * a.K + k) = make_uint2(l0, l1);
    }
    ssync();
}

// The producer of the tensor-core kernel: stage s = rows r0 + s rps .. (SwiGLU: the gate rows, then the up rows),
// one bulk copy per row into a row pitch of sp.pitch bytes.
__device__ void stream_producer_rows(const GemvArgs& a, int r0, int r1, const MmaPlan& sp, uint64_t* full,
                                     uint64_t* empty, uint8_t* ring, int lane) {
    const bool pair = a.pair_off != 0;
    const int nst = (r1 - r0 + sp.rps - 1) / sp.rps;
    int st = 0;
    for (; st < nst; st++) {
        const int slot = st % sp.nslot;
        if (st >= sp.nslot) {
            int ok = 1;
            if (lane == 0) ok = mbar_wait(&empty[slot], ((st / sp.nslot) - 1) & 1);
            if (!__shfl_sync(0xffffffffu, ok, 0)) break;
        }
        const int row = r0 + st * sp.rps, cnt = min(sp.rps, r1 - row);
        uint8_t* dst = ring + size_t(slot) * sp.slot_bytes;
        if (lane == 0) mbar_arrive_expect_tx(&full[slot], uint32_t((pair ? 2 : 1) * cnt) * uint32_t(a.row_bytes));
        __syncwarp();
        for (int c = lane; c < (pair ? 2 : 1) * cnt; c += 32) {
            const int half = c >= cnt ? 1 : 0, r = c - half * cnt;
            bulk_g2s(dst + size_t(half * sp.rps + r) * sp.pitch,
                     a.W + (int64_t(row + r) + (half ? a.pair_off : 0)) * a.row_bytes, uint32_t(a.row_bytes),
                     &full[slot]);
        }
    }
    if (lane == 0)  // leave only when no copy of ours is still landing (a consumer may have given up)
        for (int s = st > sp.nslot ? st - sp.nslot : 0; s < st; s++) mbar_wait(&full[s % sp.nslot], (s / sp.nslot) & 1);
}

template <int FMT>
__global__ void __launch_bounds__(kSThr, 1) gemv_mma_kernel(const GemvArgs a, const MmaPlan sp) {
    uint64_t* full = reinterpret_cast<uint64_t*>(gsm);
    uint64_t* empty = full + kSMaxSlots;
    __half* xh = reinterpret_cast<__half*>(gsm + kSHdr);
    __half* xl = xh + a.M * a.K;
    uint8_t* ring = gsm + kSHdr + sp.xs_bytes;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, c = lane & 3;
    const bool pair = a.pair_off != 0;
    const int r0 = blockIdx.x * sp.rows_per_cta, r1 = min(a.rows, r0 + sp.rows_per_cta);
    pdl_trigger();
    if (r0 >= r1) return;
    const int n = r1 - r0, rps = sp.rps, nst = (n + rps - 1) / rps;
    const int T = sp.tiles, ngroups = sp.groups;
    if (threadIdx.x == 0) {
        for (int s = 0; s < sp.nslot; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], T);  // the T warps of the group that takes the stage
        }
        fence_barrier_init();
    }
    if (threadIdx.x < kDecodeMaxSeqs) tsh().key[threadIdx.x] = 0ull;
    __syncthreads();
    if (warp == kSW) {  // producer: weights only, so it never waits for the previous kernel
        stream_producer_rows(a, r0, r1, sp, full, empty, ring, lane);
        return;
    }

    // ---------------- consumers
    pdl_wait();  // the activations come from the previous kernel
    stage_act_hilo(a, xh, xl, warp, lane);
    constexpr float kF = FMT == kFP8 ? kFp8HwFactor : kFp4Factor;
    const int cbytes = code_bytes(FMT, a.K), nblk = a.K / kQuantBlock;
    const int group = warp / T, tile = warp % T;  // warps of group >= ngroups take no stage
    const bool xrow = g < a.M;  // this lane's activation row exists (MMA rows past M stay zero)
    const __half* xhr = xh + (xrow ? g : 0) * a.K + 4 * c;
    const __half* xlr = xl + (xrow ? g : 0) * a.K + 4 * c;
    unsigned long long best = 0ull;  // this lane's activation row g
    for (int st = group; group < ngroups && st < nst; st += ngroups) {
        const int slot = st % sp.nslot;
        int ok = 1;
        if (lane == 0) ok = mbar_wait(&full[slot], uint32_t(st / sp.nslot) & 1u);
        ok = __shfl_sync(0xffffffffu, ok, 0);  // a wait that gave up is a device error; the stage is skipped
        const int srow = st * rps, in_stage = min(rps, n - srow);
        const uint8_t* base = ring + size_t(slot) * sp.slot_bytes;
        // this lane's weight row (B operand) and the two rows whose outputs it holds (D columns 2c, 2c + 1)
        const int qb = min(8 * tile + g, in_stage - 1);
        const uint8_t* wb = base + size_t(qb) * sp.pitch;
        const uint8_t* wu = base + size_t(rps + qb) * sp.pitch;  // up row (SwiGLU)
        const int qd0 = min(8 * tile + 2 * c, in_stage - 1), qd1 = min(8 * tile + 2 * c + 1, in_stage - 1);
        const uint16_t* sc0 = reinterpret_cast<const uint16_t*>(base + size_t(qd0) * sp.pitch + cbytes);
        const uint16_t* sc1 = reinterpret_cast<const uint16_t*>(base + size_t(qd1) * sp.pitch + cbytes);
        const uint16_t* su0 = reinterpret_cast<const uint16_t*>(base + size_t(rps + qd0) * sp.pitch + cbytes);
        const uint16_t* su1 = reinterpret_cast<const uint16_t*>(base + size_t(rps + qd1) * sp.pitch + cbytes);
        float acc[2][2] = {{0.0f, 0.0f}, {0.0f, 0.0f}};  // [gate | up][column 2c + e]
        if (ok && 8 * tile < in_stage) {
#pragma unroll 2
            for (int b = 0; b < nblk; b++) {
                uint32_t ah0[4] = {0u, 0u, 0u, 0u}, al0[4] = {0u, 0u, 0u, 0u}, ah1[4] = {0u, 0u, 0u, 0u},
                         al1[4] = {0u, 0u, 0u, 0u};
                if (xrow) {  // steps 2b (weights 32b + 4c ..) and 2b + 1 (32b + 16 + 4c ..)
                    const uint2 h0 = *reinterpret_cast<const uint2*>(xhr + 32 * b);
                    const uint2 l0 = *reinterpret_cast<const uint2*>(xlr + 32 * b);
                    const uint2 h1 = *reinterpret_cast<const uint2*>(xhr + 32 * b + 16);
                    const uint2 l1 = *reinterpret_cast<const uint2*>(xlr + 32 * b + 16);
                    ah0[0] = h0.x, ah0[2] = h0.y, al0[0] = l0.x, al0[2] = l0.y;
                    ah1[0] = h1.x, ah1[2] = h1.y, al1[0] = l1.x, al1[2] = l1.y;
                }
#pragma unroll
                for (int u = 0; u < 2; u++) {  // gate (or the only) row, then the up row
                    if (u == 1 && !pair) break;
                    const uint8_t* w = u ? wu : wb;
                    uint32_t b00, b01, b10, b11;  // step 0: (b00, b01), step 1: (b10, b11)
                    if (FMT == kFP8) {
                        __half2 p0, p1, p2, p3;
                        e4m3x4_to_half2(*reinterpret_cast<const uint32_t*>(w + 32 * b + 4 * c), p0, p1);
                        e4m3x4_to_half2(*reinterpret_cast<const uint32_t*>(w + 32 * b + 16 + 4 * c), p2, p3);
                        b00 = h2u(p0), b01 = h2u(p1), b10 = h2u(p2), b11 = h2u(p3);
                    } else {  // bytes 4c..4c+3 of the block: low nibbles = weights 4c.., high = 16 + 4c..
                        const uint32_t wd = *reinterpret_cast<const uint32_t*>(w + 16 * b + 4 * c);
                        const __half2 e0 = fp4x2_to_half2(wd & 0x000F000Fu), o0 = fp4x2_to_half2((wd >> 8) & 0x000F000Fu);
                        const __half2 e1 = fp4x2_to_half2((wd >> 4) & 0x000F000Fu);
                        const __half2 o1 = fp4x2_to_half2((wd >> 12) & 0x000F000Fu);
                        b00 = h2u(__halves2half2(__low2half(e0), __low2half(o0)));
                        b01 = h2u(__halves2half2(__high2half(e0), __high2half(o0)));
                        b10 = h2u(__halves2half2(__low2half(e1), __low2half(o1)));
                        b11 = h2u(__halves2half2(__high2half(e1), __high2half(o1)));
                    }
                    float d[4], dl[4];
                    mma16816_z(d, ah0, b00, b01);
                    mma16816_z(dl, al0, b00, b01);
                    mma16816(d, ah1, b10, b11);
                    mma16816(dl, al1, b10, b11);
                    const uint16_t* s0 = u ? su0 : sc0;
                    const uint16_t* s1 = u ? su1 : sc1;
                    acc[u][0] = fmaf(half_bits_to_float(s0[b]) * kF, d[0] + dl[0], acc[u][0]);
                    acc[u][1] = fmaf(half_bits_to_float(s1[b]) * kF, d[1] + dl[1], acc[u][1]);
                }
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[slot]);  // the stage's weights are no longer read by this warp
        if (ok) {
#pragma unroll
            for (int e = 0; e < 2; e++) {
                const int q = 8 * tile + 2 * c + e;
                if (!xrow || q >= in_stage) continue;
                const int row = r0 + srow + q, m = g;
                float* dst = a.y + int64_t(m) * a.y_stride + a.n_off + row;
                float val;
                if (pair) {
                    const float gs = acc[0][e], us = acc[1][e];
                    val = gs / (1.0f + expf(-gs)) * us;  // cpu::siluMul (cpu_ops.cpp:526-533)
                } else {
                    val = acc[0][e];
                    if (a.flags & kBias) val += a.bias[row];
                    if (a.flags & kGelu) val = gelu(val);
                    if (a.flags & kAccumulate) val += *dst;
                }
                *dst = val;
                if (a.argmax) best = max(best, argmax_key(val, row));
            }
        }
    }
    if (a.argmax) {  // the 4 lanes of each activation row, then per CTA, then one global atomic per row
        best = max(best, __shfl_xor_sync(0xffffffffu, best, 1));
        best = max(best, __shfl_xor_sync(0xffffffffu, best, 2));
        if (c == 0 && xrow && best) atomicMax(&tsh().key[g], best);
        ssync();
        if (threadIdx.x < a.M && tsh().key[threadIdx.x]) atomicMax(a.argmax + threadIdx.x, tsh().key[threadIdx.x]);
    }
}

using StreamFn = void (*)(const GemvArgs, const StreamPlan);

StreamFn pick(int fmt, int M) {
    if (fmt == kFP8) return M == 1 ? gemv_stream_kernel<kFP8, 1> : gemv_stream_kernel<kFP8, kDecodeMaxSeqs>;
    return M == 1 ? gemv_stream_kernel<kFP4, 1> : gemv_stream_kernel<kFP4, kDecodeMaxSeqs>;
}

}  // namespace

// The tensor-core streaming kernel: activations as hi / lo f16 in shared memory (<= 64 KB), rows at a padded
// pitch, stages of 8 T rows (T in 4, 2, 1, at most the CTA's rows rounded up to a tile), G groups with one or
// two ring slots each: the plan with the most busy warps (G T), then two slots per group, then the larger T.
cudaError_t launch_gemv_mma(const GemvArgs& a, cudaStream_t st, bool pdl) {
    const int64_t xs = (int64_t(a.M) * a.K * 4 + 127) / 128 * 128;
    if (xs > 64 * 1024 || a.K % kQuantBlock) return cudaErrorNotSupported;
    MmaPlan sp;
    const int sms = num_sms();
    int ctas = std::max(1, std::min(sms, (a.rows + 3) / 4));
    sp.rows_per_cta = (a.rows + ctas - 1) / ctas;
    ctas = (a.rows + sp.rows_per_cta - 1) / sp.rows_per_cta;
    sp.xs_bytes = int(xs);
    sp.pitch = int(a.row_bytes) + 16;
    auto k = a.fmt == kFP8 ? gemv_mma_kernel<kFP8> : gemv_mma_kernel<kFP4>;
    const int64_t budget = int64_t(max_dyn_smem(k)) - kSHdr - xs;
    const int tneed = (sp.rows_per_cta + 7) / 8;
    sp.tiles = 0;
    int best = -1;
    for (int t = 4; t >= 1; t /= 2) {
        if (t > tneed && t > 1) continue;
        const int64_t sb = (int64_t(8 * t) * sp.pitch * (a.pair_off ? 2 : 1) + 127) / 128 * 128;
        const int slots = int(std::min<int64_t>(kSMaxSlots, budget / sb));
        for (int per_group : {2, 1}) {
            const int g = std::min(kSW / t, slots / per_group);
            if (g < 1) continue;
            const int score = (g * t) * 8 + per_group * 4 + t;  // busy warps, then slots per group, then T
            if (score > best) {
                best = score;
                sp.tiles = t;
                sp.groups = g;
                sp.slot_bytes = int(sb);
                sp.nslot = g * per_group;
            }
        }
    }
    if (!sp.tiles || sp.groups * sp.tiles < kSW / 2) return cudaErrorNotSupported;  // too few busy warps
    sp.rps = 8 * sp.tiles;
    const size_t smem = kSHdr + size_t(xs) + size_t(sp.nslot) * sp.slot_bytes;
    if (const cudaError_t e = ensure_dyn_smem(k, smem); e != cudaSuccess) return e;
    return launch_ex(k, dim3(ctas), dim3(kSThr), smem, st, pdl, a, sp);
}

// The streaming kernel takes the call when it fits: 1..4 FP8 / FP4 activation rows, activations (padded) in
// 64 KB of shared memory, a ring of at least the stages a pass can span. Returns cudaErrorNotSupported (and
// launches nothing) otherwise, so the caller falls back to the general kernel. The tensor-core variant runs
// when it fits; the CUDA-core one otherwise.
cudaError_t launch_gemv_stream(const GemvArgs& a, cudaStream_t st, bool pdl) {
    if (a.M < 1 || a.M > kDecodeMaxSeqs || (a.fmt != kFP8 && a.fmt != kFP4)) return cudaErrorNotSupported;
    // FP8: the direct-load tensor-core kernel (k_gemv_fp8tc.cu) when it fits (any norm width: it reads the
    // activations from global memory)
    if (a.fmt == kFP8)
        if (const cudaError_t e = launch_gemv_fp8_tc(a, st, pdl); e != cudaErrorNotSupported) return e;
    if (a.x_stride % 4 || (reinterpret_cast<uintptr_t>(a.x) & 15) || a.K % 4) return cudaErrorNotSupported;
    if (a.argmax && a.pair_off) return cudaErrorNotSupported;
    const int64_t xs = (gemv_x_bytes(a.fmt, a.M, a.K) + 127) / 128 * 128;
    if (xs > 64 * 1024) return cudaErrorNotSupported;
    if (a.norm != kNormNone && !gemv_norm_fusable(a.fmt, a.M, a.K)) return cudaErrorNotSupported;
    const int64_t rbe = a.row_bytes * (a.pair_off ? 2 : 1);
    if (a.row_bytes % 16) return cudaErrorNotSupported;
    // the f16 tensor-core variant for 2..4 rows (one row: the CUDA-core kernel is faster, 54 vs 73 us at the
    // LM-head shape, where this variant's one bulk copy per row limits the stream)
    if (a.M >= 2)
        if (const cudaError_t e = launch_gemv_mma(a, st, pdl); e != cudaErrorNotSupported) return e;
    StreamPlan sp;
    const int sms = num_sms();
    int ctas = std::max(1, std::min(sms, (a.rows + 3) / 4));
    sp.rows_per_cta = (a.rows + ctas - 1) / ctas;
    ctas = (a.rows + sp.rows_per_cta - 1) / sp.rows_per_cta;
    sp.xs_bytes = int(xs);
    StreamFn k = pick(a.fmt, a.M);
    const int64_t budget = int64_t(max_dyn_smem(k)) - kSHdr - xs;
    // Stage = kSW x rpw rows: the most rows per warp (up to what a pass takes) that still leaves a ring of
    // at least four stages (three, then two, for very wide rows).
    const int rpp = (a.M == 1 ? 4 : 2) / (a.pair_off ? 2 : 1);
    sp.rpw = 0;
    for (int want : {4, 3, 2}) {
        for (int rpw = rpp; rpw >= 1 && !sp.rpw; rpw--) {
            const int64_t sb = (int64_t(kSW) * rpw * rbe + 127) / 128 * 128;
            if (budget / sb >= want) {
                sp.rpw = rpw;
                sp.slot_bytes = int(sb);
            }
        }
        if (sp.rpw) break;
    }
    if (!sp.rpw) return cudaErrorNotSupported;
    sp.rps = kSW * sp.rpw;
    sp.nslot = int(std::min<int64_t>(kSMaxSlots, budget / sp.slot_bytes));
    const size_t smem = kSHdr + size_t(xs) + size_t(sp.nslot) * sp.slot_bytes;
    if (const cudaError_t e = ensure_dyn_smem(k, smem); e != cudaSuccess) return e;
    return launch_ex(k, dim3(ctas), dim3(kSThr), smem, st, pdl, a, sp);
}

}  // namespace neko
