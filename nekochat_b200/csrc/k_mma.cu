// Tensor-core dequant matmul for 5..64+ activation rows (prefill chunks, batched decode): the MatmulQ8 /
// MatmulQ4 dispatch (matmul_q8.comp, matmul_q4.comp; cpu::matmul, cpu_ops.cpp:462-481) when the multiply-adds,
// not the weight bytes, are the cost (from M = 8 the CUDA-core GEMV is compute bound at 2-4 TFLOP/s).
//
// y[m][n] (+)= act(x[m] . deq(W[n]) + b[n]) on mma.sync m16n8k16 (f16 operands, fp32 accumulation), with the
// precision of the fp32 kernels:
//  * weights enter as their codes, exactly: an e4m3 code (hardware e4m3 -> f16 conversion) or an e2m1 nibble
//    (bit arithmetic) is exactly representable in f16; each 32-weight block's f16 scale is applied in fp32 to
//    that block's partial sums (two k16 steps), as dequantizeRow multiplies code by scale in fp32;
//  * activations are split x = hi + lo into two f16 (round to nearest, then the rounding error rounded again):
//    two MMAs per step, about 22 bits of each activation kept (fp32 has 24), products exact in fp32;
//  * CTA tile: 64 activation rows x 64 weight rows (SwiGLU: 32 gate + 32 up rows); K walked in stages of 64
//    through a 4-deep cp.async pipeline; per stage the CTA converts the codes once into padded shared memory;
//    8 warps: warp w owns activation rows 16(w % 4)..+15 and weight rows 32(w / 4)..+31 of the tile (warps
//    without activation rows skip the math), ldmatrix.x4 fragments; two warps per scheduler per CTA and two
//    CTAs per SM hide the MMA and shared-memory latencies;
//  * when the tiles alone leave SMs idle, K is split over a thread-block cluster of up to 8 CTAs: each leaves
//    its fp32 partial tile in its own shared memory, and after a cluster barrier CTA z sums rows z, z + ks, ...
//    of the tile over the cluster's shared memory (distributed shared memory) in split order 0, 1, ...
//    (deterministic) and runs the epilogue for them;
//  * when 8+ tiles share the activations, one small kernel splits them into hi / lo f16 first, and the stages
//    copy those straight into the padded tiles (otherwise every CTA splits its own fp32 copy).
// Activations must stay within the f16 range (|x| < 65504), which the matmul inputs of the models are
// (normalised activations, attention outputs, SwiGLU products).
#include <cooperative_groups.h>

#include <algorithm>
#include <cstdlib>
#include <type_traits>

#include "gemv_core.cuh"
#include "mma_frag.cuh"
#include "neko_common.cuh"
#include "neko_internal.h"

namespace neko {

namespace {

constexpr int kTM = 64;        // activation rows per CTA
constexpr int kTK = 64;        // K per stage
constexpr int kTP = kTK + 8;   // padded row pitch of the converted tiles (halves): ldmatrix without conflicts
constexpr int kTThreads = 256;
constexpr int kTStages = 4;   // cp.async pipeline depth

// Raw stage: W codes [BNW][kTK] (FP8 bytes / FP4 kTK / 2 bytes), scales [BNW][2] f16, and the activations:
// fp32 [kTM][kTK], or (split once per matmul beforehand) f16 hi and lo [2][kTM][kTP] read by ldmatrix in place.
struct XsF32 {
    float v[kTM][kTK];
};
struct XsHiLo {
    __half v[2][kTM][kTP];
};
template <int FMT, int BNW, bool PRE>
struct Stage {
    static constexpr int kCode = FMT == kFP8 ? kTK : kTK / 2;
    uint8_t w[BNW][kCode];
    uint16_t sc[BNW][2];
    typename std::conditional<PRE, XsHiLo, XsF32>::type x;
};

constexpr int kTMaxSplit = 8;  // CTAs of a cluster (portable limit)

// How a launch divides K and where its activations come from.
struct TcSplit {
    int ksplit;              // CTAs along K = the cluster's size; partial tiles summed over distributed smem
    int sper;                // K stages per split
    const __half* xh;        // activations split into f16 hi / lo ([M][K] each), or null: split per stage
    const __half* xl;
};

// x = hi + lo, both f16 (round to nearest): once per matmul when many CTAs read the same activations.
__global__ void split_act_kernel(const float* __restrict__ x, int64_t x_stride, int M, int K, __half* __restrict__ xh,
                                 __half* __restrict__ xl) {
    pdl_wait();
    const int64_t n = int64_t(M) * (K / 4);
    for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < n; i += int64_t(gridDim.x) * blockDim.x) {
        const int m = int(i / (K / 4)), k = 4 * int(i - int64_t(m) * (K / 4));
        const float4 v = *reinterpret_cast<const float4*>(x + int64_t(m) * x_stride + k);
        const __half2 h01 = __floats2half2_rn(v.x, v.y), h23 = __floats2half2_rn(v.z, v.w);
        const float2 f01 = __half22float2(h01), f23 = __half22float2(h23);
        const int64_t o = int64_t(m) * K + k;
        *reinterpret_cast<uint2*>(xh + o) = make_uint2(h2u(h01), h2u(h23));
        *reinterpret_cast<uint2*>(xl + o) = make_uint2(h2u(__floats2half2_rn(v.x - f01.x, v.y - f01.y)),
                                                       h2u(__floats2half2_rn(v.z - f23.x, v.w - f23.y)));
    }
    pdl_trigger();
}

// RMSNorm / LayerNorm of each activation row (norm_kernel's arithmetic: sums in double, cpu_ops.cpp:483-511),
// written as hi / lo f16 for the matmul: one CTA per row, the row read once into shared memory.
constexpr int kNsThreads = 256;
constexpr int kNsMaxK = 10240;  // row cached in static shared memory (40 KB)
__global__ void __launch_bounds__(kNsThreads) norm_split_kernel(const GemvArgs a, __half* __restrict__ xh,
                                                                __half* __restrict__ xl) {
    __shared__ float row[kNsMaxK];
    __shared__ double red[kNsThreads / 32];
    pdl_wait();
    const float* xr = a.x + int64_t(blockIdx.x) * a.x_stride;
    const int K = a.K;
    auto block_sum = [&](double v) {
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
        const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
        __syncthreads();
        if (l == 0) red[w] = v;
        __syncthreads();
        double t = l < kNsThreads / 32 ? red[l] : 0.0;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
        return t;
    };
    double s1 = 0.0, s2 = 0.0;
    for (int c = threadIdx.x; c < K; c += kNsThreads) {
        const float v = xr[c];
        row[c] = v;
        s1 += v;
        s2 += double(v) * v;
    }
    const bool rms = a.norm == kNormRms;
    float r, mean = 0.0f;
    if (rms) {
        r = float(1.0 / sqrt(block_sum(s2) / K + double(a.eps)));
    } else {
        const double mu = block_sum(s1) / K;
        double var = 0.0;
        for (int c = threadIdx.x; c < K; c += kNsThreads) {
            const double d = row[c] - mu;
            var += d * d;
        }
        r = float(1.0 / sqrt(block_sum(var) / K + double(a.eps)));
        mean = float(mu);
    }
    pdl_trigger();
    for (int c = 2 * threadIdx.x; c < K; c += 2 * kNsThreads) {
        float y[2];
#pragma unroll
        for (int e = 0; e < 2; e++) {
            const float v = row[c + e];
            y[e] = rms ? __fmul_rn(__fmul_rn(v, r), a.gamma[c + e])
                       : __fadd_rn(__fmul_rn(__fmul_rn(__fsub_rn(v, mean), r), a.gamma[c + e]), a.beta[c + e]);
        }
        uint32_t hi, lo;
        split_hilo(y[0], y[1], hi, lo);
        const int64_t o = int64_t(blockIdx.x) * K + c;
        *reinterpret_cast<uint32_t*>(xh + o) = hi;
        *reinterpret_cast<uint32_t*>(xl + o) = lo;
    }
}

template <int FMT, int BN, bool PAIR, bool PRE>
__global__ void __launch_bounds__(kTThreads, 2) tc_gemm_kernel(const GemvArgs a, const TcSplit sp) {
    constexpr int BNW = PAIR ? 2 * BN : BN;  // weight rows per CTA
    constexpr int NT = BNW / 16;             // n8 tiles per warp (half of the tile's columns)
    using St = Stage<FMT, BNW, PRE>;
    extern __shared__ __align__(128) uint8_t tsm[];
    St* raw = reinterpret_cast<St*>(tsm);                                        // [kTStages]
    __half* wh = reinterpret_cast<__half*>(tsm + kTStages * sizeof(St));         // [BNW][kTP] codes
    __half* xhi = wh + BNW * kTP;                                                // [kTM][kTP] (!PRE)
    __half* xlo = xhi + kTM * kTP;                                               // [kTM][kTP] (!PRE)
    float* scs = reinterpret_cast<float*>(PRE ? xhi : xlo + kTM * kTP);         // [2][BNW] block scales
    __shared__ unsigned long long keys[kTM];

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int wm = warp & 3, wn = warp >> 2;  // activation rows 16 wm.., weight rows (columns) 8 NT wn..
    const int n0 = blockIdx.x * BN, m0 = blockIdx.y * kTM, z = blockIdx.z;
    const int mv = min(kTM, a.M - m0);  // activation rows of this tile
    const int cbytes = FMT == kFP8 ? a.K : a.K / 2;
    const int s_begin = z * sp.sper, s_end = min(a.K / kTK, s_begin + sp.sper), nst = s_end - s_begin;
    constexpr float kCodeFactor = FMT == kFP8 ? kFp8HwFactor : kFp4Factor;  // code value -> engine decode
    if (a.argmax && tid < kTM) keys[tid] = 0ull;

    // weight row r of the tile -> packed row in W (rows past the end repeat the last row; never stored)
    auto wrow = [&](int r) -> const uint8_t* {
        const int n = PAIR ? (r < BN ? n0 + r : n0 + (r - BN)) : n0 + r;
        const int nc = min(n, a.rows - 1);
        return a.W + (int64_t(nc) + (PAIR && r >= BN ? a.pair_off : 0)) * a.row_bytes;
    };
    auto issue_w = [&](int i_s) {  // weights and scales of stage i_s (an index within this CTA's range)
        St& S = raw[i_s % kTStages];
        const int s = s_begin + i_s;
        constexpr int kPieces = St::kCode / 16;  // 16-byte pieces of codes per row
        for (int i = tid; i < BNW * kPieces; i += kTThreads) {
            const int r = i / kPieces, q = i - r * kPieces;
            cp16(&S.w[r][16 * q], wrow(r) + s * St::kCode + 16 * q, 16);
        }
        for (int r = tid; r < BNW; r += kTThreads) cp4(&S.sc[r][0], wrow(r) + cbytes + 4 * s);
    };
    auto issue_x = [&](int i_s) {  // activations of stage i_s
        St& S = raw[i_s % kTStages];
        const int s = s_begin + i_s;
        if constexpr (PRE) {  // hi / lo halves straight into their padded tiles
            for (int i = tid; i < 2 * mv * (kTK / 8); i += kTThreads) {
                const int h = i >= mv * (kTK / 8) ? 1 : 0, j = i - h * mv * (kTK / 8);
                const int m = j / (kTK / 8), q = j - m * (kTK / 8);
                cp16(&S.x.v[h][m][8 * q], (h ? sp.xl : sp.xh) + int64_t(m0 + m) * a.K + s * kTK + 8 * q, 16);
            }
        } else {
            for (int i = tid; i < mv * (kTK / 4); i += kTThreads) {
                const int m = i / (kTK / 4), q = i - m * (kTK / 4);
                cp16(&S.x.v[m][4 * q], a.x + int64_t(m0 + m) * a.x_stride + s * kTK + 4 * q, 16);
            }
        }
    };

    float acc[NT][4];
#pragma unroll
    for (int t = 0; t < NT; t++) acc[t][0] = acc[t][1] = acc[t][2] = acc[t][3] = 0.0f;

    // Prologue: the weights of the first stages (one group each) stream before the wait for the previous kernel
    // (weights never depend on it), then their activations (one group).
#pragma unroll
    for (int s = 0; s < kTStages - 1; s++) {
        if (s < nst) issue_w(s);
        cp_commit();
    }
    pdl_wait();
#pragma unroll
    for (int s = 0; s < kTStages - 1; s++) {  // one group per stage, so stage 0 waits for its own activations only
        if (s < nst) issue_x(s);
        cp_commit();
    }
    for (int s = 0; s < nst; s++) {
        // stage s landed (this thread's copies): groups are the prologue's weights of stages 0..2, their
        // activations one group each, then one group per stage issued in the loop; all but the newest
        // kTStages - 2 are complete
        cp_wait<kTStages - 2>();
        __syncthreads();  // ... every thread's; and every warp is done with stage s - 1 (its buffer, which
                          // pre-split activations feed to the mma directly, and wh / xhi / xlo)
        if (s + kTStages - 1 < nst) {  // into the buffer of stage s - 1
            issue_w(s + kTStages - 1);
            issue_x(s + kTStages - 1);
        }
        cp_commit();
        const St& S = raw[s % kTStages];
        // codes -> f16 (exact)
        if (FMT == kFP8) {
            for (int i = tid; i < BNW * (kTK / 8); i += kTThreads) {
                const int r = i / (kTK / 8), q = i - r * (kTK / 8);  // 8 codes at k = 8q
                const uint2 c = *reinterpret_cast<const uint2*>(&S.w[r][8 * q]);
                __half2 h0, h1, h2, h3;
                e4m3x4_to_half2(c.x, h0, h1);
                e4m3x4_to_half2(c.y, h2, h3);
                *reinterpret_cast<uint4*>(wh + r * kTP + 8 * q) = make_uint4(h2u(h0), h2u(h1), h2u(h2), h2u(h3));
            }
        } else {
            for (int i = tid; i < BNW * (kTK / 8); i += kTThreads) {
                // 4 bytes j..j+3 of a 32-block: weights j..j+3 (low nibbles) and 16+j..16+j+3 (high nibbles)
                const int r = i / (kTK / 8), q = i - r * (kTK / 8);
                const int blk = q >> 2, j = 4 * (q & 3);
                const uint32_t word = *reinterpret_cast<const uint32_t*>(&S.w[r][16 * blk + j]);
                const __half2 lo02 = fp4x2_to_half2(word & 0x000F000Fu);          // w j, j+2
                const __half2 lo13 = fp4x2_to_half2((word >> 8) & 0x000F000Fu);   // w j+1, j+3
                const __half2 hi02 = fp4x2_to_half2((word >> 4) & 0x000F000Fu);   // w 16+j, 16+j+2
                const __half2 hi13 = fp4x2_to_half2((word >> 12) & 0x000F000Fu);  // w 16+j+1, 16+j+3
                __half* dw = wh + r * kTP + 32 * blk;
                *reinterpret_cast<uint2*>(dw + j) =
                    make_uint2(h2u(__halves2half2(__low2half(lo02), __low2half(lo13))),
                               h2u(__halves2half2(__high2half(lo02), __high2half(lo13))));
                *reinterpret_cast<uint2*>(dw + 16 + j) =
                    make_uint2(h2u(__halves2half2(__low2half(hi02), __low2half(hi13))),
                               h2u(__halves2half2(__high2half(hi02), __high2half(hi13))));
            }
        }
        for (int r = tid; r < BNW; r += kTThreads) {  // block scales, with the code factor, in fp32
            scs[r] = __half2float(__ushort_as_half(S.sc[r][0])) * kCodeFactor;
            scs[BNW + r] = __half2float(__ushort_as_half(S.sc[r][1])) * kCodeFactor;
        }
        // activations -> hi + lo f16 (rows of the tile only; rows past mv only feed discarded outputs)
        for (int i = tid; !PRE && i < mv * (kTK / 4); i += kTThreads) {
            const int m = i / (kTK / 4), q = i - m * (kTK / 4);
            const float4 v = *reinterpret_cast<const float4*>(&reinterpret_cast<const XsF32&>(S.x).v[m][4 * q]);
            const __half2 h01 = __floats2half2_rn(v.x, v.y), h23 = __floats2half2_rn(v.z, v.w);
            const float2 f01 = __half22float2(h01), f23 = __half22float2(h23);
            *reinterpret_cast<uint2*>(xhi + m * kTP + 4 * q) = make_uint2(h2u(h01), h2u(h23));
            *reinterpret_cast<uint2*>(xlo + m * kTP + 4 * q) =
                make_uint2(h2u(__floats2half2_rn(v.x - f01.x, v.y - f01.y)),
                           h2u(__floats2half2_rn(v.z - f23.x, v.w - f23.y)));
        }
        __syncthreads();
        // tensor cores: per 32-block, exact partial sums of codes x (hi + lo), then the block scale in fp32
        const int c2 = 2 * (lane & 3);
        const __half* ahi = PRE ? &reinterpret_cast<const XsHiLo&>(S.x).v[0][0][0] : xhi;
        const __half* alo = PRE ? &reinterpret_cast<const XsHiLo&>(S.x).v[1][0][0] : xlo;
#pragma unroll
        for (int blk = 0; blk < 2; blk++) {
            if (16 * wm >= mv) break;  // no activation row of this warp
            float part[NT][4];
#pragma unroll
            for (int kk = 2 * blk; kk < 2 * blk + 2; kk++) {
                uint32_t ah[4], al[4], bf[NT / 2][4];
                const int ao = (16 * wm + (lane & 15)) * kTP + 16 * kk + 8 * (lane >> 4);
                ldsm_x4(ah, ahi + ao);
                ldsm_x4(al, alo + ao);
#pragma unroll
                for (int t = 0; t < NT; t += 2)
                    ldsm_x4(bf[t / 2],
                            wh + (8 * (NT * wn + t) + 8 * (lane >> 4) + (lane & 7)) * kTP + 16 * kk + 8 * ((lane >> 3) & 1));
                // every tile's hi product, then every tile's lo product: NT independent MMAs between dependent ones
#pragma unroll
                for (int t = 0; t < NT; t++) {
                    if (kk == 2 * blk) mma16816_z(part[t], ah, bf[t / 2][2 * (t & 1)], bf[t / 2][2 * (t & 1) + 1]);
                    else mma16816(part[t], ah, bf[t / 2][2 * (t & 1)], bf[t / 2][2 * (t & 1) + 1]);
                }
#pragma unroll
                for (int t = 0; t < NT; t++) mma16816(part[t], al, bf[t / 2][2 * (t & 1)], bf[t / 2][2 * (t & 1) + 1]);
            }
#pragma unroll
            for (int t = 0; t < NT; t++) {
                const float2 sc = *reinterpret_cast<const float2*>(scs + blk * BNW + 8 * (NT * wn + t) + c2);
                acc[t][0] = fmaf(sc.x, part[t][0], acc[t][0]);
                acc[t][1] = fmaf(sc.y, part[t][1], acc[t][1]);
                acc[t][2] = fmaf(sc.x, part[t][2], acc[t][2]);
                acc[t][3] = fmaf(sc.y, part[t][3], acc[t][3]);
            }
        }
    }

    pdl_trigger();  // the next kernel may start streaming its weights while this one finishes
    // epilogue. acc[t] holds rows (g, g + 8) x columns (2c, 2c + 1) of n8 tile NT wn + t: to a row-major fp32 tile in
    // this CTA's shared memory (the stage buffers are free once every warp is past its last stage)
    const int g = lane >> 2, c = lane & 3;
    constexpr int TPF = BNW + 4;  // padded row pitch (floats)
    static_assert(kTM * TPF * 4 <= kTStages * sizeof(St), "partial tile fits the stage buffers");
    __syncthreads();
    float* tile = reinterpret_cast<float*>(tsm);
    if (16 * wm < mv) {
#pragma unroll
        for (int t = 0; t < NT; t++) {
            const int col = 8 * (NT * wn + t) + 2 * c;
            *reinterpret_cast<float2*>(tile + (16 * wm + g) * TPF + col) = make_float2(acc[t][0], acc[t][1]);
            *reinterpret_cast<float2*>(tile + (16 * wm + g + 8) * TPF + col) = make_float2(acc[t][2], acc[t][3]);
        }
    }
    namespace cg = cooperative_groups;
    const int ks = sp.ksplit;
    // rows z, z + ks, ... of the tile: sums over the splits in order, then bias / GELU / accumulate or SiLU * up.
    // Element i of this CTA (row z + ks * (i / OC), column i % OC) belongs to thread i % kTThreads; a thread takes
    // kEpi elements per pass with every load of the pass issued first, and the global operands of the first pass
    // (residual, bias, gamma, the row scales) are fetched before the cluster barrier.
    constexpr int OC = PAIR ? BN : BNW;  // output columns of the tile
    constexpr int kEpi = 4;
    const int nrow = (mv - z + ks - 1) / ks;  // rows of this CTA
    const int total = nrow * OC;
    static_assert(OC % 32 == 0, "a warp's 32 elements share a row");
    static_assert(kTThreads % 32 == 0, "whole warps per pass");
    // RMSNorm as a row scale (the activations held x * gamma): rstd of each row from the producer's per-tile
    // sums of squares, summed in tile order (deterministic)
    __shared__ float rs[kTM];
    __shared__ float ssp[kTM][OC / 32];  // per row and 32-column group: sum of squares of the outputs
    if (a.in_ss) {
        for (int r = tid; r < nrow; r += kTThreads) {
            const int row = z + ks * r;
            double s2 = 0.0;
            for (int t = 0; t < a.in_ss_tiles; t++) s2 += double(a.in_ss[int64_t(t) * a.M + m0 + row]);
            rs[row] = float(1.0 / sqrt(s2 / a.K + double(a.eps)));
        }
    }
    // 16-byte path: 4 consecutive columns per thread (distributed-shared-memory, residual, bias and gamma loads
    // of 16 bytes, f16 hi / lo stores of 8 bytes) when the output layout allows it; a row is OC / 4 lanes
    const auto al = [](const void* p, uintptr_t n) { return (reinterpret_cast<uintptr_t>(p) & (n - 1)) == 0; };
    const bool vec = a.y_stride % 4 == 0 && a.n_off % 4 == 0 && a.rows % 4 == 0 && al(a.y, 16) &&
                     (!(a.flags & kBias) || al(a.bias, 16)) &&
                     (!a.out_hi || (a.out_ld % 4 == 0 && al(a.out_hi, 8) && al(a.out_lo, 8) &&
                                    (!a.out_gamma || al(a.out_gamma, 16))));
    const float* peer[kTMaxSplit];
    if (vec) {
        constexpr int G4 = OC / 4;  // lanes per row
        static_assert(32 % G4 == 0, "a row's lanes lie in one warp");
        const int total4 = nrow * G4;
        float4 v_old = make_float4(0.f, 0.f, 0.f, 0.f), v_bias = v_old, v_gam = make_float4(1.f, 1.f, 1.f, 1.f);
        auto fetch4 = [&](int i) {  // global operands of group i
            v_old = make_float4(0.f, 0.f, 0.f, 0.f);
            v_bias = v_old;
            v_gam = make_float4(1.f, 1.f, 1.f, 1.f);
            const int row = z + ks * (i / G4), n = n0 + 4 * (i - (i / G4) * G4);
            if (i < total4 && n < a.rows) {
                if (!PAIR && (a.flags & kAccumulate))
                    v_old = *reinterpret_cast<const float4*>(a.y + int64_t(m0 + row) * a.y_stride + a.n_off + n);
                if (!PAIR && (a.flags & kBias)) v_bias = *reinterpret_cast<const float4*>(a.bias + n);
                if (a.out_hi && a.out_gamma) v_gam = *reinterpret_cast<const float4*>(a.out_gamma + n);
            }
        };
        fetch4(tid);
        if (ks > 1) cg::this_cluster().sync();  // every split's partial tile is in place
        else __syncthreads();                   // (both also publish rs)
#pragma unroll
        for (int zz = 0; zz < kTMaxSplit; zz++)
            peer[zz] = zz < ks ? (ks > 1 ? cg::this_cluster().map_shared_rank(tile, zz) : tile) : tile;
        // every lane of a warp runs the same passes (the row reductions shuffle across the warp)
        for (int i = tid; i - lane < total4; i += kTThreads) {
            if (i != tid) fetch4(i);
            const bool live = i < total4;
            const int row = z + ks * ((live ? i : 0) / G4), col = 4 * ((live ? i : 0) % G4);
            float vv[4] = {0.f, 0.f, 0.f, 0.f}, uu[4] = {0.f, 0.f, 0.f, 0.f};
            if (live) {
                float4 pv[kTMaxSplit], pu[kTMaxSplit];
#pragma unroll
                for (int zz = 0; zz < kTMaxSplit; zz++) {
                    if (zz < ks) {
                        pv[zz] = *reinterpret_cast<const float4*>(peer[zz] + row * TPF + col);
                        if (PAIR) pu[zz] = *reinterpret_cast<const float4*>(peer[zz] + row * TPF + BN + col);
                    }
                }
#pragma unroll
                for (int zz = 0; zz < kTMaxSplit; zz++) {
                    if (zz < ks) {
                        vv[0] += pv[zz].x; vv[1] += pv[zz].y; vv[2] += pv[zz].z; vv[3] += pv[zz].w;
                        if (PAIR) { uu[0] += pu[zz].x; uu[1] += pu[zz].y; uu[2] += pu[zz].z; uu[3] += pu[zz].w; }
                    }
                }
            }
            const int m = m0 + row, n = n0 + col;
            const bool out = live && n < a.rows;
            unsigned long long key = 0ull;
            float sq = 0.0f;
            if (out) {
                const float old[4] = {v_old.x, v_old.y, v_old.z, v_old.w};
                const float bia[4] = {v_bias.x, v_bias.y, v_bias.z, v_bias.w};
                const float gam[4] = {v_gam.x, v_gam.y, v_gam.z, v_gam.w};
                float val[4];
                __half h[4], l[4];
#pragma unroll
                for (int e = 0; e < 4; e++) {
                    float x = vv[e], u = uu[e];
                    if (a.in_ss) {
                        x *= rs[row];
                        u *= rs[row];
                    }
                    if (PAIR) {
                        x = x / (1.0f + expf(-x)) * u;  // cpu::siluMul (cpu_ops.cpp:526-533)
                    } else {
                        if (a.flags & kBias) x += bia[e];
                        if (a.flags & kGelu) x = gelu(x);
                        if (a.flags & kAccumulate) x += old[e];
                    }
                    val[e] = x;
                    key = max(key, argmax_key(x, n + e));
                    sq += x * x;
                    const float yv = x * gam[e];
                    h[e] = __float2half_rn(yv);
                    l[e] = __float2half_rn(yv - __half2float(h[e]));
                }
                *reinterpret_cast<float4*>(a.y + int64_t(m) * a.y_stride + a.n_off + n) =
                    make_float4(val[0], val[1], val[2], val[3]);
                if (a.out_hi) {  // the next matmul's activations: val * gamma as f16 hi + lo
                    *reinterpret_cast<uint2*>(a.out_hi + int64_t(m) * a.out_ld + n) =
                        make_uint2(h2u(__halves2half2(h[0], h[1])), h2u(__halves2half2(h[2], h[3])));
                    *reinterpret_cast<uint2*>(a.out_lo + int64_t(m) * a.out_ld + n) =
                        make_uint2(h2u(__halves2half2(l[0], l[1])), h2u(__halves2half2(l[2], l[3])));
                }
            }
            if (a.out_ss) {  // the row's G4 lanes, in a fixed order; the whole row lands in its first column group
#pragma unroll
                for (int o = G4 / 2; o > 0; o >>= 1) sq += __shfl_xor_sync(0xffffffffu, sq, o);
                if (live && (lane % G4) == 0) {
                    ssp[row][0] = sq;
#pragma unroll
                    for (int hh = 1; hh < OC / 32; hh++) ssp[row][hh] = 0.0f;
                }
            }
            if (a.argmax) {
#pragma unroll
                for (int o = G4 / 2; o > 0; o >>= 1) key = max(key, __shfl_xor_sync(0xffffffffu, key, o));
                if (live && (lane % G4) == 0 && key) atomicMax(&keys[row], key);
            }
        }
    } else {
        float g_old[kEpi], g_bias[kEpi], g_gam[kEpi];  // residual, bias and gamma of the pass's elements
        auto fetch = [&](int base) {
    #pragma unroll
            for (int e = 0; e < kEpi; e++) {
                const int i = base + e * kTThreads;
                g_old[e] = 0.0f;
                g_bias[e] = 0.0f;
                g_gam[e] = 1.0f;
                const int row = z + ks * (i / OC), n = n0 + (i - (i / OC) * OC);
                if (i < total && n < a.rows) {
                    if (!PAIR && (a.flags & kAccumulate)) g_old[e] = a.y[int64_t(m0 + row) * a.y_stride + a.n_off + n];
                    if (!PAIR && (a.flags & kBias)) g_bias[e] = a.bias[n];
                    if (a.out_hi && a.out_gamma) g_gam[e] = a.out_gamma[n];
                }
            }
        };
        fetch(tid);
        if (ks > 1) cg::this_cluster().sync();  // every split's partial tile is in place
        else __syncthreads();                   // (both also publish rs)
    #pragma unroll
        for (int zz = 0; zz < kTMaxSplit; zz++)
            peer[zz] = zz < ks ? (ks > 1 ? cg::this_cluster().map_shared_rank(tile, zz) : tile) : tile;
        for (int base = tid; base < total; base += kEpi * kTThreads) {
            if (base != tid) fetch(base);
            float v[kEpi], u[kEpi];
    #pragma unroll
            for (int e = 0; e < kEpi; e++) {
                const int i = base + e * kTThreads;
                v[e] = u[e] = 0.0f;
                if (i < total) {
                    const int row = z + ks * (i / OC), col = i - (i / OC) * OC;
    #pragma unroll
                    for (int zz = 0; zz < kTMaxSplit; zz++) {
                        if (zz >= ks) break;
                        v[e] += peer[zz][row * TPF + col];
                        if (PAIR) u[e] += peer[zz][row * TPF + BN + col];
                    }
                }
            }
    #pragma unroll
            for (int e = 0; e < kEpi; e++) {
                const int i = base + e * kTThreads;
                if (i >= total) break;  // whole warps: total and the pass stride are multiples of 32
                const int row = z + ks * (i / OC), col = i - (i / OC) * OC;
                const int m = m0 + row, n = n0 + col;
                float vv = v[e], uu = u[e];
                if (a.in_ss) {
                    vv *= rs[row];
                    uu *= rs[row];
                }
                unsigned long long key = 0ull;
                float sq = 0.0f;
                if (n < a.rows) {
                    float val = vv;
                    if (PAIR) {
                        val = val / (1.0f + expf(-val)) * uu;  // cpu::siluMul (cpu_ops.cpp:526-533)
                    } else {
                        if (a.flags & kBias) val += g_bias[e];
                        if (a.flags & kGelu) val = gelu(val);
                        if (a.flags & kAccumulate) val += g_old[e];
                    }
                    a.y[int64_t(m) * a.y_stride + a.n_off + n] = val;
                    key = argmax_key(val, n);
                    if (a.out_hi) {  // the next matmul's activations: val * gamma as f16 hi + lo
                        const float yv = val * g_gam[e];
                        const __half h = __float2half_rn(yv);
                        a.out_hi[int64_t(m) * a.out_ld + n] = h;
                        a.out_lo[int64_t(m) * a.out_ld + n] = __float2half_rn(yv - __half2float(h));
                    }
                    sq = val * val;
                }
                if (a.out_ss) {  // the warp's 32 columns of the row
                    sq = warp_sum(sq);
                    if (lane == 0) ssp[row][col >> 5] = sq;
                }
                if (a.argmax) {  // the warp's 32 columns of the row, then one shared atomic
    #pragma unroll
                    for (int o = 16; o > 0; o >>= 1) key = max(key, __shfl_xor_sync(0xffffffffu, key, o));
                    if (lane == 0 && key) atomicMax(&keys[row], key);
                }
            }
        }
    }
    // this CTA's reads of its peers' tiles are done: the cluster barrier's arrival now, its wait at exit (no CTA
    // leaves while a peer may still read its tile)
    if (ks > 1) cg::this_cluster().barrier_arrive();
    if (a.out_ss) {  // one partial per (column tile, row), the column groups summed in order
        __syncthreads();
        for (int r = tid; r < nrow; r += kTThreads) {
            const int row = z + ks * r;
            float s2 = 0.0f;
#pragma unroll
            for (int h = 0; h < OC / 32; h++) s2 += ssp[row][h];
            a.out_ss[int64_t(blockIdx.x) * a.M + m0 + row] = s2;
        }
    }
    if (a.argmax) {  // one global atomic per row of this CTA
        __syncthreads();
        if (tid < nrow && keys[z + ks * tid]) atomicMax(a.argmax + m0 + z + ks * tid, keys[z + ks * tid]);
    }
    if (ks > 1) cg::this_cluster().barrier_wait();
}

using TcFn = void (*)(const GemvArgs, const TcSplit);

// CTA tiles: 64 weight rows, or 32 gate + 32 up rows for SwiGLU
template <int FMT, bool PRE>
TcFn pick(bool pair) {
    return pair ? tc_gemm_kernel<FMT, 32, true, PRE> : tc_gemm_kernel<FMT, 64, false, PRE>;
}

template <int FMT, bool PRE>
constexpr size_t tc_smem() {
    return kTStages * sizeof(Stage<FMT, 64, PRE>) + size_t(PRE ? 64 : 64 + 2 * kTM) * kTP * 2 + 2 * 64 * 4;
}

// Tile plan of a call: weight rows per CTA, row blocks, tiles, K splits (the workspace decides how many).
struct TcPlan {
    int bn, mblk, ntile, ksplit, sper;
    bool presplit;
    int64_t x_floats;  // workspace: hi / lo activations (as floats)
};

TcPlan tc_plan(const GemvArgs& a, int64_t ws_floats) {
    TcPlan p;
    const bool pair = a.pair_off != 0;
    const int sms = num_sms(), nst = a.K / kTK;
    p.mblk = (a.M + kTM - 1) / kTM;
    p.bn = pair ? 32 : 64;  // at most 64 weight rows per CTA (the registers of the partial sums)
    p.ntile = (a.rows + p.bn - 1) / p.bn;
    const int64_t tiles = int64_t(p.ntile) * p.mblk;
    // activations split once when at least 8 tiles share them
    p.x_floats = int64_t(a.M) * a.K;  // hi + lo halves
    p.presplit = (p.ntile >= 8 || a.norm != kNormNone || a.M >= 64) && ws_floats >= p.x_floats;
    // K splits (one cluster per tile): about two CTAs per SM, each with at least 2 stages. Rounding down (one
    // wave on paper) measured slower for the SwiGLU matmul of a batch-64 step: 3 splits of 6 stages left 3
    // clusters unplaced until others finished (the previous kernel's CTAs still hold SMs when it launches),
    // 4 splits of 4 stages run in 1.3 waves of shorter CTAs.
    p.ksplit = 1;
    if (tiles < 2 * sms)
        p.ksplit = int(std::min<int64_t>({(2 * sms + tiles - 1) / tiles, int64_t(kTMaxSplit), std::max(1, nst / 2)}));
    p.sper = (nst + p.ksplit - 1) / p.ksplit;
    p.ksplit = (nst + p.sper - 1) / p.sper;  // no empty split
    return p;
}

size_t tc_smem_for(int fmt, bool pre) {
    if (fmt == kFP8) return pre ? tc_smem<kFP8, true>() : tc_smem<kFP8, false>();
    return pre ? tc_smem<kFP4, true>() : tc_smem<kFP4, false>();
}

}  // namespace

bool gemm_tc_fits(const GemvArgs& a) {
    return a.M >= 5 && (a.fmt == kFP8 || a.fmt == kFP4) && a.K % kTK == 0 &&
           (a.norm == kNormNone || a.K <= kNsMaxK) &&
           a.x_stride % 4 == 0 && (reinterpret_cast<uintptr_t>(a.x) & 15) == 0 && a.row_bytes % 16 == 0 &&
           !(a.pair_off && a.argmax);
}

namespace {
GemvArgs shape_args(int fmt, int rows, int K, int M, bool pair, bool norm) {
    GemvArgs a;
    a.norm = norm ? kNormRms : kNormNone;
    a.fmt = fmt;
    a.rows = rows;
    a.K = K;
    a.M = M;
    a.x_stride = K;
    a.row_bytes = 16;
    a.pair_off = pair ? rows : 0;
    return a;
}
}  // namespace

int gemm_tc_launches(int fmt, int rows, int K, int M, bool pair, bool norm) {
    const GemvArgs a = shape_args(fmt, rows, K, M, pair, norm);
    if (!gemm_tc_fits(a)) return 0;
    return tc_plan(a, int64_t(1) << 40).presplit ? 2 : 1;
}

void gemm_tc_scratch(int fmt, int rows, int K, int M, bool pair, bool norm, int64_t* floats, int64_t* tickets) {
    *floats = 0;
    *tickets = 0;
    const GemvArgs a = shape_args(fmt, rows, K, M, pair, norm);
    if (!gemm_tc_fits(a)) return;
    const TcPlan p = tc_plan(a, int64_t(1) << 40);
    *floats = p.presplit ? p.x_floats : 0;
    // 256+ rows: room for the dequantised hi / lo weight rows after the activations (SwiGLU: gate and up rows)
    if (p.presplit && M >= kGemmDqMinRows) *floats += int64_t(pair ? 2 * rows : rows) * K;
}

// The tensor-core kernel takes 5+ activation rows of FP8 / FP4 weights, K a multiple of 64; cudaErrorNotSupported
// otherwise. a.ws (a.ws_floats floats) lets it split the activations once (without it every CTA splits its own
// copy); a norm prologue is applied by that split, so it needs the workspace.
cudaError_t launch_gemm_tc(const GemvArgs& a, cudaStream_t st, bool pdl) {
    if (!gemm_tc_fits(a)) return cudaErrorNotSupported;
    const bool pair = a.pair_off != 0;
    TcPlan pl = tc_plan(a, a.ws ? a.ws_floats : 0);
    const bool chained = a.x_hi || a.in_ss || a.out_hi || a.out_ss;
    if (chained) {  // this kernel only (not tcgen05); norms only as row scales
        if (a.norm != kNormNone || (a.x_hi && !a.x_lo) || (a.in_ss && a.in_ss_tiles <= 0) ||
            (a.out_hi && (!a.out_lo || a.out_ld < a.rows)))
            return cudaErrorInvalidValue;
        if (a.x_hi) pl.presplit = true;
    }
    if (a.norm != kNormNone && !pl.presplit) return cudaErrorNotSupported;
    TcSplit sp{};
    sp.ksplit = pl.ksplit;
    sp.sper = pl.sper;
    if (a.x_hi) {
        sp.xh = a.x_hi;
        sp.xl = a.x_lo;
    } else if (pl.presplit) {
        sp.xh = reinterpret_cast<const __half*>(a.ws);
        sp.xl = sp.xh + int64_t(a.M) * a.K;
        cudaError_t e;
        if (a.norm != kNormNone) {
            e = launch_ex(norm_split_kernel, dim3(a.M), dim3(kNsThreads), 0, st, pdl, a, const_cast<__half*>(sp.xh),
                          const_cast<__half*>(sp.xl));
        } else {
            const int64_t n4 = int64_t(a.M) * (a.K / 4);
            const int blocks = int(std::min<int64_t>((n4 + 255) / 256, 4 * num_sms()));
            e = launch_ex(split_act_kernel, dim3(blocks), dim3(256), 0, st, pdl, a.x, a.x_stride, a.M, a.K,
                          const_cast<__half*>(sp.xh), const_cast<__half*>(sp.xl));
        }
        if (e != cudaSuccess) return e;
        // 256+ rows: weights dequantised once, then the TMA-fed tcgen05 GEMM; 128+ rows: the tcgen05 kernel that
        // converts the codes per CTA (both TMEM accumulators, on the split activations)
        if (!chained) {
            e = launch_gemm_umma_dq(a, sp.xh, sp.xl, st, true);
            if (e != cudaErrorNotSupported) return e;
            e = launch_gemm_umma(a, sp.xh, sp.xl, st, true);
            if (e != cudaErrorNotSupported) return e;
        }
    }
    // 5..64 rows on split activations: the warp-specialised tcgen05 kernel (k_umma_ws.cu), after this call's
    // split kernel (programmatic launch) or chained to the previous matmul as asked; NEKO_GEMM_WS=0 in the
    // environment keeps this kernel for comparison
    static const bool ws_on = [] {
        const char* v = std::getenv("NEKO_GEMM_WS");
        return !(v && v[0] == '0');
    }();
    if (ws_on && pl.presplit && a.M <= 64) {
        const cudaError_t e = launch_gemm_ws(a, sp.xh, sp.xl, st, a.x_hi ? pdl : true);
        if (e != cudaErrorNotSupported) return e;
    }
    const bool pre = pl.presplit;
    TcFn k = a.fmt == kFP8 ? (pre ? pick<kFP8, true>(pair) : pick<kFP8, false>(pair))
                           : (pre ? pick<kFP4, true>(pair) : pick<kFP4, false>(pair));
    const size_t smem = tc_smem_for(a.fmt, pre);
    static int attr_set[8 * 8] = {};  // per (format, pair, pre-split, device), device < 8
    int dev = 0;
    cudaGetDevice(&dev);
    const int slot = ((a.fmt == kFP8 ? 0 : 4) + (pair ? 2 : 0) + (pre ? 1 : 0)) * 8 + dev;
    if (dev >= 8 || attr_set[slot] < int(smem)) {
        const cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
        if (e != cudaSuccess) return e;
        if (dev < 8) attr_set[slot] = int(smem);
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(pl.ntile, pl.mblk, pl.ksplit);
    cfg.blockDim = dim3(kTThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[2];
    int na = 0;
    if (pdl || (pl.presplit && !a.x_hi)) {  // after the split kernel of this call, or as asked
        attr[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[na].val.programmaticStreamSerializationAllowed = 1;
        na++;
    }
    if (pl.ksplit > 1) {  // the K splits of a tile form one cluster
        attr[na].id = cudaLaunchAttributeClusterDimension;
        attr[na].val.clusterDim.x = 1;
        attr[na].val.clusterDim.y = 1;
        attr[na].val.clusterDim.z = pl.ksplit;
        na++;
    }
    cfg.attrs = attr;
    cfg.numAttrs = na;
    return cudaLaunchKernelEx(&cfg, k, a, sp);
}

}  // namespace neko
