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
//  * CTA tile: 64 activation rows x BN output rows (16 / 32 / 64 by N so that there are enough CTAs; SwiGLU:
//    BN gate + BN up rows, BN <= 32); K walked in stages of 64 through a 4-deep cp.async pipeline; per stage
//    the CTA converts codes and activations once into padded shared memory; 4 warps, warp w owns activation
//    rows 16w..16w+15 of the tile, ldmatrix.x4 fragments, all BN columns.
// Activations must stay within the f16 range (|x| < 65504), which the matmul inputs of the models are
// (normalised activations, attention outputs, SwiGLU products).
#include <algorithm>

#include "gemv_core.cuh"
#include "neko_common.cuh"
#include "neko_internal.h"

namespace neko {

namespace {

constexpr int kTM = 64;        // activation rows per CTA
constexpr int kTK = 64;        // K per stage
constexpr int kTP = kTK + 8;   // padded row pitch of the converted tiles (halves): ldmatrix without conflicts
constexpr int kTThreads = 128;
constexpr int kTStages = 4;   // cp.async pipeline depth

__device__ __forceinline__ void cp16(void* dst, const void* src, int src_bytes) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(dst)), "l"(src), "r"(src_bytes)
                 : "memory");
}
__device__ __forceinline__ void cp4(void* dst, const void* src) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_wait() {
    asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}
__device__ __forceinline__ void ldsm_x4(uint32_t (&r)[4], const void* p) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(smem_u32(p)));
}
__device__ __forceinline__ void mma16816(float (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
__device__ __forceinline__ uint32_t h2u(__half2 h) { return *reinterpret_cast<uint32_t*>(&h); }

// Raw stage: W codes [BNW][kTK] (FP8 bytes / FP4 kTK / 2 bytes), scales [BNW][2] f16, activations [kTM][kTK] f32.
template <int FMT, int BNW>
struct Stage {
    static constexpr int kCode = FMT == kFP8 ? kTK : kTK / 2;
    uint8_t w[BNW][kCode];
    uint16_t sc[BNW][2];
    float x[kTM][kTK];
};

template <int FMT, int BN, bool PAIR>
__global__ void __launch_bounds__(kTThreads) tc_gemm_kernel(const GemvArgs a) {
    constexpr int BNW = PAIR ? 2 * BN : BN;  // weight rows per CTA
    constexpr int NT = BNW / 8;              // n8 tiles per warp
    using St = Stage<FMT, BNW>;
    extern __shared__ __align__(128) uint8_t tsm[];
    St* raw = reinterpret_cast<St*>(tsm);                                        // [kTStages]
    __half* wh = reinterpret_cast<__half*>(tsm + kTStages * sizeof(St));         // [BNW][kTP] codes
    __half* xhi = wh + BNW * kTP;                                                // [kTM][kTP]
    __half* xlo = xhi + kTM * kTP;                                               // [kTM][kTP]
    float* scs = reinterpret_cast<float*>(xlo + kTM * kTP);                      // [2][BNW] block scales
    __shared__ unsigned long long keys[kTM];

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int n0 = blockIdx.x * BN, m0 = blockIdx.y * kTM;
    const int cbytes = FMT == kFP8 ? a.K : a.K / 2;
    const int nst = a.K / kTK;
    constexpr float kCodeFactor = FMT == kFP8 ? kFp8HwFactor : kFp4Factor;  // code value -> engine decode
    pdl_wait();
    if (a.argmax && tid < kTM) keys[tid] = 0ull;

    // weight row r of the tile -> packed row in W (rows past the end repeat the last row; never stored)
    auto wrow = [&](int r) -> const uint8_t* {
        const int n = PAIR ? (r < BN ? n0 + r : n0 + (r - BN)) : n0 + r;
        const int nc = min(n, a.rows - 1);
        return a.W + (int64_t(nc) + (PAIR && r >= BN ? a.pair_off : 0)) * a.row_bytes;
    };
    auto issue = [&](int s) {
        St& S = raw[s % kTStages];
        constexpr int kPieces = St::kCode / 16;  // 16-byte pieces of codes per row
        for (int i = tid; i < BNW * kPieces; i += kTThreads) {
            const int r = i / kPieces, q = i - r * kPieces;
            cp16(&S.w[r][16 * q], wrow(r) + s * St::kCode + 16 * q, 16);
        }
        for (int r = tid; r < BNW; r += kTThreads) cp4(&S.sc[r][0], wrow(r) + cbytes + 4 * s);
        for (int i = tid; i < kTM * (kTK / 4); i += kTThreads) {
            const int m = i / (kTK / 4), q = i - m * (kTK / 4);
            const bool in = m0 + m < a.M;
            cp16(&S.x[m][4 * q], in ? a.x + int64_t(m0 + m) * a.x_stride + s * kTK + 4 * q : a.x, in ? 16 : 0);
        }
    };

    float acc[NT][4];
#pragma unroll
    for (int t = 0; t < NT; t++) acc[t][0] = acc[t][1] = acc[t][2] = acc[t][3] = 0.0f;

#pragma unroll
    for (int s = 0; s < kTStages - 1; s++) {  // prologue: the first stages in flight (one group each)
        if (s < nst) issue(s);
        cp_commit();
    }
    for (int s = 0; s < nst; s++) {
        if (s + kTStages - 1 < nst) issue(s + kTStages - 1);
        cp_commit();
        cp_wait<kTStages - 1>();  // stage s landed (this thread's copies)
        __syncthreads();          // ... every thread's; and the previous stage's mma is done with wh / xhi / xlo
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
        // activations -> hi + lo f16
        for (int i = tid; i < kTM * (kTK / 4); i += kTThreads) {
            const int m = i / (kTK / 4), q = i - m * (kTK / 4);
            const float4 v = *reinterpret_cast<const float4*>(&S.x[m][4 * q]);
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
#pragma unroll
        for (int blk = 0; blk < 2; blk++) {
            float part[NT][4];
#pragma unroll
            for (int t = 0; t < NT; t++) part[t][0] = part[t][1] = part[t][2] = part[t][3] = 0.0f;
#pragma unroll
            for (int kk = 2 * blk; kk < 2 * blk + 2; kk++) {
                uint32_t ah[4], al[4];
                const int ao = (16 * warp + (lane & 15)) * kTP + 16 * kk + 8 * (lane >> 4);
                ldsm_x4(ah, xhi + ao);
                ldsm_x4(al, xlo + ao);
#pragma unroll
                for (int t = 0; t < NT; t += 2) {
                    uint32_t bf[4];
                    ldsm_x4(bf, wh + (8 * t + 8 * (lane >> 4) + (lane & 7)) * kTP + 16 * kk + 8 * ((lane >> 3) & 1));
                    mma16816(part[t], ah, bf[0], bf[1]);
                    mma16816(part[t], al, bf[0], bf[1]);
                    mma16816(part[t + 1], ah, bf[2], bf[3]);
                    mma16816(part[t + 1], al, bf[2], bf[3]);
                }
            }
#pragma unroll
            for (int t = 0; t < NT; t++) {
                const float2 sc = *reinterpret_cast<const float2*>(scs + blk * BNW + 8 * t + c2);
                acc[t][0] = fmaf(sc.x, part[t][0], acc[t][0]);
                acc[t][1] = fmaf(sc.y, part[t][1], acc[t][1]);
                acc[t][2] = fmaf(sc.x, part[t][2], acc[t][2]);
                acc[t][3] = fmaf(sc.y, part[t][3], acc[t][3]);
            }
        }
    }

    // epilogue: acc[t] holds rows (g, g + 8) x columns (2c, 2c + 1) of n8 tile t
    const int g = lane >> 2, c = lane & 3;
    unsigned long long best[2] = {0ull, 0ull};
#pragma unroll
    for (int t = 0; t < (PAIR ? NT / 2 : NT); t++) {
#pragma unroll
        for (int e = 0; e < 4; e++) {
            const int mr = 16 * warp + g + (e >= 2 ? 8 : 0), m = m0 + mr;
            const int n = n0 + 8 * t + 2 * c + (e & 1);
            if (m >= a.M || n >= a.rows) continue;
            float* dst = a.y + int64_t(m) * a.y_stride + a.n_off + n;
            float val = acc[t][e];
            if (PAIR) {
                const float u = acc[t + NT / 2][e];
                val = val / (1.0f + expf(-val)) * u;  // cpu::siluMul (cpu_ops.cpp:526-533)
            } else {
                if (a.flags & kBias) val += a.bias[n];
                if (a.flags & kGelu) val = gelu(val);
                if (a.flags & kAccumulate) val += *dst;
            }
            *dst = val;
            if (a.argmax) best[e >> 1] = max(best[e >> 1], argmax_key(val, n));
        }
    }
    if (a.argmax) {  // rows g and g + 8: the 4 lanes of a row, then one shared and one global atomic per row
        __syncthreads();
#pragma unroll
        for (int h = 0; h < 2; h++) {
            unsigned long long k = best[h];
            k = max(k, __shfl_xor_sync(0xffffffffu, k, 1));
            k = max(k, __shfl_xor_sync(0xffffffffu, k, 2));
            if (c == 0 && k) atomicMax(&keys[16 * warp + g + 8 * h], k);
        }
        __syncthreads();
        if (tid < kTM && m0 + tid < a.M && keys[tid]) atomicMax(a.argmax + m0 + tid, keys[tid]);
    }
    pdl_trigger();
}

using TcFn = void (*)(const GemvArgs);

template <int FMT, int BN>
TcFn pick_pair(bool pair) {
    if constexpr (BN > 32) return tc_gemm_kernel<FMT, BN, false>;  // SwiGLU tiles take BN <= 32
    else return pair ? tc_gemm_kernel<FMT, BN, true> : tc_gemm_kernel<FMT, BN, false>;
}
template <int FMT>
TcFn pick_bn(int bn, bool pair) {
    return bn == 16 ? pick_pair<FMT, 16>(pair) : bn == 32 ? pick_pair<FMT, 32>(pair) : pick_pair<FMT, 64>(pair);
}

template <int FMT, int BNW>
constexpr size_t tc_smem() {
    return kTStages * sizeof(Stage<FMT, BNW>) + size_t(BNW + 2 * kTM) * kTP * 2 + 2 * BNW * 4;
}

size_t tc_smem_for(int fmt, int bn, bool pair) {
    const int bnw = pair ? 2 * bn : bn;
    if (fmt == kFP8)
        return bnw == 16 ? tc_smem<kFP8, 16>() : bnw == 32 ? tc_smem<kFP8, 32>() : bnw == 64 ? tc_smem<kFP8, 64>()
                                                                                           : tc_smem<kFP8, 128>();
    return bnw == 16 ? tc_smem<kFP4, 16>() : bnw == 32 ? tc_smem<kFP4, 32>() : bnw == 64 ? tc_smem<kFP4, 64>()
                                                                                     : tc_smem<kFP4, 128>();
}

}  // namespace

// The tensor-core kernel takes 5+ activation rows of FP8 / FP4 weights without a norm prologue, K a multiple of
// 64; cudaErrorNotSupported otherwise.
cudaError_t launch_gemm_tc(const GemvArgs& a, cudaStream_t st, bool pdl) {
    if (a.M < 5 || (a.fmt != kFP8 && a.fmt != kFP4) || a.norm != kNormNone || a.K % kTK) return cudaErrorNotSupported;
    if (a.x_stride % 4 || (reinterpret_cast<uintptr_t>(a.x) & 15) || a.row_bytes % 16) return cudaErrorNotSupported;
    const bool pair = a.pair_off != 0;
    if (pair && a.argmax) return cudaErrorNotSupported;
    const int sms = num_sms();
    const int mblk = (a.M + kTM - 1) / kTM;
    int bn = pair ? 32 : 64;  // at most 64 weight rows per CTA (the registers of the partial sums)
    while (bn > 16 && int64_t((a.rows + bn - 1) / bn) * mblk < sms) bn /= 2;
    TcFn k = a.fmt == kFP8 ? pick_bn<kFP8>(bn, pair) : pick_bn<kFP4>(bn, pair);
    const size_t smem = tc_smem_for(a.fmt, bn, pair);
    static int attr_set[2 * 6 * 8] = {};  // per (format, BN, pair, device), device < 8
    int dev = 0;
    cudaGetDevice(&dev);
    const int slot = ((a.fmt == kFP8 ? 0 : 1) * 6 + (bn == 16 ? 0 : bn == 32 ? 1 : 2) * 2 + (pair ? 1 : 0)) * 8 + dev;
    if (dev >= 8 || attr_set[slot] < int(smem)) {
        const cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
        if (e != cudaSuccess) return e;
        if (dev < 8) attr_set[slot] = int(smem);
    }
    return launch_ex(k, dim3((a.rows + bn - 1) / bn, mblk), dim3(kTThreads), smem, st, pdl, a);
}

}  // namespace neko
