// Shared pieces of the dequantising dot products (the GEMV kernel and the decode-step kernel): the engine's
// packed weight rows (quant.cpp:199-208) are walked in 512-byte segments of codes, lane l taking bytes
// [16 l, 16 l + 16) of each segment, and activations are staged in a permuted shared-memory layout so that
// each lane reads its activations as bank-conflict-free float4s.
#pragma once
#include "neko_common.cuh"

namespace neko {

constexpr int kSegBytes = 512;  // bytes of one row segment (16 per lane)
constexpr float kFp8HwFactor = 1.0f;  // FP8 sums of seg_dot_rows are already at full scale (e4m3 decode)

// Weights per segment and float4s of activations per lane per segment, by format.
template <int FMT> struct Seg;
template <> struct Seg<kFP8> { static constexpr int W = 512, Q = 4; };
template <> struct Seg<kFP4> { static constexpr int W = 1024, Q = 8; };
template <> struct Seg<kF16> { static constexpr int W = 256, Q = 2; };

__host__ __device__ inline int code_bytes(int fmt, int K) { return fmt == kFP8 ? K : fmt == kFP4 ? K / 2 : 2 * K; }
__host__ __device__ inline int seg_count(int fmt, int K) { return (code_bytes(fmt, K) + kSegBytes - 1) / kSegBytes; }

// Staged-activation index (in floats) of logical activation k: segment s, lane l, float4 q, element e.
template <int FMT>
__device__ __forceinline__ int xperm(int k) {
    constexpr int W = Seg<FMT>::W, Q = Seg<FMT>::Q, WL = W / 32;
    const int s = k / W, r = k % W, l = r / WL, t = r % WL;
    return (((s * Q + t / 4) * 32 + l) << 2) + (t & 3);
}

// Greedy argmax key: the float's order-preserving bit pattern in the high word, the complement of the index in
// the low word, so the largest key is the largest value with the smallest index (std::max_element).
__device__ __forceinline__ unsigned long long argmax_key(float v, int n) {
    const unsigned b = __float_as_uint(v);
    const unsigned ord = (b & 0x80000000u) ? ~b : (b | 0x80000000u);
    return (static_cast<unsigned long long>(ord) << 32) | static_cast<unsigned>(0xFFFFFFFFu - unsigned(n));
}

// dot of 4 fp32 activations with 4 weights (even = weights 0, 2; odd = weights 1, 3)
__device__ __forceinline__ float dot4(const float4 x, const float2 e, const float2 o, float p) {
    p = fmaf(x.x, e.x, p);
    p = fmaf(x.y, o.x, p);
    p = fmaf(x.z, e.y, p);
    return fmaf(x.w, o.y, p);
}

// One lane's 16 weight bytes of one row (segment s) against MT activation rows; accumulates into acc[m].
template <int FMT, int MT>
__device__ __forceinline__ void seg_dot(const uint8_t* row, int cbytes, int s, int lane,
                                        const float4 (&xv)[MT][Seg<FMT>::Q], float (&acc)[MT]) {
    const uint4 w = *reinterpret_cast<const uint4*>(row + s * kSegBytes + 16 * lane);
    const uint32_t wd[4] = {w.x, w.y, w.z, w.w};
    if (FMT == kFP8) {
        const float sc =
            half_bits_to_float(*reinterpret_cast<const uint16_t*>(row + cbytes + 2 * (16 * s + (lane >> 1))));
        float2 e[4], o[4];
#pragma unroll
        for (int i = 0; i < 4; i++) {
            __half2 he, ho;
            fp8x4_to_half2(wd[i], he, ho);
            e[i] = __half22float2(he);
            o[i] = __half22float2(ho);
        }
#pragma unroll
        for (int m = 0; m < MT; m++) {
            float p0 = dot4(xv[m][0], e[0], o[0], 0.0f);
            float p1 = dot4(xv[m][1], e[1], o[1], 0.0f);
            p0 = dot4(xv[m][2], e[2], o[2], p0);
            p1 = dot4(xv[m][3], e[3], o[3], p1);
            acc[m] = fmaf(sc, p0 + p1, acc[m]);
        }
    } else if (FMT == kFP4) {
        const float sc = half_bits_to_float(*reinterpret_cast<const uint16_t*>(row + cbytes + 2 * (32 * s + lane)));
        float2 le[4], lo[4], he[4], ho[4];
#pragma unroll
        for (int i = 0; i < 4; i++) {
            le[i] = __half22float2(fp4x2_to_half2(wd[i] & 0x000F000Fu));
            lo[i] = __half22float2(fp4x2_to_half2((wd[i] >> 8) & 0x000F000Fu));
            he[i] = __half22float2(fp4x2_to_half2((wd[i] >> 4) & 0x000F000Fu));
            ho[i] = __half22float2(fp4x2_to_half2((wd[i] >> 12) & 0x000F000Fu));
        }
#pragma unroll
        for (int m = 0; m < MT; m++) {
            float p0 = 0.0f, p1 = 0.0f;
#pragma unroll
            for (int i = 0; i < 4; i++) {
                p0 = dot4(xv[m][i], le[i], lo[i], p0);      // weights 4i .. 4i+3 (low nibbles)
                p1 = dot4(xv[m][4 + i], he[i], ho[i], p1);  // weights 16+4i .. (high nibbles)
            }
            acc[m] = fmaf(sc, p0 + p1, acc[m]);
        }
    } else {
        float2 h[4];
#pragma unroll
        for (int i = 0; i < 4; i++) h[i] = __half22float2(*reinterpret_cast<const __half2*>(&wd[i]));
#pragma unroll
        for (int m = 0; m < MT; m++) {
            float p0 = xv[m][0].x * h[0].x;
            p0 = fmaf(xv[m][0].y, h[0].y, p0);
            p0 = fmaf(xv[m][0].z, h[1].x, p0);
            p0 = fmaf(xv[m][0].w, h[1].y, p0);
            float p1 = xv[m][1].x * h[2].x;
            p1 = fmaf(xv[m][1].y, h[2].y, p1);
            p1 = fmaf(xv[m][1].z, h[3].x, p1);
            p1 = fmaf(xv[m][1].w, h[3].y, p1);
            acc[m] += p0 + p1;
        }
    }
}

// seg_dot with the activations read from the permuted shared-memory staging row by row (xs4: float4 view,
// xrow4 float4s per staged row) instead of preloaded registers, for up to NM activation rows of which M are
// live. Same operations in the same order as seg_dot, so both give identical sums.
template <int FMT, int NM>
__device__ __forceinline__ void seg_dot_xs(const uint8_t* row, int cbytes, int s, int lane, const float4* xs4,
                                           int xrow4, int M, float (&acc)[NM]) {
    constexpr int Q = Seg<FMT>::Q;
    const uint4 w = *reinterpret_cast<const uint4*>(row + s * kSegBytes + 16 * lane);
    const uint32_t wd[4] = {w.x, w.y, w.z, w.w};
    const float4* xb = xs4 + s * Q * 32 + lane;
    if (FMT == kFP8) {
        const float sc =
            half_bits_to_float(*reinterpret_cast<const uint16_t*>(row + cbytes + 2 * (16 * s + (lane >> 1))));
        float2 e[4], o[4];
#pragma unroll
        for (int i = 0; i < 4; i++) {
            __half2 he, ho;
            fp8x4_to_half2(wd[i], he, ho);
            e[i] = __half22float2(he);
            o[i] = __half22float2(ho);
        }
#pragma unroll
        for (int m = 0; m < NM; m++) {
            if (m >= M) break;
            const float4* xm = xb + m * xrow4;
            float p0 = dot4(xm[0], e[0], o[0], 0.0f);
            float p1 = dot4(xm[32], e[1], o[1], 0.0f);
            p0 = dot4(xm[64], e[2], o[2], p0);
            p1 = dot4(xm[96], e[3], o[3], p1);
            acc[m] = fmaf(sc, p0 + p1, acc[m]);
        }
    } else {
        const float sc = half_bits_to_float(*reinterpret_cast<const uint16_t*>(row + cbytes + 2 * (32 * s + lane)));
        float2 le[4], lo[4], he[4], ho[4];
#pragma unroll
        for (int i = 0; i < 4; i++) {
            le[i] = __half22float2(fp4x2_to_half2(wd[i] & 0x000F000Fu));
            lo[i] = __half22float2(fp4x2_to_half2((wd[i] >> 8) & 0x000F000Fu));
            he[i] = __half22float2(fp4x2_to_half2((wd[i] >> 4) & 0x000F000Fu));
            ho[i] = __half22float2(fp4x2_to_half2((wd[i] >> 12) & 0x000F000Fu));
        }
#pragma unroll
        for (int m = 0; m < NM; m++) {
            if (m >= M) break;
            const float4* xm = xb + m * xrow4;
            float p0 = 0.0f, p1 = 0.0f;
#pragma unroll
            for (int i = 0; i < 4; i++) {
                p0 = dot4(xm[32 * i], le[i], lo[i], p0);
                p1 = dot4(xm[32 * (4 + i)], he[i], ho[i], p1);
            }
            acc[m] = fmaf(sc, p0 + p1, acc[m]);
        }
    }
}

// Four FP8 codes (one 32-bit word, code i in byte i) to two f16x2 (codes 0, 1 and 2, 3) with the hardware e4m3
// conversion. The engine's FP8 code is e4m3 (sign, 4 exponent bits with bias 7, 3 mantissa bits, subnormals):
// its decode (f16 bits (c & 0x80) << 8 | (c & 0x7F) << 7, times 256, quant.h:27) gives the same value as e4m3 for
// every code except 0x7F / 0xFF (480 there, NaN in e4m3), which the quantizer never emits (it clamps to 0x7E).
// The values come out 256 times those of fp8x4_to_half2, so sums over them equal those sums times 256 exactly.
__device__ __forceinline__ void e4m3x4_to_half2(uint32_t q, __half2& lo, __half2& hi) {
    uint32_t a, b;
    asm("{.reg .b16 l, h;\n\tmov.b32 {l, h}, %2;\n\tcvt.rn.f16x2.e4m3x2 %0, l;\n\tcvt.rn.f16x2.e4m3x2 %1, h;\n\t}"
        : "=r"(a), "=r"(b)
        : "r"(q));
    lo = *reinterpret_cast<__half2*>(&a);
    hi = *reinterpret_cast<__half2*>(&b);
}

// RR rows' segment s at once: all weight and scale loads first, then the math for the first nr rows, so the
// rows' latencies overlap. Every rows[r] must point at a readable row (callers repeat a valid row for missing
// ones). Per row the operations and their order are those of seg_dot.
template <int FMT, int NM, int RR>
__device__ __forceinline__ void seg_dot_rows(const uint8_t* const (&rows)[RR], int nr, int cbytes, int s, int lane,
                                             const float4* xs4, int xrow4, int M, float (&acc)[RR][NM]) {
    constexpr int Q = Seg<FMT>::Q;
    uint4 w[RR];
    float sc[RR];
#pragma unroll
    for (int r = 0; r < RR; r++) {
        w[r] = *reinterpret_cast<const uint4*>(rows[r] + s * kSegBytes + 16 * lane);
        const int so = FMT == kFP8 ? 2 * (16 * s + (lane >> 1)) : 2 * (32 * s + lane);
        sc[r] = half_bits_to_float(*reinterpret_cast<const uint16_t*>(rows[r] + cbytes + so));
    }
    const float4* xb = xs4 + s * Q * 32 + lane;
#pragma unroll
    for (int m = 0; m < NM; m++) {
        if (m >= M) break;
        const float4* xm = xb + m * xrow4;
        float4 xv[Q];
#pragma unroll
        for (int q = 0; q < Q; q++) xv[q] = xm[32 * q];
#pragma unroll
        for (int r = 0; r < RR; r++) {
            if (r >= nr) break;  // rows past nr were only loaded (their loads keep the pass branch-free)
            const uint32_t wd[4] = {w[r].x, w[r].y, w[r].z, w[r].w};
            if (FMT == kFP8) {  // hardware decode: sums are 256 x those of seg_dot (kFp8HwFactor)
                float p0 = 0.0f, p1 = 0.0f;
#pragma unroll
                for (int i = 0; i < 4; i++) {
                    __half2 a, b;
                    e4m3x4_to_half2(wd[i], a, b);
                    const float2 fa = __half22float2(a), fb = __half22float2(b);
                    float& p = (i & 1) ? p1 : p0;
                    p = fmaf(xv[i].x, fa.x, p);
                    p = fmaf(xv[i].y, fa.y, p);
                    p = fmaf(xv[i].z, fb.x, p);
                    p = fmaf(xv[i].w, fb.y, p);
                }
                acc[r][m] = fmaf(sc[r], p0 + p1, acc[r][m]);
            } else {
                float p0 = 0.0f, p1 = 0.0f;
#pragma unroll
                for (int i = 0; i < 4; i++) {
                    const float2 le = __half22float2(fp4x2_to_half2(wd[i] & 0x000F000Fu));
                    const float2 lo = __half22float2(fp4x2_to_half2((wd[i] >> 8) & 0x000F000Fu));
                    const float2 he = __half22float2(fp4x2_to_half2((wd[i] >> 4) & 0x000F000Fu));
                    const float2 ho = __half22float2(fp4x2_to_half2((wd[i] >> 12) & 0x000F000Fu));
                    p0 = dot4(xv[i], le, lo, p0);
                    p1 = dot4(xv[Q / 2 + i], he, ho, p1);
                }
                acc[r][m] = fmaf(sc[r], p0 + p1, acc[r][m]);
            }
        }
    }
}

// RR weight rows (stage pointers wr, all readable, the first nr real) against the M (<= NM) staged activations.
template <int FMT, int NM, int RR>
__device__ __forceinline__ void dot_rows(const uint8_t* const (&wr)[RR], int nr, int cbytes, int nseg,
                                         const float* xs, int xrow, int M, int lane, float (&acc)[RR][NM]) {
#pragma unroll
    for (int r = 0; r < RR; r++)
#pragma unroll
        for (int m = 0; m < NM; m++) acc[r][m] = 0.0f;
    const float4* xs4 = reinterpret_cast<const float4*>(xs);
    for (int s = 0; s < nseg; s++) {
        if (s * kSegBytes + 16 * lane >= cbytes) continue;  // lanes past the end of a partial last segment
        seg_dot_rows<FMT, NM, RR>(wr, nr, cbytes, s, lane, xs4, xrow / 4, M, acc);
    }
}

// Where a warp's current row lies in the producer's stages, advanced without divisions: stage s of the
// phase (ring slot, mbarrier parity) and row o inside it.
struct RowWalk {
    int s, o, slot, par;
    __device__ __forceinline__ void advance(int k, int rps, int nslot) {
        o += k;
        while (o >= rps) {
            o -= rps;
            s++;
            if (++slot == nslot) {
                slot = 0;
                par ^= 1;
            }
        }
    }
};

}  // namespace neko
