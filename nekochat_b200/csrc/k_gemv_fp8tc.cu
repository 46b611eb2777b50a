// Dequantising GEMV for 1..4 FP8 activation rows on the tensor cores (mma.sync m16n8k16, f16 x f16 -> f32): the
// MatmulQ8 dispatch (matmul_q8.comp; cpu::matmul, cpu_ops.cpp:462-481) at decode batch 1 to 4.
//
// 16 weight rows are the A operand, the activations the B operand: column 2 m holds the f16 rounding hi of
// activation row m, column 2 m + 1 the f16 rounding of the remainder lo (x = hi + lo to about 22 bits). The
// engine's FP8 code is e4m3 (gemv_core.cuh), so the hardware e4m3 -> f16 conversion gives each weight code's value
// exactly; products are exact in the MMA's fp32 accumulation. Each 32-weight block's f16 scale multiplies the
// block's sums in fp32, as in the CUDA-core kernel.
//
// The weights go from HBM straight into the MMA registers, with no shared-memory staging (at these sizes plain
// loads from many warps reach HBM bandwidth sooner than a bulk-copy ring):
//  * a warp takes a tile of 16 rows; in 64-byte spans (two quantisation blocks) lane (g, t) loads bytes
//    [8 t, 8 t + 8) of each block of rows g and g + 8: 8 rows x 2 x 32 contiguous bytes per four loads;
//  * the MMA's K order is free as long as A and B agree, so lane t's k slots are its own bytes: block k of the
//    span is two MMAs, the first on the lane's bytes 8t .. 8t + 3, the second on 8t + 4 .. 8t + 7, and the lane's
//    B registers hold the same four activations of its column (one 128-bit shared-memory load per block);
//  * two spans' batches are in flight per warp (the next batch's loads go out before this one's MMAs);
//  * tiles are dealt round-robin over all warps of the grid (phase 0: whole tiles, one warp each); the tiles
//    left over after the last full round (phase 1) are dealt round-robin over the CTAs and split over the K
//    dimension, q warps each, so that the tail is one short round on every SM; the q partial sums meet in shared
//    memory and are added in K order.
#include <algorithm>

#include "gemv_core.cuh"
#include "mma_frag.cuh"
#include "neko_common.cuh"
#include "neko_internal.h"

namespace neko {

namespace {

constexpr int kEW = 16;              // warps per CTA (one CTA per SM)
constexpr int kENT = kEW * 32;
constexpr int kEMaxM = 4;            // activation rows (2 B columns each)
constexpr int kENB = 4;              // spans loaded ahead per warp

// Dynamic shared memory: EShared | B columns (2 M x xp bytes). The per-CTA arrays live in the dynamic region:
// file-scope __shared__ arrays are placed by the device linker in one window shared with the other files' and
// would make this kernel's static shared memory depend on them.
extern __shared__ __align__(128) uint8_t esm[];
struct EShared {
    float part[kEW][2][kEMaxM][16];  // [warp][gate | up][activation row][tile row]
    double stat[kEMaxM][kEW][2];     // norm sums per warp
    float max[kEMaxM][kEW];          // largest magnitude per warp
    unsigned long long key[kEMaxM];
    int last;
};
constexpr int kEHdr = int(sizeof(EShared) + 127) / 128 * 128;  // bytes before the B columns
__device__ __forceinline__ EShared& esh() { return *reinterpret_cast<EShared*>(esm); }

struct E4Plan {
    int tiles;       // 16-row tiles
    int n0;          // tiles of phase 0: whole tiles, round-robin over every warp of the grid
    int tpc, q1;     // phase 1 (tiles n0 ..): at most tpc tiles per CTA (round-robin), each split q1 ways over K
    int xp;          // bytes per B column (2 K + 64)
};

__device__ __forceinline__ void esync() { asm volatile("bar.sync 1, %0;" ::"n"(kENT) : "memory"); }
__device__ __forceinline__ void tile_sync(int tile, int threads) {
    asm volatile("bar.sync %0, %1;" ::"r"(2 + tile), "r"(threads) : "memory");
}

__device__ __forceinline__ double wsum_e(double v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

__device__ __forceinline__ uint2 ldg_stream64(const uint8_t* p) {
    uint2 v;
    asm volatile("ld.global.nc.L1::no_allocate.v2.u32 {%0,%1}, [%2];" : "=r"(v.x), "=r"(v.y) : "l"(p));
    return v;
}

__device__ __forceinline__ uint32_t ld_nc_u32(const uint8_t* p) {
    uint32_t v;
    asm volatile("ld.global.nc.u32 %0, [%1];" : "=r"(v) : "l"(p));
    return v;
}

// The M activation rows (with the norm prologue, sums in double as in cpu_ops.cpp:483-511), each divided by a power
// of two s[m] that puts its largest magnitude in [2^14, 2^15) (inside f16's range, whatever the row's scale), as
// f16 hi / lo pairs (x / s = hi + lo, about 22 bits): B column 2 m = hi, 2 m + 1 = lo of activation row m, at
// xh + n * xp bytes, in natural K order. Reads x straight from global memory (a few KB, L2-resident).
__device__ void stage_hilo(const GemvArgs& a, int xp, uint8_t* xh, float (&s)[kEMaxM], int warp, int lane) {
    const int tid = threadIdx.x, K4 = a.K / 4, total = a.M * K4;
    float r[kEMaxM], mean[kEMaxM];
#pragma unroll
    for (int m = 0; m < kEMaxM; m++) r[m] = 1.0f, mean[m] = 0.0f;
    if (a.norm != kNormNone) {
        double s1[kEMaxM], s2[kEMaxM];
#pragma unroll
        for (int m = 0; m < kEMaxM; m++) s1[m] = s2[m] = 0.0;
        for (int i = tid; i < total; i += kENT) {
            const int m = i / K4, k = 4 * (i - m * K4);
            const float4 v = *reinterpret_cast<const float4*>(a.x + int64_t(m) * a.x_stride + k);
            const double d1 = double(v.x) + double(v.y) + double(v.z) + double(v.w);
            const double d2 = double(v.x) * v.x + double(v.y) * v.y + double(v.z) * v.z + double(v.w) * v.w;
#pragma unroll
            for (int mm = 0; mm < kEMaxM; mm++)
                if (mm == m) {
                    s1[mm] += d1;
                    s2[mm] += d2;
                }
        }
#pragma unroll
        for (int m = 0; m < kEMaxM; m++) {
            const double t1 = wsum_e(s1[m]), t2 = wsum_e(s2[m]);
            if (lane == 0) {
                esh().stat[m][warp][0] = t1;
                esh().stat[m][warp][1] = t2;
            }
        }
        esync();
#pragma unroll
        for (int m = 0; m < kEMaxM; m++) {
            double a1 = 0.0, a2 = 0.0;
            for (int w = 0; w < kEW; w++) {
                a1 += esh().stat[m][w][0];
                a2 += esh().stat[m][w][1];
            }
            if (a.norm == kNormRms) {
                r[m] = float(1.0 / sqrt(a2 / a.K + double(a.eps)));
            } else {
                const double mu = a1 / a.K;
                mean[m] = float(mu);
                r[m] = float(1.0 / sqrt(a2 / a.K - mu * mu + double(a.eps)));
            }
        }
    }
    auto load = [&](int i, int& m, int& k) {
        m = i / K4;
        k = 4 * (i - m * K4);
        float4 y = *reinterpret_cast<const float4*>(a.x + int64_t(m) * a.x_stride + k);
        if (a.norm != kNormNone) {
            float rm = r[0], mm = mean[0];
#pragma unroll
            for (int q = 1; q < kEMaxM; q++)
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
        return y;
    };
    float mx[kEMaxM];
#pragma unroll
    for (int m = 0; m < kEMaxM; m++) mx[m] = 0.0f;
    for (int i = tid; i < total; i += kENT) {  // largest magnitude per activation row
        int m, k;
        const float4 y = load(i, m, k);
        const float v = fmaxf(fmaxf(fabsf(y.x), fabsf(y.y)), fmaxf(fabsf(y.z), fabsf(y.w)));
#pragma unroll
        for (int q = 0; q < kEMaxM; q++)
            if (q == m) mx[q] = fmaxf(mx[q], v);
    }
#pragma unroll
    for (int m = 0; m < kEMaxM; m++) {
        const float v = warp_max(mx[m]);
        if (lane == 0) esh().max[m][warp] = v;
    }
    esync();
    float inv[kEMaxM];
#pragma unroll
    for (int m = 0; m < kEMaxM; m++) {
        float v = 0.0f;
        for (int w = 0; w < kEW; w++) v = fmaxf(v, esh().max[m][w]);
        const int F = int((__float_as_uint(v) >> 23) & 0xFF) - 127;  // v in [2^F, 2^(F+1)) (v = 0: any scale)
        const int e = max(-126, min(127, F - 14)), ie = max(-126, min(127, -e));
        s[m] = __uint_as_float(uint32_t(e + 127) << 23);
        inv[m] = __uint_as_float(uint32_t(ie + 127) << 23);
    }
    for (int i = tid; i < total; i += kENT) {
        int m, k;
        float4 y = load(i, m, k);
        float iv = inv[0];
#pragma unroll
        for (int q = 1; q < kEMaxM; q++)
            if (q == m) iv = inv[q];
        y.x *= iv;  // exact (a power of two)
        y.y *= iv;
        y.z *= iv;
        y.w *= iv;
        uint32_t h0, l0, h1, l1;
        split_hilo(y.x, y.y, h0, l0);
        split_hilo(y.z, y.w, h1, l1);
        *reinterpret_cast<uint2*>(xh + (2 * m) * xp + 2 * k) = make_uint2(h0, h1);
        *reinterpret_cast<uint2*>(xh + (2 * m + 1) * xp + 2 * k) = make_uint2(l0, l1);
    }
    esync();
}

// One batch of kENB spans of rows g and g + 8, loaded ahead of its use: per span, the lane's 8 code bytes of each
// of the span's two blocks (bytes 8t .. 8t + 7 and 32 + 8t ..) and the two blocks' scales.
struct Batch {
    uint2 ag[kENB][2], ah[kENB][2];
    uint32_t sg[kENB], sh[kENB];
};

// Loads spans [s, s + kENB) of the rows at wg / wh (spans past ns - 1 repeat it; their sums are dropped).
__device__ __forceinline__ void load_batch(Batch& b, const uint8_t* wg, const uint8_t* wh, int cbytes, int s, int ns,
                                           int t) {
#pragma unroll
    for (int i = 0; i < kENB; i++) {
        const int sp = min(s + i, ns - 1);
#pragma unroll
        for (int k = 0; k < 2; k++) {
            b.ag[i][k] = ldg_stream64(wg + 64 * sp + 32 * k + 8 * t);
            b.ah[i][k] = ldg_stream64(wh + 64 * sp + 32 * k + 8 * t);
        }
        b.sg[i] = ld_nc_u32(wg + cbytes + 4 * sp);
        b.sh[i] = ld_nc_u32(wh + cbytes + 4 * sp);
    }
}

// Lane (g, t)'s sums of a loaded batch (spans s .. up to s1) into c0 (row g) and c1 (row g + 8) for activation row
// t (columns 2t = hi, 2t + 1 = lo). xq: this lane's B column (nullptr: a column past 2 M, whose B operand is
// zero). Per block, two m16n8k16 MMAs: lane t's k slots (2t, 2t + 1, 2t + 8, 2t + 9) are its code bytes 8t + 4j
// .. 8t + 4j + 3 of MMA j, and its B registers the same four activations of its column.
__device__ __forceinline__ void batch_sums(const Batch& b, int s, int s1, const uint8_t* xq, int t, float& c0,
                                           float& c1) {
#pragma unroll
    for (int i = 0; i < kENB; i++) {
        if (s + i >= s1) break;
        const float2 fg = __half22float2(*reinterpret_cast<const __half2*>(&b.sg[i]));
        const float2 fh = __half22float2(*reinterpret_cast<const __half2*>(&b.sh[i]));
#pragma unroll
        for (int k = 0; k < 2; k++) {
            uint4 xv = make_uint4(0u, 0u, 0u, 0u);
            if (xq) xv = *reinterpret_cast<const uint4*>(xq + 2 * (64 * (s + i) + 32 * k + 8 * t));
            __half2 g0, g1, g2, g3, h0, h1, h2, h3;
            e4m3x4_to_half2(b.ag[i][k].x, g0, g1);
            e4m3x4_to_half2(b.ag[i][k].y, g2, g3);
            e4m3x4_to_half2(b.ah[i][k].x, h0, h1);
            e4m3x4_to_half2(b.ah[i][k].y, h2, h3);
            float d[4];
            const uint32_t a0[4] = {h2u(g0), h2u(h0), h2u(g1), h2u(h1)};
            const uint32_t a1[4] = {h2u(g2), h2u(h2), h2u(g3), h2u(h3)};
            mma16816_z(d, a0, xv.x, xv.y);
            mma16816(d, a1, xv.z, xv.w);
            const float sgk = k ? fg.y : fg.x, shk = k ? fh.y : fh.x;
            c0 = fmaf(sgk, d[0] + d[1], c0);
            c1 = fmaf(shk, d[2] + d[3], c1);
        }
    }
}

// Lane (g, t)'s sums over spans [s0, s1) of the tile whose rows g and g + 8 start at wg and wh (acc[0] row g,
// acc[1] row g + 8), batch by batch.
__device__ __forceinline__ void tile_sums(const uint8_t* wg, const uint8_t* wh, int cbytes, int s0, int s1,
                                          const uint8_t* xq, float (&acc)[2]) {
    const int t = threadIdx.x & 3;
    float c0 = 0.0f, c1 = 0.0f;
    for (int s = s0; s < s1; s += kENB) {
        Batch b;
        load_batch(b, wg, wh, cbytes, s, s1, t);
        batch_sums(b, s, s1, xq, t, c0, c1);
    }
    acc[0] = c0;
    acc[1] = c1;
}

// Output of a finished tile: lane (g, t) holds activation row m = t's sums for rows g, g + 8 (v[u][h]: gate or only
// row u = 0, up row u = 1), of the row divided by sc.
__device__ __forceinline__ void tile_store(const GemvArgs& a, int row0, const float (&v)[2][2], float sc, int m,
                                           int g, unsigned long long& best) {
    const bool pair = a.pair_off != 0;
#pragma unroll
    for (int h = 0; h < 2; h++) {
        const int row = row0 + g + 8 * h;
        if (row >= a.rows) continue;
        float* dst = a.y + int64_t(m) * a.y_stride + a.n_off + row;
        float val;
        if (pair) {
            const float gs = v[0][h] * sc, us = v[1][h] * sc;
            val = gs / (1.0f + expf(-gs)) * us;  // cpu::siluMul (cpu_ops.cpp:526-533)
        } else {
            val = v[0][h] * sc;
            if (a.flags & kBias) val += a.bias[row];
            if (a.flags & kGelu) val = gelu(val);
            if (a.flags & kAccumulate) val += *dst;
        }
        *dst = val;
        if (a.argmax) best = max(best, argmax_key(val, row));
    }
}

__global__ void __launch_bounds__(kENT, 1) gemv_fp8_tc_kernel(const GemvArgs a, const E4Plan p) {
    uint8_t* xh = esm + kEHdr;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
    const bool pair = a.pair_off != 0;
    const int rb = int(a.row_bytes), cbytes = a.K, ns = a.K / 64;
    if (threadIdx.x < kEMaxM) esh().key[threadIdx.x] = 0ull;
    auto rows_of = [&](int tile, int u, const uint8_t*& wg, const uint8_t*& wh) {
        const int r = 16 * tile + g;
        const int64_t base = u ? a.pair_off : 0;
        wg = a.W + (base + min(r, a.rows - 1)) * rb;  // rows past the end repeat the last (never stored)
        wh = a.W + (base + min(r + 8, a.rows - 1)) * rb;
    };
    // phase 0: whole tiles, one warp each, round-robin over the grid's warps. A warp's tiles are one sequence of
    // batches (a tile: nb batches of its gate or only rows, then nb of its up rows), software-pipelined: the next
    // batch's loads are issued before the current one's MMAs, so each warp keeps two batches in flight. The first
    // batch (weights only) is loaded before waiting for the previous kernel.
    const int nw = gridDim.x * kEW, nb = (ns + kENB - 1) / kENB, nbt = nb * (pair ? 2 : 1);
    const int F = p.n0 / nw * nbt;  // batches of this warp
    int lt = blockIdx.x * kEW + warp, lb = 0;  // next batch to load: tile, batch in the tile
    auto load_next = [&](Batch& b) {
        const int u = lb >= nb ? 1 : 0;
        const uint8_t *wg, *wh;
        rows_of(lt, u, wg, wh);
        load_batch(b, wg, wh, cbytes, (lb - u * nb) * kENB, ns, t);
        if (++lb == nbt) {
            lb = 0;
            lt += nw;
        }
    };
    Batch b0, b1;
    if (F > 0) load_next(b0);
    pdl_trigger();
    pdl_wait();  // the activations come from the previous kernel
    float sc[kEMaxM];
    stage_hilo(a, p.xp, xh, sc, warp, lane);
    // B: column g = hi (g even) or lo (g odd) of activation row g >> 1 (none past 2 M)
    const uint8_t* xq = g < 2 * a.M ? xh + g * p.xp : nullptr;
    const bool out_lane = t < a.M;  // lane (g, t) holds activation row t's sums
    float sl = sc[0];
#pragma unroll
    for (int q = 1; q < kEMaxM; q++)
        if (q == t) sl = sc[q];
    unsigned long long best = 0ull;
    {
        int ct = blockIdx.x * kEW + warp, cb = 0;  // next batch to add up
        float c[2][2] = {{0.0f, 0.0f}, {0.0f, 0.0f}};
        auto add_next = [&](const Batch& b) {
            const int u = cb >= nb ? 1 : 0;
            batch_sums(b, (cb - u * nb) * kENB, ns, xq, t, c[u][0], c[u][1]);
            if (++cb == nbt) {  // the tile is complete
                if (out_lane) tile_store(a, 16 * ct, c, sl, t, g, best);
                c[0][0] = c[0][1] = c[1][0] = c[1][1] = 0.0f;
                cb = 0;
                ct += nw;
            }
        };
        for (int f = 0; f < F; f += 2) {
            if (f + 1 < F) load_next(b1);
            add_next(b0);
            if (f + 1 >= F) break;
            if (f + 2 < F) load_next(b0);
            add_next(b1);
        }
    }
    // phase 1: the remaining tiles, dealt round-robin over the CTAs (at most tpc each), each split over q1 warps
    // along K
    {
        const int tl = warp / p.q1, ks = warp % p.q1;
        const int tile = p.n0 + tl * gridDim.x + blockIdx.x;
        if (tl < p.tpc && tile < p.tiles) {  // uniform over the tile's q1 warps
            const int s0 = ks * ns / p.q1, s1 = (ks + 1) * ns / p.q1;
            float v[2][2] = {{0.0f, 0.0f}, {0.0f, 0.0f}};
#pragma unroll
            for (int u = 0; u < 2; u++) {
                if (u == 1 && !pair) break;
                const uint8_t *wg, *wh;
                rows_of(tile, u, wg, wh);
                if (s0 < s1) tile_sums(wg, wh, cbytes, s0, s1, xq, v[u]);
            }
            if (p.q1 > 1) {  // partial sums through shared memory, added in K order by the tile's first warp
                if (out_lane)
#pragma unroll
                    for (int u = 0; u < 2; u++) {
                        esh().part[warp][u][t][g] = v[u][0];
                        esh().part[warp][u][t][g + 8] = v[u][1];
                    }
                tile_sync(tl, p.q1 * 32);
                if (ks == 0 && out_lane)
#pragma unroll
                    for (int u = 0; u < 2; u++) {
                        float x0 = 0.0f, x1 = 0.0f;
                        for (int k = 0; k < p.q1; k++) {
                            x0 += esh().part[warp + k][u][t][g];
                            x1 += esh().part[warp + k][u][t][g + 8];
                        }
                        v[u][0] = x0;
                        v[u][1] = x1;
                    }
            }
            if (ks == 0 && out_lane) tile_store(a, 16 * tile, v, sl, t, g, best);
        }
    }
    if (a.argmax) {  // lanes of the same t (activation row t), then per CTA, then one global atomic per row
        best = max(best, __shfl_xor_sync(0xffffffffu, best, 4));
        best = max(best, __shfl_xor_sync(0xffffffffu, best, 8));
        best = max(best, __shfl_xor_sync(0xffffffffu, best, 16));
        if (g == 0 && out_lane && best) atomicMax(&esh().key[t], best);
        esync();
        if (threadIdx.x < a.M && esh().key[threadIdx.x]) atomicMax(a.argmax + threadIdx.x, esh().key[threadIdx.x]);
        if (a.fin_count) {  // the last CTA: every other CTA's keys are in (each fenced before counting itself)
            __threadfence();
            esync();
            if (threadIdx.x == 0) esh().last = atomicAdd(a.fin_count, 1u) == gridDim.x - 1 ? 1 : 0;
            esync();
            if (esh().last) {
                __threadfence();
                if (threadIdx.x < a.M) {
                    const int m = threadIdx.x;
                    const unsigned long long key = atomicExch(a.argmax + m, 0ull);
                    int idx = int(0xFFFFFFFFu - unsigned(key & 0xFFFFFFFFull));
                    if (idx < 0 || idx >= a.rows) {  // no logit was reduced
                        set_device_error(kErrBadIndex);
                        idx = 0;
                    }
                    a.fin_argmax[m] = idx;
                    if (a.fin_advance) {
                        a.fin_tokens[m] = idx;
                        if (a.fin_pos[m] + 1 < a.fin_context) a.fin_pos[m] += 1;
                        else set_device_error(kErrBadIndex);
                    }
                }
                if (threadIdx.x == 0) *a.fin_count = 0u;
            }
        }
    }
}

}  // namespace

// The tensor-core GEMV for 1..4 FP8 activation rows: one CTA of 16 warps per SM. Phase 0 takes the full rounds
// of 16-row tiles (one warp per tile), phase 1 the rest in one round: tpc = the leftover tiles per CTA (rounded
// up), each split over q1 = 16 / tpc warps. cudaErrorNotSupported (nothing launched) when the call does not fit:
// K a multiple of 128, rows a multiple of 16 bytes, weights and activations 16-byte aligned.
cudaError_t launch_gemv_fp8_tc(const GemvArgs& a, cudaStream_t st, bool pdl) {
    if (a.fmt != kFP8 || a.M < 1 || a.M > kEMaxM || a.K % 128 || a.row_bytes % 16) return cudaErrorNotSupported;
    if (a.x_stride % 4 || (reinterpret_cast<uintptr_t>(a.x) & 15)) return cudaErrorNotSupported;
    if (a.argmax && a.pair_off) return cudaErrorNotSupported;
    if ((reinterpret_cast<uintptr_t>(a.W) & 15) || (a.pair_off * a.row_bytes) % 16) return cudaErrorNotSupported;
    E4Plan p{};
    p.tiles = (a.rows + 15) / 16;
    const int sms = num_sms(), nw = sms * kEW;
    p.n0 = p.tiles / nw * nw;
    const int rem = p.tiles - p.n0;
    p.tpc = std::max(1, (rem + sms - 1) / sms);
    p.q1 = kEW / p.tpc;
    const int ctas = p.n0 ? sms : std::max(1, std::min(sms, rem));
    p.xp = 2 * a.K + 64;
    const size_t smem = kEHdr + size_t(2 * a.M) * p.xp;
    if (const cudaError_t e = ensure_dyn_smem(gemv_fp8_tc_kernel, smem); e != cudaSuccess) return e;
    return launch_ex(gemv_fp8_tc_kernel, dim3(ctas), dim3(kENT), smem, st, pdl, a, p);
}

}  // namespace neko
