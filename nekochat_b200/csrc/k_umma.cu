// Dequant matmul on the 5th-generation tensor cores (tcgen05 / UMMA, TMEM accumulators) for 128+ activation rows
// (prefill chunks): the MatmulQ8 / MatmulQ4 dispatch (matmul_q8.comp, matmul_q4.comp;
// cpu::matmul, cpu_ops.cpp:462-481) where the multiply-adds are the cost.
//
// y[m][n] (+)= act(x[m] . deq(W[n]) + b[n]) with the precision of the fp32 kernels:
//  * each weight enters as its dequantised value w = code x scale (QMatrix::dequantizeRow's product, exact in fp32
//    with at most 15 significant bits) split into two f16, w = w_hi + w_lo: w_hi = f16(code x scale) (hmul),
//    w_lo = fma(code, scale, -w_hi) (the exact residual, rounded only when it falls below f16's subnormal step,
//    an absolute error under 3e-8 per weight). Folding the block scale into the operand lets TMEM accumulate over
//    all of K, with no per-block rescaling;
//  * the activations arrive split into hi + lo f16 (split_act_kernel / norm_split_kernel, about 22 bits);
//  * D = x_hi w_hi + x_lo w_hi + x_hi w_lo (three UMMAs per 16-wide K step; x_lo w_lo is below 2^-22 relative),
//    fp32 in TMEM.
// CTA tile: 128 activation rows (UMMA M = 128; rows past M are zero) x BN = 64 / 128 weight rows (SwiGLU: BN / 2
// gate + BN / 2 up rows), K in stages of 64 (one 128-byte swizzle atom of f16). Eight warps: every thread stages
// the activations (cp.async into the 128B-swizzled K-major layout) and converts the weight codes of a stage into
// the same layout; thread 0 issues the UMMAs and commits them to the stage's mbarrier, which frees the stage's
// buffers for a later stage (3 buffers at BN = 128, 4 at BN = 64: the copies run 2 or 3 stages ahead). K is split over a thread-block cluster when the tiles leave SMs
// idle (clusters of up to 4): each CTA moves its fp32 tile from TMEM to shared memory and CTA z sums rows z,
// z + ks, ... over the cluster in split order (deterministic), then runs the epilogue. All waits are bounded; TMEM is always freed.
#include <cooperative_groups.h>

#include <algorithm>
#include <cstdint>

#include "gemv_core.cuh"
#include "mma_frag.cuh"
#include "neko_common.cuh"
#include "neko_internal.h"
#include "tc5_core.cuh"
#include "tma_host.h"

namespace neko {

namespace {

constexpr int kUM = 128;       // activation rows per CTA (UMMA M)
constexpr int kUK = 64;        // K per stage: 64 f16 = one 128-byte swizzle atom
constexpr int kUMaxBufs = 4;   // f16 operand buffers (3 at BN = 128, 4 at BN = 64: shared memory)
constexpr int kUThreads = 256;
// CTAs of a split-K cluster. At ~210 KB of shared memory a CTA fills an SM, and clusters of 8 such CTAs only
// find room a few per GPC (measured: SMs active 38% of the kernel at M = 128, K = 3072, N = 1024); clusters of 4
// schedule freely (that shape 36.5 -> 30.3 us, M = 256: 47.5 -> 31.2 us).
constexpr int kUMaxSplit = 4;
// Below 128 rows the mma.sync kernel is faster (measured: M = 64 decode-layer shapes 27-31 us there vs 33 us
// here, where two stages of prefetch leave the pipeline latency-bound); from 128 rows on, this one (M = 512:
// 1.3-1.5x).
constexpr int kUMinRows = 128;

struct UmmaSplit {
    int ksplit, sper;
    const __half* xh;  // activations as f16 hi / lo, [M][K] each
    const __half* xl;
};

template <int FMT, int BN, bool PAIR>
struct UmmaSmem {
    static constexpr int kCode = FMT == kFP8 ? kUK : kUK / 2;            // code bytes per row per stage
    static constexpr int kATile = kUM * kUK * 2;                         // bytes of one f16 A tile
    static constexpr int kBTile = BN * kUK * 2;                          // bytes of one f16 B tile
    static constexpr int kBuf = 2 * kATile + 2 * kBTile;                 // A hi, A lo, B hi, B lo
    static constexpr int NB = BN == 64 ? 4 : 3;                          // operand buffers
    static constexpr int P = NB - 1;                                     // stages in flight ahead
    static constexpr int kRaw = BN * kCode + BN * 4;                     // codes + 2 scales per row
    static constexpr int kRawOff = NB * kBuf;
    static constexpr int kBytes = kRawOff + P * kRaw;                    // + P raw code buffers
    static constexpr int kTilePitch = BN + 4;                            // epilogue fp32 tile pitch
    static_assert(NB <= kUMaxBufs, "barriers");
    static_assert(kUM * kTilePitch * 4 <= NB * kBuf, "epilogue tile fits the operand buffers");
};

// After the UMMAs of a CTA: TMEM (BN fp32 columns x 128 lanes at tmem) -> the CTA's fp32 tile in shared memory
// (usm, pitch BN + 4), TMEM freed, then (ks > 1) the K splits of the cluster summed in split order, rows z,
// z + ks, ... per CTA, and the epilogue: bias / GELU / accumulate or SiLU * up, greedy argmax keys. ok = false
// (a bounded wait gave up) writes zeros and records the error.
template <int BN, bool PAIR>
__device__ __forceinline__ void umma_finish(const GemvArgs& a, int ks, int z, int n0, int m0, int mv, uint32_t tmem,
                                            uint8_t* usm, bool ok, bool failed, unsigned long long* keys) {
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    constexpr int TP = BN + 4;
    float* tile = reinterpret_cast<float*>(usm);
    {
        const int quarter = warp & 3, row = 32 * quarter + lane;
        constexpr int kHalf = BN / (kUThreads / 128);  // columns per warp of a lane quarter
#pragma unroll 1
        for (int c0 = (warp >> 2) * kHalf; c0 < (warp >> 2) * kHalf + kHalf; c0 += 16) {
            float v[16];
            if (ok) tmem_ld16(tmem + (uint32_t(32 * quarter) << 16) + uint32_t(c0), v);
            else
#pragma unroll
                for (int u = 0; u < 16; u++) v[u] = 0.0f;
#pragma unroll
            for (int u = 0; u < 16; u += 4)
                *reinterpret_cast<float4*>(tile + row * TP + c0 + u) = make_float4(v[u], v[u + 1], v[u + 2], v[u + 3]);
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0)
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(BN) : "memory");
    namespace cg = cooperative_groups;
    if (ks > 1) cg::this_cluster().sync();  // every split's tile is in place
    if (failed) set_device_error(kErrMbarTimeout);

    // rows z, z + ks, ...: the splits summed in order, then bias / GELU / accumulate or SiLU * up
    constexpr int OC = PAIR ? BN / 2 : BN;
    const float* peer[kUMaxSplit];
#pragma unroll
    for (int zz = 0; zz < kUMaxSplit; zz++)
        peer[zz] = zz < ks ? (ks > 1 ? cg::this_cluster().map_shared_rank(tile, zz) : tile) : tile;
    if (a.argmax && tid < kUM) keys[tid] = 0ull;  // [kUM] argmax keys of the CTA's rows
    __syncthreads();
    const int nrow = (mv - z + ks - 1) / ks;
    static_assert(OC % 32 == 0, "a warp's 32 elements share a row");
    for (int i = tid; i < nrow * OC; i += kUThreads) {
        const int row = z + ks * (i / OC), col = i - (i / OC) * OC;
        const int m = m0 + row, n = n0 + col;
        float v = 0.0f, u = 0.0f;
#pragma unroll
        for (int zz = 0; zz < kUMaxSplit; zz++) {
            if (zz >= ks) break;
            v += peer[zz][row * TP + col];
            if (PAIR) u += peer[zz][row * TP + BN / 2 + col];
        }
        unsigned long long key = 0ull;
        if (n < a.rows) {
            float* dst = a.y + int64_t(m) * a.y_stride + a.n_off + n;
            float val = v;
            if (PAIR) {
                val = val / (1.0f + expf(-val)) * u;  // cpu::siluMul (cpu_ops.cpp:526-533)
            } else {
                if (a.flags & kBias) val += a.bias[n];
                if (a.flags & kGelu) val = gelu(val);
                if (a.flags & kAccumulate) val += *dst;
            }
            *dst = val;
            key = argmax_key(val, n);
        }
        if (a.argmax) {
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) key = max(key, __shfl_xor_sync(0xffffffffu, key, o));
            if (lane == 0 && key) atomicMax(&keys[row], key);
        }
    }
    if (a.argmax) {
        __syncthreads();
        if (tid < nrow && keys[z + ks * tid]) atomicMax(a.argmax + m0 + z + ks * tid, keys[z + ks * tid]);
    }
    if (ks > 1) cg::this_cluster().sync();  // no CTA leaves while a peer may still read its tile
}

template <int FMT, int BN, bool PAIR>
__global__ void __launch_bounds__(kUThreads, 1) umma_gemm_kernel(const GemvArgs a, const UmmaSplit sp) {
    using L = UmmaSmem<FMT, BN, PAIR>;
    extern __shared__ uint8_t usm_raw[];
    __shared__ uint64_t mma_bar[kUMaxBufs];
    constexpr int NB = L::NB, P = L::P;
    __shared__ uint32_t tmem_base;
    __shared__ int s_fail;
    // operand tiles need 1024-byte alignment (the swizzle pattern is anchored on address bits 7..9)
    uint8_t* usm = usm_raw + ((1024 - (smem_u32(usm_raw) & 1023)) & 1023);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int n0 = blockIdx.x * (PAIR ? BN / 2 : BN), m0 = blockIdx.y * kUM, z = blockIdx.z;
    const int mv = min(kUM, a.M - m0);
    const int cbytes = FMT == kFP8 ? a.K : a.K / 2;
    const int s_begin = z * sp.sper, nst = min(a.K / kUK, s_begin + sp.sper) - s_begin;
    constexpr uint32_t kIdesc = f16_idesc(kUM, BN);

    if (warp == 0) {  // TMEM: BN fp32 columns x 128 lanes
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&tmem_base)),
                     "r"(BN)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    if (tid == 0) {
        for (int b = 0; b < NB; b++) mbar_init(&mma_bar[b], 1);
        fence_barrier_init();
        // the descriptors assume 1024-byte aligned tiles; a misaligned base (static shared variables sit beside
        // the run-time aligned dynamic block) is recorded and the UMMAs are skipped
        s_fail = (smem_u32(usm) & 1023u) ? 1 : 0;
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = tmem_base;

    // weight row r of the tile (SwiGLU: gate rows, then up rows) -> packed row (rows past the end repeat the last)
    auto wrow = [&](int r) -> const uint8_t* {
        const int n = PAIR ? (r < BN / 2 ? n0 + r : n0 + (r - BN / 2)) : n0 + r;
        const int nc = min(n, a.rows - 1);
        return a.W + (int64_t(nc) + (PAIR && r >= BN / 2 ? a.pair_off : 0)) * a.row_bytes;
    };
    auto buf = [&](int i) { return usm + (i % NB) * L::kBuf; };
    auto raw = [&](int i) { return usm + L::kRawOff + (i % P) * L::kRaw; };
    // weight codes + scales of stage i (index within this CTA's range) -> raw buffer i % P
    auto issue_w = [&](int i) {
        const int s = s_begin + i;
        uint8_t* rb = raw(i);
        constexpr int kPieces = L::kCode / 16;
        for (int j = tid; j < BN * kPieces; j += kUThreads) {
            const int r = j / kPieces, q = j - r * kPieces;
            cp16(rb + r * L::kCode + 16 * q, wrow(r) + s * L::kCode + 16 * q, 16);
        }
        for (int r = tid; r < BN; r += kUThreads) cp4(rb + BN * L::kCode + 4 * r, wrow(r) + cbytes + 4 * s);
    };
    // activations (hi, lo) of stage i -> the A tiles of buffer i, swizzled (rows past M stay zero: cleared once)
    auto issue_x = [&](int i) {
        const int s = s_begin + i;
        uint8_t* bb = buf(i);
        for (int j = tid; j < 2 * mv * 8; j += kUThreads) {
            const int h = j >= mv * 8 ? 1 : 0, jj = j - h * mv * 8, r = jj >> 3, q = jj & 7;
            cp16(bb + h * L::kATile + sw128_off(r, q), (h ? sp.xl : sp.xh) + int64_t(m0 + r) * a.K + s * kUK + 8 * q,
                 16);
        }
    };
    if (mv < kUM) {  // A rows past M: zero in every buffer, never written again
        for (int j = tid; j < NB * 2 * (kUM - mv) * 8; j += kUThreads) {
            const int b = j / (2 * (kUM - mv) * 8), jj = j - b * 2 * (kUM - mv) * 8;
            const int h = jj >= (kUM - mv) * 8 ? 1 : 0, k2 = jj - h * (kUM - mv) * 8, r = mv + (k2 >> 3), q = k2 & 7;
            *reinterpret_cast<uint4*>(usm + b * L::kBuf + h * L::kATile + sw128_off(r, q)) = make_uint4(0, 0, 0, 0);
        }
    }
    // raw buffer i % P -> B hi / lo tiles of buffer i: w = code x scale split into two f16
    auto convert = [&](int i) {
        const uint8_t* rb = raw(i);
        uint8_t* bb = buf(i) + 2 * L::kATile;
        for (int j = tid; j < BN * 8; j += kUThreads) {
            const int r = j >> 3, q = j & 7;  // row r, weights 8q .. 8q + 7 of the stage
            const uint16_t sbits = *reinterpret_cast<const uint16_t*>(rb + BN * L::kCode + 4 * r + 2 * (q >> 2));
            __half2 sc = __halves2half2(__ushort_as_half(sbits), __ushort_as_half(sbits));
            __half2 c[4];
            if (FMT == kFP8) {
                const uint2 w = *reinterpret_cast<const uint2*>(rb + r * L::kCode + 8 * q);
                e4m3x4_to_half2(w.x, c[0], c[1]);
                e4m3x4_to_half2(w.y, c[2], c[3]);
            } else {  // weights 8q.. of a 32-block: low nibbles of bytes 8(q%4).. (q%4 < 2) or high nibbles
                const int blk = q >> 2, j0 = 8 * (q & 3);
                const uint2 w = *reinterpret_cast<const uint2*>(rb + r * L::kCode + 16 * blk + (j0 & 15));
                const int sh = j0 >= 16 ? 4 : 0;
                const __half2 k16 = __float2half2_rn(kFp4Factor);  // engine FP4 decode (value / 16384) x 16384
                const uint32_t wd[2] = {w.x >> sh, w.y >> sh};
#pragma unroll
                for (int u = 0; u < 2; u++) {
                    const __half2 e = fp4x2_to_half2(wd[u] & 0x000F000Fu);         // weights 4u, 4u + 2
                    const __half2 o = fp4x2_to_half2((wd[u] >> 8) & 0x000F000Fu);  // weights 4u + 1, 4u + 3
                    c[2 * u] = __hmul2(__halves2half2(__low2half(e), __low2half(o)), k16);
                    c[2 * u + 1] = __hmul2(__halves2half2(__high2half(e), __high2half(o)), k16);
                }
            }
            uint32_t hi[4], lo[4];
#pragma unroll
            for (int u = 0; u < 4; u++) {
                const __half2 h = __hmul2(c[u], sc);
                hi[u] = h2u(h);
                lo[u] = h2u(__hfma2(c[u], sc, __hneg2(h)));
            }
            *reinterpret_cast<uint4*>(bb + sw128_off(r, q)) = make_uint4(hi[0], hi[1], hi[2], hi[3]);
            *reinterpret_cast<uint4*>(bb + L::kBTile + sw128_off(r, q)) = make_uint4(lo[0], lo[1], lo[2], lo[3]);
        }
    };
    // bounded wait for the UMMAs of stage i (their commit): their buffer is free / their results are in TMEM;
    // nothing to wait for when the alignment check failed (no UMMA is issued then)
    const bool issuing = !s_fail;
    auto mma_wait = [&](int i) {
        if (issuing && !mbar_wait(&mma_bar[i % NB], uint32_t(i / NB) & 1u)) s_fail = 1;
    };

    // prologue: stages 0 .. P - 1 (weights before the dependency wait: they never depend on the previous kernel;
    // one commit group per stage's activations, the first also holding every prologue weight copy)
#pragma unroll
    for (int j = 0; j < P; j++)
        if (j < nst) issue_w(j);
    pdl_wait();
#pragma unroll
    for (int j = 0; j < P; j++) {
        if (j < nst) issue_x(j);
        cp_commit();
    }
    for (int i = 0; i < nst; i++) {
        cp_wait<P - 1>();  // stage i landed (this thread's copies)
        __syncthreads();
        if (i >= NB) mma_wait(i - NB);  // buffer i % NB was last read by the UMMAs of stage i - NB
        convert(i);
        fence_proxy_async();  // generic-proxy writes (conversions, cp.async) -> visible to the tensor cores
        __syncthreads();
        if (tid == 0 && !s_fail) {
            tc_fence_after();
            const uint8_t* bb = buf(i);
            const uint32_t ah = smem_u32(bb), al = ah + L::kATile, bh = al + L::kATile, bl = bh + L::kBTile;
#pragma unroll
            for (int k = 0; k < kUK / 16; k++) {  // 16-wide K steps: 32 bytes into each swizzled row
                const uint32_t o = 32 * k;
                umma_f16(tmem, sw128_desc(ah + o), sw128_desc(bh + o), kIdesc, (i > 0 || k > 0) ? 1u : 0u);
                umma_f16(tmem, sw128_desc(al + o), sw128_desc(bh + o), kIdesc, 1u);
                umma_f16(tmem, sw128_desc(ah + o), sw128_desc(bl + o), kIdesc, 1u);
            }
            umma_commit(&mma_bar[i % NB]);
        }
        // stage i + P: its weights into the raw buffer just converted, its activations into buffer (i + P) % NB,
        // last read by the UMMAs of stage i - 1
        if (i + P < nst) {
            if (i >= 1) mma_wait(i - 1);
            issue_w(i + P);
            issue_x(i + P);
        }
        cp_commit();
    }
    // every UMMA of this CTA has completed (the last commit tracks all earlier ones)
    if (nst > 0) mma_wait(nst - 1);
    pdl_trigger();
    tc_fence_after();
    __syncthreads();

    __shared__ unsigned long long keys[kUM];
    umma_finish<BN, PAIR>(a, sp.ksplit, z, n0, m0, mv, tmem, usm, !s_fail && nst > 0, s_fail != 0, keys);
}

// ------------------------------------------------------------------------------------ dequantise, then GEMM
// From 256 activation rows on, each weight is converted once per call instead of once per CTA: a bandwidth-bound
// kernel writes w = code x scale as hi + lo f16 rows ([rows][K] each, 4 bytes per weight against the code's
// 1 / 0.5), then a plain f16 GEMM streams both operands with TMA tensor copies (128-byte swizzle, the K-major
// layout the UMMA descriptors read) through an mbarrier ring driven by one thread; no CTA barrier and no
// conversion in the K loop.
constexpr int kDqMinRows = 256;
constexpr int kDqStages = 3;  // 64 KB per stage (A hi / lo, B hi / lo at BN = 128)

// Weights 8q .. 8q + 7 of row r (i = r * K / 8 + q) as hi / lo f16: the arithmetic of umma_gemm_kernel's convert.
template <int FMT>
__global__ void dequant_hilo_kernel(const uint8_t* __restrict__ W, int64_t row_bytes, int rows, int K,
                                    __half* __restrict__ wh, __half* __restrict__ wl) {
    pdl_wait();  // the previous kernel may still read the buffers this one writes
    const int cbytes = FMT == kFP8 ? K : K / 2, q8 = K / 8;
    const int64_t n = int64_t(rows) * q8;
    for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < n; i += int64_t(gridDim.x) * blockDim.x) {
        const int r = int(i / q8), q = int(i - int64_t(r) * q8);
        const uint8_t* row = W + int64_t(r) * row_bytes;
        const uint16_t sbits = *reinterpret_cast<const uint16_t*>(row + cbytes + 2 * (q >> 2));
        const __half2 sc = __halves2half2(__ushort_as_half(sbits), __ushort_as_half(sbits));
        __half2 c[4];
        if (FMT == kFP8) {
            const uint2 w = *reinterpret_cast<const uint2*>(row + 8 * q);
            e4m3x4_to_half2(w.x, c[0], c[1]);
            e4m3x4_to_half2(w.y, c[2], c[3]);
        } else {  // weights 8(q % 4).. of 32-block q / 4: low nibbles of its bytes (q % 4 < 2), else high nibbles
            const int blk = q >> 2, j0 = 8 * (q & 3);
            const uint2 w = *reinterpret_cast<const uint2*>(row + 16 * blk + (j0 & 15));
            const int sh = j0 >= 16 ? 4 : 0;
            const __half2 k16 = __float2half2_rn(kFp4Factor);
            const uint32_t wd[2] = {w.x >> sh, w.y >> sh};
#pragma unroll
            for (int u = 0; u < 2; u++) {
                const __half2 e = fp4x2_to_half2(wd[u] & 0x000F000Fu);
                const __half2 o = fp4x2_to_half2((wd[u] >> 8) & 0x000F000Fu);
                c[2 * u] = __hmul2(__halves2half2(__low2half(e), __low2half(o)), k16);
                c[2 * u + 1] = __hmul2(__halves2half2(__high2half(e), __high2half(o)), k16);
            }
        }
        uint32_t hi[4], lo[4];
#pragma unroll
        for (int u = 0; u < 4; u++) {
            const __half2 h = __hmul2(c[u], sc);
            hi[u] = h2u(h);
            lo[u] = h2u(__hfma2(c[u], sc, __hneg2(h)));
        }
        const int64_t o = int64_t(r) * K + 8 * q;
        *reinterpret_cast<uint4*>(wh + o) = make_uint4(hi[0], hi[1], hi[2], hi[3]);
        *reinterpret_cast<uint4*>(wl + o) = make_uint4(lo[0], lo[1], lo[2], lo[3]);
    }
    pdl_trigger();
}

__device__ __forceinline__ void tma_load_2d_u(uint32_t dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], "
        "[%4];" ::"r"(dst),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
        : "memory");
}

// f16 hi / lo operands: A = activations [M][K] (maps ta_h, ta_l), B = dequantised weights [rows][K] (tb_h, tb_l;
// SwiGLU: the up rows at row pair_off + n). CTA tile 128 x BN (BN = 128; SwiGLU 64 gate + 64 up rows), K stages of
// 64 through kDqStages buffers; thread 0 issues the tensor copies and the UMMAs, every wait bounded.
template <int BN, bool PAIR>
__global__ void __launch_bounds__(kUThreads, 1)
    umma_dq_gemm_kernel(const GemvArgs a, const UmmaSplit sp, const __grid_constant__ CUtensorMap ta_h,
                        const __grid_constant__ CUtensorMap ta_l, const __grid_constant__ CUtensorMap tb_h,
                        const __grid_constant__ CUtensorMap tb_l) {
    constexpr int kA = kUM * kUK * 2, kB = BN * kUK * 2, kStage = 2 * kA + 2 * kB, NS = kDqStages;
    static_assert(kUM * (BN + 4) * 4 <= NS * kStage, "epilogue tile fits the stage buffers");
    extern __shared__ uint8_t usm_raw[];
    // operand tiles need 1024-byte alignment; barriers and flags follow the stages in the same dynamic block
    uint8_t* usm = usm_raw + ((1024 - (smem_u32(usm_raw) & 1023)) & 1023);
    uint64_t* full = reinterpret_cast<uint64_t*>(usm + NS * kStage);   // [NS] copies landed
    uint64_t* empty = full + NS;                                      // [NS] UMMAs done with the buffer
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(empty + NS);
    int* fail = reinterpret_cast<int*>(tmem_slot + 1);
    // argmax keys in the same block too: the kernel declares no static shared variables beside the run-time
    // aligned dynamic block
    unsigned long long* keys = reinterpret_cast<unsigned long long*>(usm + NS * kStage + 64);
    const int tid = threadIdx.x, warp = tid >> 5;
    const int n0 = blockIdx.x * (PAIR ? BN / 2 : BN), m0 = blockIdx.y * kUM, z = blockIdx.z;
    const int mv = min(kUM, a.M - m0);
    const int s_begin = z * sp.sper, nst = min(a.K / kUK, s_begin + sp.sper) - s_begin;
    constexpr uint32_t kIdesc = f16_idesc(kUM, BN);

    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(BN)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    if (tid == 0) {
        for (int b = 0; b < NS; b++) {
            mbar_init(&full[b], 1);
            mbar_init(&empty[b], 1);
        }
        fence_barrier_init();
        *fail = (smem_u32(usm) & 1023u) || (reinterpret_cast<uintptr_t>(&ta_h) & 63u) ? 1 : 0;
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    pdl_wait();  // activations, dequantised weights and the epilogue's operands come from the previous kernels

    if (tid == 0 && !*fail) {
        auto issue = [&](int t) {  // stage t's four tiles into buffer t % NS
            const uint32_t b = smem_u32(usm + (t % NS) * kStage);
            uint64_t* bar = &full[t % NS];
            const int k = (s_begin + t) * kUK;
            mbar_arrive_expect_tx(bar, uint32_t(kStage));
            tma_load_2d_u(b, &ta_h, k, m0, bar);
            tma_load_2d_u(b + kA, &ta_l, k, m0, bar);
            if (PAIR) {
                tma_load_2d_u(b + 2 * kA, &tb_h, k, n0, bar);
                tma_load_2d_u(b + 2 * kA + kB / 2, &tb_h, k, int(a.pair_off) + n0, bar);
                tma_load_2d_u(b + 2 * kA + kB, &tb_l, k, n0, bar);
                tma_load_2d_u(b + 2 * kA + kB + kB / 2, &tb_l, k, int(a.pair_off) + n0, bar);
            } else {
                tma_load_2d_u(b + 2 * kA, &tb_h, k, n0, bar);
                tma_load_2d_u(b + 2 * kA + kB, &tb_l, k, n0, bar);
            }
        };
        for (int t = 0; t < NS - 1 && t < nst; t++) issue(t);
        for (int i = 0; i < nst; i++) {
            if (!mbar_wait(&full[i % NS], uint32_t(i / NS) & 1u)) {
                *fail = 1;
                break;
            }
            tc_fence_after();
            const uint32_t ah = smem_u32(usm + (i % NS) * kStage), al = ah + kA, bh = al + kA, bl = bh + kB;
#pragma unroll
            for (int k = 0; k < kUK / 16; k++) {  // 16-wide K steps: 32 bytes into each swizzled row
                const uint32_t o = 32 * k;
                umma_f16(tmem, sw128_desc(ah + o), sw128_desc(bh + o), kIdesc, (i > 0 || k > 0) ? 1u : 0u);
                umma_f16(tmem, sw128_desc(al + o), sw128_desc(bh + o), kIdesc, 1u);
                umma_f16(tmem, sw128_desc(ah + o), sw128_desc(bl + o), kIdesc, 1u);
            }
            umma_commit(&empty[i % NS]);
            // stage i + NS - 1 into the buffer of stage i - 1, once its UMMAs are done (stage i is queued behind)
            const int t = i + NS - 1;
            if (t < nst) {
                if (t >= NS && !mbar_wait(&empty[t % NS], uint32_t(t / NS - 1) & 1u)) {
                    *fail = 1;
                    break;
                }
                issue(t);
            }
        }
        // every UMMA done (the last commit tracks all earlier ones); copies in flight have all been consumed
        if (!*fail && nst > 0 && !mbar_wait(&empty[(nst - 1) % NS], uint32_t((nst - 1) / NS) & 1u)) *fail = 1;
    }
    __syncthreads();
    pdl_trigger();
    tc_fence_after();
    const bool failed = *fail != 0;
    umma_finish<BN, PAIR>(a, sp.ksplit, z, n0, m0, mv, tmem, usm, !failed && nst > 0, failed, keys);
}

using UmmaFn = void (*)(const GemvArgs, const UmmaSplit);

template <int FMT>
UmmaFn pick_umma(int bn, bool pair) {
    if (pair) return bn == 128 ? umma_gemm_kernel<FMT, 128, true> : umma_gemm_kernel<FMT, 64, true>;
    return bn == 128 ? umma_gemm_kernel<FMT, 128, false> : umma_gemm_kernel<FMT, 64, false>;
}
template <int FMT>
size_t umma_smem(int bn, bool pair) {
    const int b = pair ? (bn == 128 ? UmmaSmem<FMT, 128, true>::kBytes : UmmaSmem<FMT, 64, true>::kBytes)
                       : (bn == 128 ? UmmaSmem<FMT, 128, false>::kBytes : UmmaSmem<FMT, 64, false>::kBytes);
    return size_t(b) + 1024;  // + alignment slack
}

}  // namespace

// 256+ rows with workspace room: dequantise the weights once (hi / lo f16 rows after the split activations in
// ws), then the TMA-fed f16 GEMM. cudaErrorNotSupported when the call does not qualify.
cudaError_t launch_gemm_umma_dq(const GemvArgs& a, const __half* xh, const __half* xl, cudaStream_t st, bool pdl) {
    const bool pair = a.pair_off != 0;
    const int64_t rtot = pair ? a.pair_off + a.rows : a.rows;  // matrix rows (SwiGLU: gate rows, then up rows)
    if (a.M < kDqMinRows || (a.fmt != kFP8 && a.fmt != kFP4) || a.K % kUK || !xh || !xl || !a.ws ||
        a.row_bytes % 16 || (a.pair_off && (a.argmax || a.pair_off < a.rows)) ||
        a.ws_floats < int64_t(a.M) * a.K + rtot * a.K || rtot >= (int64_t(1) << 31))
        return cudaErrorNotSupported;
    __half* wh = reinterpret_cast<__half*>(a.ws + int64_t(a.M) * a.K);
    __half* wl = wh + rtot * a.K;
    const int sms = num_sms();
    {
        const int64_t n = rtot * (a.K / 8);
        const int blocks = int(std::min<int64_t>((n + 255) / 256, 8 * sms));
        auto dq = a.fmt == kFP8 ? dequant_hilo_kernel<kFP8> : dequant_hilo_kernel<kFP4>;
        if (cudaError_t e = launch_ex(dq, dim3(blocks), dim3(256), 0, st, pdl, a.W, a.row_bytes, int(rtot), a.K, wh, wl);
            e != cudaSuccess)
            return e;
    }
    constexpr int BN = 128;
    CUtensorMap ta_h{}, ta_l{}, tb_h{}, tb_l{};
    const int brows = pair ? BN / 2 : BN;
    if (!encode_f16_2d_sw128(&ta_h, xh, uint64_t(a.K), uint64_t(a.M), uint64_t(a.K) * 2, kUK, kUM) ||
        !encode_f16_2d_sw128(&ta_l, xl, uint64_t(a.K), uint64_t(a.M), uint64_t(a.K) * 2, kUK, kUM) ||
        !encode_f16_2d_sw128(&tb_h, wh, uint64_t(a.K), uint64_t(rtot), uint64_t(a.K) * 2, kUK, brows) ||
        !encode_f16_2d_sw128(&tb_l, wl, uint64_t(a.K), uint64_t(rtot), uint64_t(a.K) * 2, kUK, brows))
        return cudaErrorInvalidValue;
    const int nst = a.K / kUK, mblk = (a.M + kUM - 1) / kUM, outs = pair ? BN / 2 : BN;
    const int ntile = (a.rows + outs - 1) / outs;
    const int64_t tiles = int64_t(ntile) * mblk;
    // K splits (clusters of up to 4, at least 2 stages each): one CTA fits an SM, so the launch runs in waves of
    // sms CTAs, each CTA costing its stages plus about 4 stages of fixed work (TMEM, the first copies, the
    // epilogue) and 4 more for a cluster reduction. Measured at 512 rows: (2560 -> 9728) whole tiles 3 waves
    // 140 us vs 3 splits 178 us; the Qwen3-4B step with o_proj / down / qkv split 3 / 3 / 2 ways +4%.
    int ks = 1;
    int64_t best = INT64_MAX;
    for (int c = 1; c <= kUMaxSplit; c++) {
        if (c > 1 && nst / c < 2) break;
        const int64_t cost = (tiles * c + sms - 1) / sms * ((nst + c - 1) / c + 4 + (c > 1 ? 4 : 0));
        if (cost < best) {
            best = cost;
            ks = c;
        }
    }
    UmmaSplit sp;
    sp.sper = (nst + ks - 1) / ks;
    sp.ksplit = (nst + sp.sper - 1) / sp.sper;
    sp.xh = xh;
    sp.xl = xl;
    auto k = pair ? umma_dq_gemm_kernel<BN, true> : umma_dq_gemm_kernel<BN, false>;
    const size_t smem = size_t(kDqStages) * (2 * kUM * kUK * 2 + 2 * BN * kUK * 2) + 64 + kUM * 8 + 1024;
    static int attr_set[2][8] = {};  // per (pair, device < 8)
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 8 || !attr_set[pair][dev]) {
        if (cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
            e != cudaSuccess)
            return e;
        if (dev < 8) attr_set[pair][dev] = 1;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(ntile, mblk, sp.ksplit);
    cfg.blockDim = dim3(kUThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[2];
    int na = 0;
    attr[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;  // after the dequantising kernel
    attr[na].val.programmaticStreamSerializationAllowed = 1;
    na++;
    if (sp.ksplit > 1) {
        attr[na].id = cudaLaunchAttributeClusterDimension;
        attr[na].val.clusterDim.x = 1;
        attr[na].val.clusterDim.y = 1;
        attr[na].val.clusterDim.z = sp.ksplit;
        na++;
    }
    cfg.attrs = attr;
    cfg.numAttrs = na;
    return cudaLaunchKernelEx(&cfg, k, a, sp, ta_h, ta_l, tb_h, tb_l);
}

// The tcgen05 kernel takes 128+ activation rows of FP8 / FP4 weights whose activations were split into hi / lo
// f16 (xh, xl: [M][K]); K a multiple of 64. cudaErrorNotSupported otherwise.
cudaError_t launch_gemm_umma(const GemvArgs& a, const __half* xh, const __half* xl, cudaStream_t st, bool pdl) {
    if (a.M < kUMinRows || (a.fmt != kFP8 && a.fmt != kFP4) || a.K % kUK || !xh || !xl || a.row_bytes % 16 ||
        (a.pair_off && a.argmax))
        return cudaErrorNotSupported;
    const bool pair = a.pair_off != 0;
    const int sms = num_sms(), nst = a.K / kUK;
    const int mblk = (a.M + kUM - 1) / kUM;
    // 128 weight rows per CTA when that still gives every SM a tile, else 64
    int bn = 128;
    if (int64_t((a.rows + (pair ? 63 : 127)) / (pair ? 64 : 128)) * mblk < sms) bn = 64;
    const int outs = pair ? bn / 2 : bn;
    const int ntile = (a.rows + outs - 1) / outs;
    const int64_t tiles = int64_t(ntile) * mblk;
    int ks = 1;
    if (tiles < sms) ks = int(std::min<int64_t>({(sms + tiles - 1) / tiles, int64_t(kUMaxSplit), std::max(1, nst / 2)}));
    UmmaSplit sp;
    sp.sper = (nst + ks - 1) / ks;
    sp.ksplit = (nst + sp.sper - 1) / sp.sper;
    sp.xh = xh;
    sp.xl = xl;
    UmmaFn k = a.fmt == kFP8 ? pick_umma<kFP8>(bn, pair) : pick_umma<kFP4>(bn, pair);
    const size_t smem = a.fmt == kFP8 ? umma_smem<kFP8>(bn, pair) : umma_smem<kFP4>(bn, pair);
    if (smem > 227 * 1024) return cudaErrorNotSupported;
    static int attr_set[2][2][2][8] = {};  // per (format, BN, pair, device < 8)
    int dev = 0;
    cudaGetDevice(&dev);
    int* set = dev < 8 ? &attr_set[a.fmt == kFP8 ? 0 : 1][bn == 128][pair][dev] : nullptr;
    if (!set || *set < int(smem)) {
        if (cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
            e != cudaSuccess)
            return e;
        if (set) *set = int(smem);
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(ntile, mblk, sp.ksplit);
    cfg.blockDim = dim3(kUThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[2];
    int na = 0;
    if (pdl) {
        attr[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[na].val.programmaticStreamSerializationAllowed = 1;
        na++;
    }
    if (sp.ksplit > 1) {  // the K splits of a tile form one cluster
        attr[na].id = cudaLaunchAttributeClusterDimension;
        attr[na].val.clusterDim.x = 1;
        attr[na].val.clusterDim.y = 1;
        attr[na].val.clusterDim.z = sp.ksplit;
        na++;
    }
    cfg.attrs = attr;
    cfg.numAttrs = na;
    return cudaLaunchKernelEx(&cfg, k, a, sp);
}

}  // namespace neko
