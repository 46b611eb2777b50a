// Dequant matmul for 5..64 activation rows (batched decode, prefill chunks) on the 5th-generation tensor cores
// with warp-specialised roles: the MatmulQ8 / MatmulQ4 dispatch (matmul_q8.comp, matmul_q4.comp;
// cpu::matmul, cpu_ops.cpp:462-481).
//
// The weights are the UMMA's M side (128 packed rows per CTA; SwiGLU: 64 gate + 64 up rows) and the activation
// rows its N side (32 or 64, rows past M read as zeros), so each weight code is fetched and converted once per
// call, and the arithmetic is that of the other tcgen05 kernels (k_umma.cu): w = code x scale split into f16
// hi + lo (hi = f16(code x scale), lo = the exact residual), activations split into f16 hi + lo beforehand,
// D = w_hi x_hi + w_hi x_lo + w_lo x_hi accumulated in fp32 in TMEM over all of K (w_hi x [x_hi; x_lo] as one
// UMMA of 2 N columns, the halves added in the epilogue).
//
// Roles (352 threads; one CTA per SM, or two: when a launch has no K split and more than two waves of tiles, the
// ~30% of a CTA's time outside its K loop, the first copies and the epilogue, then overlaps the other's K loop
// (M = 64 LM head 211 -> 138 us); when one raw stage per split fits every tile in one wave of two per SM, K is
// split further and each K loop is shorter (batch-64 SwiGLU matmul), K in stages of 64:
//  * warp 0, one lane: weight producer. Raw stages of four K stages (the code bytes of the 128 rows, 256 bytes a
//    row for FP8, with the 128-byte swizzle, and the 16-byte scale group holding their eight block scales) into a
//    2-deep ring (1-deep in the split two-per-SM layout) with TMA tensor copies of 64-row boxes; weights never
//    depend on the previous kernel, so this lane never waits for it;
//  * warp 10, one lane: activation producer. The activations' hi / lo tiles (128-byte swizzled, K-major) of each
//    stage into a 6-deep ring (2-deep at two CTAs per SM), after the dependency wait;
//  * warps 2..9: converters, one tile row (TMEM lane) and half a stage's K each. Raw stage -> the A stage's
//    w_hi / w_lo tiles in TMEM (tcgen05.st; the weights never pass through shared memory again, which leaves its
//    bandwidth to the copies); one arrival per warp on the A stage's barrier, one on the raw stage's release
//    barrier after its fourth K stage;
//  * warp 1, one lane: issues the 8 UMMAs of a stage (4 K steps x 2, A from TMEM, B from shared memory) once its
//    A and B halves are complete and commits them to their release barriers; a final commit marks the
//    accumulator complete.
// The single-issuer roles run on one lane (their warp's other lanes go straight to the epilogue: keeping the
// whole warp in the loop measured slower). No CTA barrier in the K loop; every wait is bounded and gives up as
// soon as another role has failed.
// Epilogue: the converter warps move the accumulator TMEM -> registers and push it, 16 bytes per store, into the
// receive buffer of the CTA that owns those activation rows (with K split over a thread-block cluster of 2, 4 or
// 8 CTAs, CTA z owns a block of rows; distributed shared memory). After one cluster barrier each CTA sums its
// rows' partials in split order (deterministic), applies the row scale (chained RMSNorm), bias / GELU /
// accumulate or SiLU * up, greedy argmax keys, the next matmul's f16 hi / lo input and per-64-column sums of
// squares, as tc_gemm_kernel's epilogue does (k_mma.cu).
#include <cooperative_groups.h>

#include <algorithm>
#include <climits>
#include <cstdlib>
#include <cstdint>

#include "gemv_core.cuh"
#include "mma_frag.cuh"
#include "neko_common.cuh"
#include "neko_internal.h"
#include "tc5_core.cuh"
#include "tma_host.h"

namespace neko {

namespace {

constexpr int kWM = 128;                      // weight rows per CTA (UMMA M)
constexpr int kWK = 64;                       // K per stage: 64 f16 = one 128-byte swizzle atom of B
constexpr int kWSub = 4;                      // K stages per raw stage (one 16-byte scale group per row)
constexpr int kWConv = 8;                     // converter warps
constexpr int kWThreads = 32 * (3 + kWConv);  // weight producer, MMA, converters, activation producer
constexpr int kWActWarp = 2 + kWConv;         // the activation producer's warp
constexpr int kWRaw = 2;                      // raw stages (4 K stages each)
constexpr int kWOps = 2;                      // A stages (weight tiles in TMEM)
constexpr int kWB = 6;                        // B stages (activation tiles in shared memory)
constexpr int kWBLite = 2;                    // the same for two CTAs per SM
constexpr int kWMaxSplit = 8;                 // CTAs of a split-K cluster (portable limit)
constexpr int kWMaxRows = 64;                 // activation rows (UMMA N <= 64)
// TMEM columns: the accumulators in [0, 2 NT) (column n < NT: w_hi x_hi + w_lo x_hi of activation row n,
// NT + n: w_hi x_lo), A stage o's tiles in [128 + 64 o, 192 + 64 o): w_hi in the first 32 columns, w_lo in the
// next 32 (two f16 of consecutive K per 32-bit column, row = lane)
constexpr int kWTmemCols = 256;
constexpr int kWAcol = 2 * kWMaxRows;
static_assert(kWAcol + 64 * kWOps <= kWTmemCols, "TMEM columns");

// Activation rows owned per CTA of a ks-way cluster (ks in 1, 2, 4, 8): NT / ks, whole 16-byte quads; the receive
// buffer's row pitch in floats: an odd number of 16-byte chunks, so 16-byte accesses by consecutive rows spread
// over all banks.
__host__ __device__ constexpr int ws_rows_per_owner(int nt, int ks) { return nt / ks; }
__host__ __device__ constexpr int ws_recv_pitch(int mb) { return mb + ((mb / 4) % 2 == 0 ? 4 : 8); }
constexpr int ws_recv_floats(int nt, int kmax = kWMaxSplit) {  // the largest ks x 128 x pitch, ks = 1, 2, .. kmax
    int m = 0;
    for (int k = 1; k <= kmax; k *= 2) {
        const int v = k * ws_recv_pitch(ws_rows_per_owner(nt, k));
        m = m > v ? m : v;
    }
    return m * 128;
}

// Dynamic shared memory (1024-byte aligned base): B stages (activations hi / lo) | raw stages | receive buffer |
// barriers | flags | epilogue scratch. A raw stage holds [kRP / 128 column boxes][128 rows][128 bytes] of codes
// with the 128-byte swizzle (16-byte chunk c of row r at chunk c ^ (r % 8)), then [128 rows][16] scale groups.
// Layout modes. kFull: one CTA per SM. kLite (two CTAs per SM, no K split): a 2-deep B ring and the receive buffer
// over the rings, which are free once every UMMA has completed. kLite2 (two CTAs per SM, 2 or 4 K splits of one raw
// stage each): a 2-deep B ring, one raw stage, a receive buffer of its own (peers push into it while this CTA may
// still be in its K loop) sized for up to 4 splits.
enum WsMode : int { kFull = 0, kLite = 1, kLite2 = 2 };
template <int FMT, int NT, int MODE = kFull>
struct WsLayout {
    static constexpr int kB = MODE == kFull ? kWB : kWBLite;
    static constexpr int kRawN = MODE == kLite2 ? 1 : kWRaw;   // raw ring depth
    static constexpr int kCB = FMT == kFP8 ? kWK : kWK / 2;  // code bytes per row per K stage
    static constexpr int kRP = kWSub * kCB;                   // code bytes per row per raw stage (256 / 128)
    static constexpr int kBTile = NT * kWK * 2;               // one f16 B tile (activations)
    static constexpr int kOp = 2 * kBTile;                    // B hi, B lo (one 2 NT-row operand)
    static constexpr int kRawCodes = kWM * kRP;
    static constexpr int kRaw = kRawCodes + kWM * 16;
    static constexpr int kRawOff = kB * kOp;
    static constexpr int kRingEnd = kRawOff + kRawN * kRaw;
    static constexpr int kRecvOff = MODE == kLite ? 0 : kRingEnd;  // [source split][128 tile rows][pitch]
    static constexpr int kRecv = MODE == kLite    ? kWM * ws_recv_pitch(NT) * 4
                                 : MODE == kLite2 ? ws_recv_floats(NT, 4) * 4
                                                  : ws_recv_floats(NT) * 4;
    static constexpr int kBarOff = MODE == kLite ? kRingEnd : kRecvOff + kRecv;
    static constexpr int kNBar = 2 * kRawN + 2 * kWOps + 2 * kB + 1;  // raw, A, B full / empty; done
    static constexpr int kMiscOff = kBarOff + kNBar * 8;      // TMEM address, failure flag
    static constexpr int kKeysOff = (kMiscOff + 8 + 15) / 16 * 16;
    static constexpr int kRsOff = kKeysOff + NT * 8;          // row scales
    static constexpr int kSspOff = kRsOff + NT * 4;           // [NT][4] sums of squares per 32 columns
    static constexpr int kBytes = kSspOff + NT * 4 * 4;
    static_assert(kOp % 1024 == 0 && kRaw % 1024 == 0 && kRecv % 16 == 0, "tile and copy alignment");
    static_assert(MODE != kLite || kRecv <= kRingEnd, "the receive buffer fits over the rings");
};

struct WsPlan {
    int ksplit;  // CTAs along K (the cluster's size: 1, 2, 4 or 8); split z takes raw stages
                 // [z nraw / ks, (z + 1) nraw / ks) of the nraw = ceil(K / 256) (4 K stages each)
};

__device__ __forceinline__ void tma_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], "
        "[%4];" ::"r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
        : "memory");
}

// D (TMEM) += A (TMEM, 128 x 16 f16) x B (shared memory descriptor), kind::f16
__device__ __forceinline__ void umma_f16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                            uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
        "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// 32 lanes x 16 columns of 32-bit words into TMEM (this warp's lane quarter)
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&v)[16]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(
            taddr),
        "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]), "r"(v[9]),
        "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15])
        : "memory");
}

// Bounded wait that also gives up once another role has recorded a failure.
__device__ __noinline__ bool ws_wait(uint64_t* bar, uint32_t parity, volatile int* fail) {
    for (uint32_t i = 0; i < kMbarMaxTries; i++) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((i & 63u) == 63u && *fail) return false;
    }
    set_device_error(kErrMbarTimeout);
    *fail = 1;
    return false;
}

// One converter thread, K stage j (0..3) of a raw stage: tile row r, the stage's weights 32 h .. 32 h + 31 (one
// quantisation block) as w = code x scale split into f16 hi + lo, packed two per word in K order.
template <int FMT, int NT>
__device__ __forceinline__ void ws_convert(const uint8_t* raw, int r, int j, int h, uint32_t (&hi)[16],
                                           uint32_t (&lo)[16]) {
    using L = WsLayout<FMT, NT>;
    const uint16_t sbits = *reinterpret_cast<const uint16_t*>(raw + L::kRawCodes + r * 16 + 4 * j + 2 * h);
    const __half2 sc = __halves2half2(__ushort_as_half(sbits), __ushort_as_half(sbits));
    __half2 c[16];
    if (FMT == kFP8) {  // bytes [64 j + 32 h, + 32) of the raw row: box j / 2, chunks 4 (j % 2) + 2 h, + 1
        const uint8_t* box = raw + (j >> 1) * (kWM * 128) + r * 128;
        const int c0 = 4 * (j & 1) + 2 * h;
        const uint4 w0 = *reinterpret_cast<const uint4*>(box + ((c0 ^ (r & 7)) << 4));
        const uint4 w1 = *reinterpret_cast<const uint4*>(box + (((c0 + 1) ^ (r & 7)) << 4));
        const uint32_t wd[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
#pragma unroll
        for (int i = 0; i < 8; i++) e4m3x4_to_half2(wd[i], c[2 * i], c[2 * i + 1]);
    } else {  // block bytes [32 j + 16 h, + 16): weight b in the low nibble of byte b, weight b + 16 in the high
        const uint4 w = *reinterpret_cast<const uint4*>(raw + r * 128 + (((2 * j + h) ^ (r & 7)) << 4));
        const uint32_t wd[4] = {w.x, w.y, w.z, w.w};
        const __half2 k16 = __float2half2_rn(kFp4Factor);  // engine FP4 decode (value / 16384) x 16384
#pragma unroll
        for (int i = 0; i < 4; i++) {
#pragma unroll
            for (int hn = 0; hn < 2; hn++) {  // low nibbles: weights 4 i ..; high nibbles: weights 16 + 4 i ..
                const uint32_t v = wd[i] >> (4 * hn);
                const uint32_t p01 = (v & 0x0000000Fu) | ((v << 8) & 0x000F0000u);          // bytes 0, 1
                const uint32_t p23 = ((v >> 16) & 0x0000000Fu) | ((v >> 8) & 0x000F0000u);  // bytes 2, 3
                c[8 * hn + 2 * i] = __hmul2(fp4x2_to_half2(p01), k16);
                c[8 * hn + 2 * i + 1] = __hmul2(fp4x2_to_half2(p23), k16);
            }
        }
    }
#pragma unroll
    for (int v = 0; v < 16; v++) {
        const __half2 hh = __hmul2(c[v], sc);
        hi[v] = h2u(hh);
        lo[v] = h2u(__hfma2(c[v], sc, __hneg2(hh)));
    }
}

template <int FMT, int NT, bool PAIR, int MODE>
__global__ void __launch_bounds__(kWThreads, MODE == kFull ? 1 : 2)
    umma_ws_kernel(const GemvArgs a, const WsPlan pl, const __grid_constant__ CUtensorMap t_code,
                   const __grid_constant__ CUtensorMap t_scale, const __grid_constant__ CUtensorMap t_xh,
                   const __grid_constant__ CUtensorMap t_xl) {
    using L = WsLayout<FMT, NT, MODE>;
    constexpr int kWB = L::kB, kWRaw = L::kRawN;
    extern __shared__ uint8_t wsm_raw[];
    uint8_t* sm = wsm_raw + ((1024 - (smem_u32(wsm_raw) & 1023)) & 1023);
    uint64_t* raw_full = reinterpret_cast<uint64_t*>(sm + L::kBarOff);
    uint64_t* raw_empty = raw_full + kWRaw;
    uint64_t* a_full = raw_empty + kWRaw;
    uint64_t* a_empty = a_full + kWOps;
    uint64_t* b_full = a_empty + kWOps;
    uint64_t* b_empty = b_full + kWB;
    uint64_t* done = b_empty + kWB;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(sm + L::kMiscOff);
    volatile int* fail = reinterpret_cast<volatile int*>(sm + L::kMiscOff + 4);
    unsigned long long* keys = reinterpret_cast<unsigned long long*>(sm + L::kKeysOff);
    float* rs = reinterpret_cast<float*>(sm + L::kRsOff);
    float* ssp = reinterpret_cast<float*>(sm + L::kSspOff);
    float* recv = reinterpret_cast<float*>(sm + L::kRecvOff);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int tile = blockIdx.x, z = blockIdx.z, ks = pl.ksplit;
    constexpr int OC = PAIR ? kWM / 2 : kWM;  // output columns of the tile
    const int n0 = tile * OC;
    const int nst_all = a.K / kWK, nraw_all = (nst_all + kWSub - 1) / kWSub;
    const int s_begin = kWSub * (z * nraw_all / ks), nst = min(nst_all, kWSub * ((z + 1) * nraw_all / ks)) - s_begin;
    const int nraw = (nst + kWSub - 1) / kWSub;
    // Every CTA reads the same activation tiles: each tile starts its K range at a different raw stage (whole raw
    // stages when they are all full), so that the copies in flight at any moment spread over many L2 lines.
    const int rot = (nst % kWSub == 0 && nraw > 0) ? tile % nraw : 0;
    auto kstage = [&](int i) { return s_begin + kWSub * ((i / kWSub + rot) % nraw) + i % kWSub; };  // K stage of step i
    const int cbytes = FMT == kFP8 ? a.K : a.K / 2;
    const int M = a.M, mb = ws_rows_per_owner(NT, ks);  // activation rows z mb .. z mb + mb - 1 are this CTA's
    const int rp = ws_recv_pitch(mb);
    constexpr uint32_t kIdesc = f16_idesc(kWM, NT), kIdesc2 = f16_idesc(kWM, 2 * NT);

    if (warp == 1) {  // TMEM: the accumulators and the A stages' tiles
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                     "r"(kWTmemCols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    if (tid == 0) {
        for (int r = 0; r < kWRaw; r++) {
            mbar_init(&raw_full[r], 1);
            mbar_init(&raw_empty[r], kWConv);
        }
        for (int o = 0; o < kWOps; o++) {
            mbar_init(&a_full[o], kWConv);
            mbar_init(&a_empty[o], 1);
        }
        for (int o = 0; o < kWB; o++) {
            mbar_init(&b_full[o], 1);
            mbar_init(&b_empty[o], 1);
        }
        mbar_init(done, 1);
        fence_barrier_init();
        // the descriptors and swizzled copies assume 1024-byte aligned tiles and the tensor maps 64-byte aligned
        // parameters: a failure is recorded and nothing is issued
        *fail = ((smem_u32(sm) & 1023u) || (reinterpret_cast<uintptr_t>(&t_code) & 63u) ||
                 (reinterpret_cast<uintptr_t>(&t_xh) & 63u) || nst <= 0 || (MODE == kLite && ks != 1) || (MODE == kLite2 && (ks > 4 || nraw > 1)))
                    ? 1
                    : 0;
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    const bool bad = *fail != 0;

    if (warp == 0) {
        // ------------------------------------------------------------------------------ weight producer
        if (lane == 0 && !bad) {
            // tile rows 0..63 and 64..127 (SwiGLU: the gate rows, then the up rows)
            const int y0 = PAIR ? tile * (kWM / 2) : tile * kWM;
            const int y1 = PAIR ? int(a.pair_off) + tile * (kWM / 2) : tile * kWM + kWM / 2;
            int issued = 0;
            for (; issued < nraw; issued++) {
                const int r = issued % kWRaw;
                if (issued >= kWRaw && !ws_wait(&raw_empty[r], uint32_t(issued / kWRaw - 1) & 1u, fail)) break;
                uint8_t* dst = sm + L::kRawOff + r * L::kRaw;
                const int s = kstage(kWSub * issued);
                mbar_arrive_expect_tx(&raw_full[r], uint32_t(L::kRaw));
#pragma unroll
                for (int cb = 0; cb < L::kRP / 128; cb++) {  // 128-byte column boxes of the codes
                    tma_2d(dst + cb * (kWM * 128), &t_code, s * L::kCB + 128 * cb, y0, &raw_full[r]);
                    tma_2d(dst + cb * (kWM * 128) + (kWM / 2) * 128, &t_code, s * L::kCB + 128 * cb, y1, &raw_full[r]);
                }
                const int sx = cbytes + 16 * (s / kWSub);
                tma_2d(dst + L::kRawCodes, &t_scale, sx, y0, &raw_full[r]);
                tma_2d(dst + L::kRawCodes + (kWM / 2) * 16, &t_scale, sx, y1, &raw_full[r]);
            }
            if (issued < nraw)  // failed: leave no copy in flight (each slot's last stage has landed)
                for (int i = max(0, issued - kWRaw); i < issued; i++)
                    mbar_wait(&raw_full[i % kWRaw], uint32_t(i / kWRaw) & 1u);
        }
    } else if (warp == kWActWarp) {
        // ------------------------------------------------------------------------------ activation producer
        if (lane == 0 && !bad) {
            pdl_wait();  // the activations come from the previous kernel
            int issued = 0;
            for (; issued < nst; issued++) {
                const int o = issued % kWB;
                if (issued >= kWB && !ws_wait(&b_empty[o], uint32_t(issued / kWB - 1) & 1u, fail)) break;
                uint8_t* dst = sm + o * L::kOp;
                const int k = kstage(issued) * kWK;
                mbar_arrive_expect_tx(&b_full[o], uint32_t(2 * L::kBTile));
                tma_2d(dst, &t_xh, k, 0, &b_full[o]);
                tma_2d(dst + L::kBTile, &t_xl, k, 0, &b_full[o]);
            }
            if (issued < nst)
                for (int i = max(0, issued - kWB); i < issued; i++) mbar_wait(&b_full[i % kWB], uint32_t(i / kWB) & 1u);
        }
    } else if (warp == 1) {
        // ------------------------------------------------------------------------------ UMMA issuer
        if (lane == 0) {
            if (!bad) {
                for (int i = 0; i < nst; i++) {
                    const int o = i % kWOps, ob = i % kWB;
                    if (!ws_wait(&b_full[ob], uint32_t(i / kWB) & 1u, fail) ||
                        !ws_wait(&a_full[o], uint32_t(i / kWOps) & 1u, fail))
                        break;
                    tc_fence_after();
                    const uint32_t bh = smem_u32(sm + ob * L::kOp);
                    const uint32_t ah = tmem + uint32_t(kWAcol + 64 * o), al = ah + 32u;
#pragma unroll
                    for (int k = 0; k < kWK / 16; k++) {  // 16-wide K steps: 8 TMEM columns of A, 32 bytes of B rows
                        const uint32_t ac = 8u * k, off = 32u * k;
                        // w_hi x [x_hi; x_lo]: the B hi and lo tiles are one 2 NT-row operand
                        umma_f16_ts(tmem, ah + ac, sw128_desc(bh + off), kIdesc2, (i > 0 || k > 0) ? 1u : 0u);
                        umma_f16_ts(tmem, al + ac, sw128_desc(bh + off), kIdesc, 1u);
                    }
                    umma_commit(&a_empty[o]);
                    umma_commit(&b_empty[ob]);
                }
            }
            umma_commit(done);  // every UMMA issued above has completed (none: at once)
        }
    } else {
        // ------------------------------------------------------------------------------ converters
        // warp 2 + 4 h + q: tile rows 32 q .. 32 q + 31 (its TMEM lane quarter), K half h of each stage
        const int quarter = warp & 3, h = (warp - 2) >> 2, r = 32 * quarter + lane;
        const uint32_t lane_base = uint32_t(32 * quarter) << 16;
        for (int i = 0; i < nst && !bad; i++) {
            const int j = i % kWSub, rsl = (i / kWSub) % kWRaw, o = i % kWOps;
            int ok = 1;
            if (lane == 0) {
                if (j == 0) ok = ws_wait(&raw_full[rsl], uint32_t(i / kWSub / kWRaw) & 1u, fail);
                if (ok && i >= kWOps) ok = ws_wait(&a_empty[o], uint32_t(i / kWOps - 1) & 1u, fail);
            }
            if (!__shfl_sync(0xffffffffu, ok, 0)) break;
            tc_fence_after();  // the UMMAs that read this stage's A columns have completed
            uint32_t hi[16], lo[16];
            ws_convert<FMT, NT>(sm + L::kRawOff + rsl * L::kRaw, r, j, h, hi, lo);
            const uint32_t col = tmem + lane_base + uint32_t(kWAcol + 64 * o + 16 * h);
            tmem_st16(col, hi);
            tmem_st16(col + 32u, lo);
            asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
            tc_fence_before();
            __syncwarp();
            if (lane == 0) {
                mbar_arrive(&a_full[o]);
                if (j == kWSub - 1 || i == nst - 1) mbar_arrive(&raw_empty[rsl]);
            }
        }
    }

    // ------------------------------------------------------------------------------ epilogue
    pdl_wait();  // the row scales, residual and argmax keys come from earlier kernels
    pdl_trigger();
    namespace cg = cooperative_groups;
    if (warp >= 2 && warp < 2 + kWConv) {
        // accumulator rows (tile row c = TMEM lane) -> the owners' receive buffers: [split z][c][row - owner's first]
        int ok = 1;
        if (lane == 0) ok = ws_wait(done, 0u, fail) && !*fail;
        ok = __shfl_sync(0xffffffffu, ok, 0);
        tc_fence_after();
        const int quarter = warp & 3, half = (warp - 2) >> 2, c = 32 * quarter + lane;
#pragma unroll
        for (int c0 = half * (NT / 2); c0 < (half + 1) * (NT / 2); c0 += 16) {
            float v[16];
            if (ok) {
                float w[16];
                tmem_ld16(tmem + (uint32_t(32 * quarter) << 16) + uint32_t(c0), v);
                tmem_ld16(tmem + (uint32_t(32 * quarter) << 16) + uint32_t(NT + c0), w);
#pragma unroll
                for (int u = 0; u < 16; u++) v[u] += w[u];
            } else {
#pragma unroll
                for (int u = 0; u < 16; u++) v[u] = 0.0f;
            }
#pragma unroll
            for (int g = 0; g < 4; g++) {
                const int m = c0 + 4 * g, owner = m / mb;
                if (owner >= ks) continue;
                float* dst = recv + (z * kWM + c) * rp + (m - owner * mb);
                if (ks > 1) dst = cg::this_cluster().map_shared_rank(dst, owner);
                *reinterpret_cast<float4*>(dst) = make_float4(v[4 * g], v[4 * g + 1], v[4 * g + 2], v[4 * g + 3]);
            }
        }
    }
    // this CTA's rows: row scales of a chained RMSNorm (rstd from the producer's per-tile sums of squares, in tile
    // order), cleared argmax keys
    const int m_lo = z * mb, m_hi = min(M, m_lo + mb);
    for (int m = m_lo + tid; m < m_hi; m += kWThreads) {
        if (a.in_ss) {
            double s2 = 0.0;
            for (int t = 0; t < a.in_ss_tiles; t++) s2 += double(a.in_ss[int64_t(t) * M + m]);
            rs[m] = float(1.0 / sqrt(s2 / a.K + double(a.eps)));
        }
        keys[m] = 0ull;
    }
    tc_fence_before();
    if (ks > 1) cg::this_cluster().sync();  // every split's partials have landed in their owners' buffers
    else __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kWTmemCols) : "memory");
    }
    if (*fail && tid == 0) set_device_error(kErrMbarTimeout);

    // this CTA's rows x the OC output columns: item = (quad of rows, column); a warp's 32 items share the quad
    static_assert(OC % 32 == 0 && kWThreads % 32 == 0, "whole warps per quad");
    const int quads = (m_hi - m_lo + 3) / 4;
    for (int it = tid; it - lane < quads * OC; it += kWThreads) {
        const bool live = it < quads * OC;
        const int jq = live ? it / OC : 0, c = live ? it - jq * OC : 0, mq = 4 * jq;
        float4 v = make_float4(0.f, 0.f, 0.f, 0.f), u = v;
        if (live) {
#pragma unroll
            for (int zz = 0; zz < kWMaxSplit; zz++) {  // split order
                if (zz >= ks) break;
                const float4 pv = *reinterpret_cast<const float4*>(recv + (zz * kWM + c) * rp + mq);
                v.x += pv.x; v.y += pv.y; v.z += pv.z; v.w += pv.w;
                if (PAIR) {
                    const float4 pu = *reinterpret_cast<const float4*>(recv + (zz * kWM + kWM / 2 + c) * rp + mq);
                    u.x += pu.x; u.y += pu.y; u.z += pu.z; u.w += pu.w;
                }
            }
        }
        const float vv[4] = {v.x, v.y, v.z, v.w}, uu[4] = {u.x, u.y, u.z, u.w};
        const int n = n0 + c;
#pragma unroll
        for (int e = 0; e < 4; e++) {
            const int m = m_lo + mq + e;
            if (m >= m_hi) break;  // uniform over the warp (its items share the quad)
            unsigned long long key = 0ull;
            float sq = 0.0f;
            if (live && n < a.rows) {
                float x = vv[e], y = uu[e];
                if (a.in_ss) {
                    x *= rs[m];
                    y *= rs[m];
                }
                float* dst = a.y + int64_t(m) * a.y_stride + a.n_off + n;
                if (PAIR) {
                    x = x / (1.0f + expf(-x)) * y;  // cpu::siluMul (cpu_ops.cpp:526-533)
                } else {
                    if (a.flags & kBias) x += a.bias[n];
                    if (a.flags & kGelu) x = gelu(x);
                    if (a.flags & kAccumulate) x += *dst;
                }
                *dst = x;
                key = argmax_key(x, n);
                if (a.out_hi) {  // the next matmul's activations: x * gamma as f16 hi + lo
                    const float yv = x * (a.out_gamma ? a.out_gamma[n] : 1.0f);
                    const __half hh = __float2half_rn(yv);
                    a.out_hi[int64_t(m) * a.out_ld + n] = hh;
                    a.out_lo[int64_t(m) * a.out_ld + n] = __float2half_rn(yv - __half2float(hh));
                }
                sq = x * x;
            }
            if (a.out_ss) {  // the warp's 32 columns of the row
                sq = warp_sum(sq);
                if (lane == 0 && live) ssp[m * 4 + (c >> 5)] = sq;
            }
            if (a.argmax) {
#pragma unroll
                for (int o = 16; o > 0; o >>= 1) key = max(key, __shfl_xor_sync(0xffffffffu, key, o));
                if (lane == 0 && live && key) atomicMax(&keys[m], key);
            }
        }
    }
    if (a.out_ss || a.argmax) __syncthreads();
    if (a.out_ss)  // one partial per (64-column tile, row) that holds output columns: summed by the consumer in order
        for (int j = tid; j < (m_hi - m_lo) * (OC / 64); j += kWThreads) {
            const int r = j / (OC / 64), h = j - r * (OC / 64), m = m_lo + r;
            if (n0 + 64 * h < a.rows)
                a.out_ss[int64_t(n0 / 64 + h) * M + m] = ssp[m * 4 + 2 * h] + ssp[m * 4 + 2 * h + 1];
        }
    if (a.argmax)
        for (int m = m_lo + tid; m < m_hi; m += kWThreads)
            if (keys[m]) atomicMax(a.argmax + m, keys[m]);
}

template <int FMT, int NT, int MODE>
size_t ws_smem() {
    return size_t(WsLayout<FMT, NT, MODE>::kBytes) + 1024;
}

using WsFn = void (*)(const GemvArgs, const WsPlan, const CUtensorMap, const CUtensorMap, const CUtensorMap,
                      const CUtensorMap);

template <int FMT, int MODE>
WsFn ws_pick_mode(int nt, bool pair, size_t* smem) {
    if (nt == 32) {
        *smem = ws_smem<FMT, 32, MODE>();
        return pair ? umma_ws_kernel<FMT, 32, true, MODE> : umma_ws_kernel<FMT, 32, false, MODE>;
    }
    *smem = ws_smem<FMT, 64, MODE>();
    return pair ? umma_ws_kernel<FMT, 64, true, MODE> : umma_ws_kernel<FMT, 64, false, MODE>;
}
template <int FMT>
WsFn ws_pick(int mode, int nt, bool pair, size_t* smem) {
    return mode == kLite    ? ws_pick_mode<FMT, kLite>(nt, pair, smem)
           : mode == kLite2 ? ws_pick_mode<FMT, kLite2>(nt, pair, smem)
                            : ws_pick_mode<FMT, kFull>(nt, pair, smem);
}

// K splits (1, 2, 4 or 8, whole raw stages of 4 K stages each, so each split starts on a scale group): one CTA
// per SM, so the launch runs in waves of sms CTAs, each costing its stages plus a fixed part (TMEM, the first
// copies and conversion, the epilogue: about 6 stages) and 2 more for the cluster exchange.
WsPlan ws_plan(int ntile, int nst) {
    const int sms = num_sms(), nraw = (nst + kWSub - 1) / kWSub;
    WsPlan p{1};
    int64_t best = INT64_MAX;
    for (int c = 1; c <= kWMaxSplit && c <= nraw; c *= 2) {
        const int64_t cost =
            (int64_t(ntile) * c + sms - 1) / sms * (std::min(kWSub * ((nraw + c - 1) / c), nst) + 6 + (c > 1 ? 2 : 0));
        if (cost < best) {
            best = cost;
            p.ksplit = c;
        }
    }
    return p;
}

}  // namespace

bool gemm_ws_fits(const GemvArgs& a) {
    return a.M >= 1 && a.M <= kWMaxRows && (a.fmt == kFP8 || a.fmt == kFP4) && a.K % kWK == 0 &&
           a.row_bytes % 16 == 0 && (reinterpret_cast<uintptr_t>(a.W) & 15) == 0 && !(a.pair_off && a.argmax) &&
           (a.pair_off == 0 || a.pair_off >= a.rows);
}

cudaError_t launch_gemm_ws(const GemvArgs& a, const __half* xh, const __half* xl, cudaStream_t st, bool pdl) {
    if (!gemm_ws_fits(a) || !xh || !xl || (reinterpret_cast<uintptr_t>(xh) & 15) ||
        (reinterpret_cast<uintptr_t>(xl) & 15))
        return cudaErrorNotSupported;
    const bool pair = a.pair_off != 0;
    const int64_t rtot = pair ? a.pair_off + a.rows : a.rows;  // matrix rows (SwiGLU: gate rows, then up rows)
    if (rtot >= (int64_t(1) << 31)) return cudaErrorNotSupported;
    const int nt = a.M <= 32 ? 32 : 64;
    CUtensorMap t_code{}, t_scale{}, t_xh{}, t_xl{};
    if (!encode_u8_2d(&t_code, a.W, uint64_t(a.row_bytes), uint64_t(rtot), uint64_t(a.row_bytes), 128u, kWM / 2,
                      true) ||
        !encode_u8_2d(&t_scale, a.W, uint64_t(a.row_bytes), uint64_t(rtot), uint64_t(a.row_bytes), 16u, kWM / 2) ||
        !encode_f16_2d_sw128(&t_xh, xh, uint64_t(a.K), uint64_t(a.M), uint64_t(a.K) * 2, kWK, uint32_t(nt)) ||
        !encode_f16_2d_sw128(&t_xl, xl, uint64_t(a.K), uint64_t(a.M), uint64_t(a.K) * 2, kWK, uint32_t(nt)))
        return cudaErrorNotSupported;
    const int outs = pair ? kWM / 2 : kWM, ntile = (a.rows + outs - 1) / outs, nst = a.K / kWK;
    WsPlan pl = ws_plan(ntile, nst);
    // Two CTAs per SM (NEKO_GEMM_WS_LITE=0 in the environment keeps one): with no K split and more tiles than two
    // waves, so that one CTA's fill and epilogue overlap the other's K loop; or, where one raw stage per split
    // (2 or 4 splits) fits every tile in one wave of two per SM and splits K further than one per SM can, so that
    // each CTA's K loop is shorter.
    static const bool lite_on = [] {
        const char* v = std::getenv("NEKO_GEMM_WS_LITE");
        return !(v && v[0] == '0');
    }();
    const int sms = num_sms(), nraw = (nst + kWSub - 1) / kWSub;
    int mode = kFull;
    if (lite_on && pl.ksplit == 1 && ntile > 2 * sms) {
        mode = kLite;
    } else if (lite_on && (nraw == 2 || nraw == 4) && nraw > pl.ksplit && int64_t(ntile) * nraw <= 2 * sms) {
        mode = kLite2;
        pl.ksplit = nraw;
    }
    size_t smem = 0;
    const WsFn k = a.fmt == kFP8 ? ws_pick<kFP8>(mode, nt, pair, &smem) : ws_pick<kFP4>(mode, nt, pair, &smem);
    if (const cudaError_t e = ensure_dyn_smem(k, smem); e != cudaSuccess) return e;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(ntile, 1, pl.ksplit);
    cfg.blockDim = dim3(kWThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[2];
    int na = 0;
    if (pdl) {
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
    return cudaLaunchKernelEx(&cfg, k, a, pl, t_code, t_scale, t_xh, t_xl);
}

}  // namespace neko
