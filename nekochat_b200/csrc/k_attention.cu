// Causal grouped-query attention over f16 KV caches: cpu::attention (app/architecture/shared/cpp/cpu_ops.cpp:
// 544-575) and the Attention kernel (gpu/shaders/attention.comp), written for sm_100a.
//
// Each activation row r (one token of some sequence) attends to cache positions [0, pos_r] of its sequence.
// Work unit = (row, KV head, split): the CTA serves the whole GQA group of the KV head (n_head / n_kv query
// heads), so each K/V byte is read once per row. A split's keys are walked in chunks staged into shared memory
// by TMA bulk copies (one copy per chunk when a head's positions are contiguous, as in the native runner's
// [slot][kv head][pos][hd] cache; one copy per key row in the engine's [pos][kv heads * hd] layout), double
// buffered so the next chunk streams in while this one is computed. Online softmax in fp32 (running max and
// sum); scores use 4 lanes per key, P.V has threads own value-dimension pairs. When a row needs several splits
// the partial (max, sum, acc) go to scratch and the last CTA of the (row, KV head) to finish merges them,
// elected by a ticket counter that it resets (so the kernel can be replayed from a CUDA graph).
#include <algorithm>
#include <cstdlib>

#include "mma_frag.cuh"
#include "neko_common.cuh"
#include "neko_internal.h"
#include "tma_host.h"

namespace neko {

namespace {

constexpr int kAttnThreads = 128;
constexpr int kMaxGroup = 8;  // query heads per KV head
constexpr int kMaxHd = 256;   // head dim (attention.comp limit)

struct Geometry {
    int splits;  // CTAs per (row, KV head)
    int span;    // keys per split (multiple of chunk)
    int chunk;   // keys per shared-memory chunk
    int smem;    // dynamic shared memory bytes
};

int chunk_for(int hd) { return hd <= 128 ? 64 : 32; }

// dynamic shared memory layout
struct Layout {
    int q, k, v, sc, stage, bars, total;
};

__host__ __device__ inline Layout layout(int G, int hd, int chunk) {
    Layout l;
    int off = 0;
    l.q = off;
    off += G * hd * 4;
    l.k = off;
    off += 2 * chunk * hd * 2;
    l.v = off;
    off += 2 * chunk * hd * 2;
    l.sc = off;
    off += G * chunk * 4;
    l.stage = off;
    off += G * hd * 4;
    off = (off + 15) / 16 * 16;
    l.bars = off;
    off += 2 * 8;
    l.total = off;
    return l;
}

__global__ void __launch_bounds__(kAttnThreads) attention_kernel(const AttnArgs a, const Geometry geo) {
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ float red[kMaxGroup][kAttnThreads / 32];
    __shared__ int last;

    const int split = blockIdx.x, kvh = blockIdx.y, r = blockIdx.z;
    const int G = a.n_head / a.n_kv, hd = a.hd, CH = geo.chunk;
    const Layout lay = layout(G, hd, CH);
    float* sq = reinterpret_cast<float*>(smem + lay.q);
    uint16_t* sk = reinterpret_cast<uint16_t*>(smem + lay.k);
    uint16_t* sv = reinterpret_cast<uint16_t*>(smem + lay.v);
    float* sc = reinterpret_cast<float*>(smem + lay.sc);
    float* stage = reinterpret_cast<float*>(smem + lay.stage);
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + lay.bars);

    pdl_wait();  // q and the newest cache rows come from the previous kernels
    pdl_trigger();
    const int pos = a.row_pos ? a.row_pos[r] : a.pos0 + r;
    const int slot = a.row_slot ? a.row_slot[r] : a.slot0;
    const int L = pos + 1;
    if (pos < 0 || pos >= a.pos_limit || L > geo.splits * geo.span) {  // outside the planned key range
        if (threadIdx.x == 0 && split == 0) set_device_error(kErrBadIndex);
        return;
    }
    const int active = (L + geo.span - 1) / geo.span;
    if (split >= active) return;
    const int j_begin = split * geo.span, j_end = min(L, j_begin + geo.span);
    const int nchunks = (j_end - j_begin + CH - 1) / CH;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const uint16_t* kbase = a.kc + int64_t(slot) * a.slot_stride + int64_t(kvh) * a.head_stride;
    const uint16_t* vbase = a.vc + int64_t(slot) * a.slot_stride + int64_t(kvh) * a.head_stride;
    const bool contiguous = a.pos_stride == hd;
    const uint32_t row_bytes = uint32_t(hd) * 2;

    // Issues the bulk copies of chunk c (keys j0 .. j0 + n) into buffer c & 1. Called by all of warp 0.
    auto issue = [&](int c) {
        const int j0 = j_begin + c * CH, n = min(CH, j_end - j0), b = c & 1;
        uint16_t* dk = sk + b * CH * hd;
        uint16_t* dv = sv + b * CH * hd;
        if (contiguous) {
            if (lane == 0) {
                mbar_arrive_expect_tx(&bars[b], 2u * uint32_t(n) * row_bytes);
                bulk_g2s(dk, kbase + int64_t(j0) * hd, uint32_t(n) * row_bytes, &bars[b]);
                bulk_g2s(dv, vbase + int64_t(j0) * hd, uint32_t(n) * row_bytes, &bars[b]);
            }
        } else {
            if (lane == 0) mbar_arrive_expect_tx(&bars[b], 2u * uint32_t(n) * row_bytes);
            __syncwarp();
            for (int j = lane; j < n; j += 32) {
                bulk_g2s(dk + j * hd, kbase + int64_t(j0 + j) * a.pos_stride, row_bytes, &bars[b]);
                bulk_g2s(dv + j * hd, vbase + int64_t(j0 + j) * a.pos_stride, row_bytes, &bars[b]);
            }
        }
    };

    if (tid == 0) {
        mbar_init(&bars[0], 1);
        mbar_init(&bars[1], 1);
        fence_barrier_init();
    }
    __syncthreads();
    if (warp == 0) {
        issue(0);
        if (nchunks > 1) issue(1);
    }
    for (int i = tid; i < G * hd; i += kAttnThreads)
        sq[i] = a.q[int64_t(r) * a.q_stride + int64_t(kvh * G + i / hd) * hd + (i % hd)];

    // P.V ownership: half2 dimension pair dp, keys kg, kg + kgroups, ...
    const int dpairs = hd / 2;
    const int kgroups = kAttnThreads / dpairs;  // >= 1 since hd <= 256
    const int dp = tid % dpairs, kg = tid / dpairs;
    const bool pv_active = kg < kgroups;
    // scores ownership: 4 lanes per key, lane part p covers dims 8p + 32i
    const int skey = tid >> 2, part = tid & 3;

    float m_run[kMaxGroup], l_run[kMaxGroup], acc[kMaxGroup][2];
#pragma unroll
    for (int g = 0; g < kMaxGroup; g++) {
        m_run[g] = -INFINITY;
        l_run[g] = 0.0f;
        acc[g][0] = acc[g][1] = 0.0f;
    }
    __syncthreads();  // q staged

    for (int c = 0; c < nchunks; c++) {
        const int j0 = j_begin + c * CH, n = min(CH, j_end - j0), b = c & 1;
        if (!mbar_wait(&bars[b], (c >> 1) & 1)) return;
        const uint16_t* ck = sk + b * CH * hd;
        const uint16_t* cv = sv + b * CH * hd;
        (void)j0;
        // scores: s = (q . k) * scale   (cpu_ops.cpp:558)
        for (int kk = skey; kk < CH; kk += kAttnThreads / 4) {
            float s[kMaxGroup];
#pragma unroll
            for (int g = 0; g < kMaxGroup; g++) s[g] = 0.0f;
            if (kk < n) {
                for (int d0 = 8 * part; d0 < hd; d0 += 32) {
                    const uint4 w = *reinterpret_cast<const uint4*>(ck + kk * hd + d0);
                    const float2 k0 = __half22float2(*reinterpret_cast<const __half2*>(&w.x));
                    const float2 k1 = __half22float2(*reinterpret_cast<const __half2*>(&w.y));
                    const float2 k2 = __half22float2(*reinterpret_cast<const __half2*>(&w.z));
                    const float2 k3 = __half22float2(*reinterpret_cast<const __half2*>(&w.w));
#pragma unroll
                    for (int g = 0; g < kMaxGroup; g++) {
                        if (g >= G) break;
                        const float4 qa = *reinterpret_cast<const float4*>(sq + g * hd + d0);
                        const float4 qb = *reinterpret_cast<const float4*>(sq + g * hd + d0 + 4);
                        float t = s[g];
                        t = fmaf(qa.x, k0.x, t);
                        t = fmaf(qa.y, k0.y, t);
                        t = fmaf(qa.z, k1.x, t);
                        t = fmaf(qa.w, k1.y, t);
                        t = fmaf(qb.x, k2.x, t);
                        t = fmaf(qb.y, k2.y, t);
                        t = fmaf(qb.z, k3.x, t);
                        t = fmaf(qb.w, k3.y, t);
                        s[g] = t;
                    }
                }
            }
#pragma unroll
            for (int g = 0; g < kMaxGroup; g++) {
                if (g >= G) break;
                float t = s[g];
                t += __shfl_xor_sync(0xffffffffu, t, 1);
                t += __shfl_xor_sync(0xffffffffu, t, 2);
                if (part == 0 && kk < n) sc[g * CH + kk] = t * a.scale;
            }
        }
        __syncthreads();
        // chunk max per head and the new running max
#pragma unroll
        for (int g = 0; g < kMaxGroup; g++) {
            if (g >= G) break;
            float w = -INFINITY;
            for (int jj = tid; jj < n; jj += kAttnThreads) w = fmaxf(w, sc[g * CH + jj]);
            w = warp_max(w);
            if (lane == 0) red[g][warp] = w;
        }
        __syncthreads();
        float m_new[kMaxGroup], corr[kMaxGroup], lsum[kMaxGroup];
#pragma unroll
        for (int g = 0; g < kMaxGroup; g++) {
            if (g >= G) break;
            float w = red[g][0];
            for (int i = 1; i < kAttnThreads / 32; i++) w = fmaxf(w, red[g][i]);
            m_new[g] = fmaxf(m_run[g], w);
            corr[g] = expf(m_run[g] - m_new[g]);  // 0 on the first chunk (m_run = -inf)
            lsum[g] = 0.0f;
        }
        __syncthreads();  // red is reused below
        for (int jj = tid; jj < n; jj += kAttnThreads) {
#pragma unroll
            for (int g = 0; g < kMaxGroup; g++) {
                if (g >= G) break;
                const float e = expf(sc[g * CH + jj] - m_new[g]);
                sc[g * CH + jj] = e;
                lsum[g] += e;
            }
        }
#pragma unroll
        for (int g = 0; g < kMaxGroup; g++) {
            if (g >= G) break;
            const float w = warp_sum(lsum[g]);
            if (lane == 0) red[g][warp] = w;
        }
        __syncthreads();  // probabilities and sums visible
#pragma unroll
        for (int g = 0; g < kMaxGroup; g++) {
            if (g >= G) break;
            float w = 0.0f;
            for (int i = 0; i < kAttnThreads / 32; i++) w += red[g][i];
            l_run[g] = l_run[g] * corr[g] + w;
            m_run[g] = m_new[g];
            acc[g][0] *= corr[g];
            acc[g][1] *= corr[g];
        }
        // P.V from the staged values
        if (pv_active) {
            for (int jj = kg; jj < n; jj += kgroups) {
                const float2 vv = __half22float2(*reinterpret_cast<const __half2*>(cv + jj * hd + 2 * dp));
#pragma unroll
                for (int g = 0; g < kMaxGroup; g++) {
                    if (g >= G) break;
                    const float p = sc[g * CH + jj];
                    acc[g][0] = fmaf(p, vv.x, acc[g][0]);
                    acc[g][1] = fmaf(p, vv.y, acc[g][1]);
                }
            }
        }
        __syncthreads();  // buffer b, sc and red are free again
        if (warp == 0 && c + 2 < nchunks) issue(c + 2);
    }

    // merge the key groups of the P.V phase through shared memory, one group at a time
    const bool split_mode = active > 1;
    for (int grp = 1; grp < kgroups; grp++) {
        __syncthreads();
        if (pv_active && kg == grp)
            for (int g = 0; g < G; g++) {
                stage[(g * dpairs + dp) * 2 + 0] = acc[g][0];
                stage[(g * dpairs + dp) * 2 + 1] = acc[g][1];
            }
        __syncthreads();
        if (pv_active && kg == 0)
            for (int g = 0; g < G; g++) {
                acc[g][0] += stage[(g * dpairs + dp) * 2 + 0];
                acc[g][1] += stage[(g * dpairs + dp) * 2 + 1];
            }
    }

    if (!split_mode) {
        if (pv_active && kg == 0)
            for (int g = 0; g < G; g++) {
                const float inv = 1.0f / l_run[g];
                float* o = a.out + int64_t(r) * a.out_stride + int64_t(kvh * G + g) * hd + 2 * dp;
                o[0] = acc[g][0] * inv;
                o[1] = acc[g][1] * inv;
            }
        return;
    }

    // split mode: write (max, sum, acc) and let the last CTA of this (row, KV head) merge
    const int64_t rec = hd + 2;
    if (pv_active && kg == 0)
        for (int g = 0; g < G; g++) {
            float* p = a.part + ((int64_t(r) * a.n_head + kvh * G + g) * geo.splits + split) * rec;
            if (dp == 0) {
                p[0] = m_run[g];
                p[1] = l_run[g];
            }
            p[2 + 2 * dp] = acc[g][0];
            p[3 + 2 * dp] = acc[g][1];
        }
    __threadfence();
    __syncthreads();
    if (tid == 0) {
        unsigned* t = a.tickets + int64_t(r) * a.n_kv + kvh;
        const unsigned ticket = atomicAdd(t, 1u);
        last = ticket == unsigned(active - 1);
        if (last) *t = 0u;  // every CTA of this (row, KV head) has taken its ticket: reset for the next launch
    }
    __syncthreads();
    if (!last) return;
    __threadfence();
    for (int i = tid; i < G * hd; i += kAttnThreads) {
        const int g = i / hd, d = i % hd;
        const float* base = a.part + (int64_t(r) * a.n_head + kvh * G + g) * geo.splits * rec;
        float M = -INFINITY;
        for (int s = 0; s < active; s++) M = fmaxf(M, __ldcg(base + s * rec));
        float num = 0.0f, den = 0.0f;
        for (int s = 0; s < active; s++) {
            const float w = expf(__ldcg(base + s * rec) - M);
            den += __ldcg(base + s * rec + 1) * w;
            num += __ldcg(base + s * rec + 2 + d) * w;
        }
        a.out[int64_t(r) * a.out_stride + int64_t(kvh * G + g) * hd + d] = num / den;
    }
}

// ------------------------------------------------------------------------------------------------ tensor cores
// The same work units and split-KV merge with the arithmetic on mma.sync m16n8k16 (f16 operands, fp32
// accumulation), for head_dim 64 / 128 and up to 8 query heads per KV head:
//  * the cache rows are f16 already, so keys and values enter the MMA exactly; the query and the probabilities
//    are split into hi + lo f16 (about 22 bits, as in the matmul), so scores and P.V keep fp32-level accuracy;
//  * keys and head dims are the MMA's rows, the group's query heads its 8 columns (heads past G are zero): the
//    scores S^T[key][head] take the key rows as A (ldmatrix) and the query fragments as B; P.V accumulates
//    O^T[dim][head] from the value rows (A, transposed by ldmatrix) and P^T as B, which 8 shuffles gather from
//    the score fragments. With G = 2 this is half the MMAs and accumulators of putting the heads on the rows;
//  * warp w owns keys 16w..16w+15 of each chunk with its own running max / sum per head (online softmax per
//    warp, no block barrier inside a chunk); the warps' (max, sum, acc) are merged once at the end of the split;
//  * cp.async variant (any cache layout): 4 warps, 64-key chunks staged by all threads with 16-byte cp.async into
//    padded shared-memory rows (pitch hd + 8 halves, conflict-free ldmatrix; rows past the last key zero-filled),
//    three buffers, one barrier per chunk;
//  * TMA variant (caches whose positions are contiguous rows of hd halves, e.g. [slot][kv head][pos][hd]): 2 warps,
//    32-key chunks that one thread stages as 2D tensor copies of 32 keys x 64 dims (128-byte swizzle: 16-byte
//    piece q of row j sits at piece q ^ (j & 7), so the ldmatrix row groups stay conflict-free without padding)
//    completing on one mbarrier per buffer; the copies read the rows past the chunk's last key too (cache
//    memory, or zeros past the tensor's end), whose values are zeroed in shared memory before use. Four CTAs
//    share an SM, so the splits are planned to fill them once (one wave).
constexpr int kTcChunk = 64;  // keys per chunk of the cp.async variant (4 warps x 16)
constexpr int kTcBufs = 3;

// Output element e (= head * hd + d) of row r, and (when asked) its f16 hi + lo split for the next matmul.
__device__ __forceinline__ void store_out(const AttnArgs& a, int r, int e, float v) {
    a.out[int64_t(r) * a.out_stride + e] = v;
    if (a.out_hi) {
        const __half h = __float2half_rn(v);
        a.out_hi[int64_t(r) * a.out_hl_stride + e] = h;
        a.out_lo[int64_t(r) * a.out_hl_stride + e] = __float2half_rn(v - __half2float(h));
    }
}
// TMA variant: 2 warps per CTA, chunks of 32 keys (boxes of 32 keys x 64 dims), 3 buffers: about 50 KB of
// shared memory, so four CTAs share an SM and a batch-64 layer's 512 (row, KV head) items run in one wave
constexpr int kTmaWarps = 2;
constexpr int kTmaChunk = 16 * kTmaWarps;
constexpr int kTmaBox = kTmaChunk * 128;  // bytes of one box (keys x 128-byte rows)
constexpr int kTcBufsTma = 3;             // buffers per CTA
constexpr int kTcCtasTma = 4;             // CTAs per SM
__host__ __device__ constexpr int tc_bufs(bool tma) { return tma ? kTcBufsTma : kTcBufs; }
__host__ __device__ constexpr int tc_warps(bool tma) { return tma ? kTmaWarps : 4; }

template <int HD, bool TMA>
constexpr int tc_attn_smem() {
    // the buffers, then (TMA) their mbarriers, then two flags; TMA: the fused decode's q / k / v rows
    // ([kMaxGroup + 2][HD] floats) and up to 1024 bytes to align the buffers
    return TMA ? kTcBufsTma * 2 * (HD / 64) * kTmaBox + 64 + (kMaxGroup + 2) * HD * 4 + 1024
               : kTcBufs * 2 * kTcChunk * (HD + 8) * 2 + 64;
}
static_assert(kTcCtasTma * (tc_attn_smem<128, true>() + 1024) <= 228 * 1024, "four TMA CTAs per SM");

__device__ __forceinline__ double warp_sum_dbl(double v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], "
        "[%4];" ::"r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
        : "memory");
}

template <int HD, bool TMA>
__global__ void __launch_bounds__(32 * tc_warps(TMA), TMA ? kTcCtasTma : 2)
    attention_tc_kernel(const AttnArgs a, const Geometry geo, const __grid_constant__ CUtensorMap tk,
                        const __grid_constant__ CUtensorMap tv) {
    constexpr int P = HD + 8;  // padded row pitch (halves)
    constexpr int W = tc_warps(TMA), NT = 32 * W;  // warps, threads
    constexpr int CH = 16 * W, KS = HD / 16, MT = HD / 16, NB = HD / 64, NBUF = tc_bufs(TMA);
    extern __shared__ __align__(128) uint8_t smem_raw[];
    // TMA boxes with the 128-byte swizzle need 1024-byte aligned destinations
    uint8_t* smem = TMA ? smem_raw + ((1024 - (smem_u32(smem_raw) & 1023)) & 1023) : smem_raw;
    uint16_t* kvb = reinterpret_cast<uint16_t*>(smem);  // [NBUF][2][CH][P]: keys, then values

    const int split = blockIdx.x, kvh = blockIdx.y, r = blockIdx.z;
    const int G = a.n_head / a.n_kv;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, gr = lane >> 2, c = lane & 3;
    pdl_wait();  // q and the newest cache rows come from the previous kernels
    const int pos = a.row_pos ? a.row_pos[r] : a.pos0 + r;
    const int slot = a.row_slot ? a.row_slot[r] : a.slot0;
    const int L = pos + 1;
    if (pos < 0 || pos >= a.pos_limit || L > geo.splits * geo.span) {  // outside the planned key range
        if (tid == 0 && split == 0) set_device_error(kErrBadIndex);
        return;
    }
    const int active = (L + geo.span - 1) / geo.span;
    if (split >= active) return;
    const int j_begin = split * geo.span, j_end = min(L, j_begin + geo.span);
    const int nchunks = (j_end - j_begin + CH - 1) / CH;
    const uint16_t* kbase = a.kc + int64_t(slot) * a.slot_stride + int64_t(kvh) * a.head_stride;
    const uint16_t* vbase = a.vc + int64_t(slot) * a.slot_stride + int64_t(kvh) * a.head_stride;
    // every thread: its 16-byte pieces of chunk cc's key and value rows into buffer cc % NBUF (one commit group
    // per chunk); rows past the chunk's last key are zero-filled without reading memory
    constexpr int BUF = TMA ? 2 * NB * kTmaBox : 2 * CH * P * 2;  // bytes per buffer
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + NBUF * BUF);  // TMA: one mbarrier per buffer
    // flags in dynamic shared memory (the kernel declares no static shared variables)
    int& last = *reinterpret_cast<int*>(smem + NBUF * BUF + 32);
    int& tma_ok = *reinterpret_cast<int*>(smem + NBUF * BUF + 36);
    // row of this (slot, KV head)'s position 0 in the tensor maps' [rows][hd] view
    const int row0 = TMA ? int((int64_t(slot) * a.slot_stride + int64_t(kvh) * a.head_stride) / HD) : 0;
    auto issue = [&](int cc) {
        const int j0 = j_begin + cc * CH, n = min(CH, j_end - j0);
        uint8_t* dst = smem + (cc % NBUF) * BUF;
        if constexpr (TMA) {  // thread 0 only
            uint64_t* bar = &bars[cc % NBUF];
            mbar_arrive_expect_tx(bar, uint32_t(BUF));
#pragma unroll
            for (int bx = 0; bx < NB; bx++) {
                tma_load_2d(dst + bx * kTmaBox, &tk, 64 * bx, row0 + j0, bar);
                tma_load_2d(dst + (NB + bx) * kTmaBox, &tv, 64 * bx, row0 + j0, bar);
            }
        } else {
            uint16_t* dk = reinterpret_cast<uint16_t*>(dst);
            constexpr int PR = HD / 8;  // pieces per row
#pragma unroll 4
            for (int i = tid; i < 2 * CH * PR; i += NT) {
                const int v = i >= CH * PR ? 1 : 0, j = (i - v * CH * PR) / PR, q = i - v * CH * PR - j * PR;
                const uint16_t* src = (v ? vbase : kbase) + int64_t(j0 + min(j, n - 1)) * a.pos_stride + 8 * q;
                cp16(dk + (v * CH + j) * P + 8 * q, src, j < n ? 16 : 0);
            }
        }
    };
    if constexpr (TMA) {
        if (tid == 0) {
            // the copies need a 1024-byte aligned destination, 8-byte aligned barriers and 64-byte aligned maps:
            // anything else is recorded and the copies are skipped (the outputs are then invalid)
            tma_ok = 1;
            if ((smem_u32(smem) & 1023u) || (smem_u32(bars) & 7u)) {
                set_device_error(kErrMisalignedSmem);
                tma_ok = 0;
            } else if ((reinterpret_cast<uintptr_t>(&tk) & 63u) || (reinterpret_cast<uintptr_t>(&tv) & 63u)) {
                set_device_error(kErrMisalignedMap);
                tma_ok = 0;
            }
#pragma unroll
            for (int b = 0; b < NBUF; b++) mbar_init(&bars[b], 1);
            fence_barrier_init();
            if (tma_ok) {
#pragma unroll
                for (int cc = 0; cc < NBUF - 1; cc++)
                    if (cc < nchunks) issue(cc);
            }
        }
        __syncthreads();  // barrier initialisation visible before any thread waits
    } else {
#pragma unroll
        for (int cc = 0; cc < NBUF - 1; cc++) {
            if (cc < nchunks) issue(cc);
            cp_commit();
        }
    }
    // Fused decode (qkv_post's arithmetic, k_ops.cu): the group's query heads, and in the split that holds
    // position pos the new key and value, prepared into shared memory; the key / value rows also go to the caches
    float* qs = reinterpret_cast<float*>(smem + NBUF * BUF + 64);  // [kMaxGroup + 2][HD]: q heads, k, v
    const bool fused = TMA && a.fuse_post;
    const bool owns_new = fused && j_end == L;
    if (fused) {
        // tasks: the G query heads, then (the split holding pos) the key and the value head; warp w takes tasks
        // w, w + W, ... Lane l holds dims l + 32j (j < J), so each rotation pair (i, i + HD / 2) is in one lane
        // (j and j + J / 2). Every load is issued before the arithmetic.
        constexpr int J = HD / 32, TMAX = (kMaxGroup + 2 + W - 1) / W;
        const float* qkv_row = a.q + int64_t(r) * a.q_stride;
        const int tasks = G + (owns_new ? 2 : 0);
        float x[TMAX][J], wq[J], wk[J], co[J / 2], sn[J / 2];
#pragma unroll
        for (int k = 0; k < TMAX; k++) {
            const int t = warp + k * W;
            if (t < tasks) {
                const int col = t < G ? (kvh * G + t) * HD : (t == G ? a.k_off : a.v_off) + kvh * HD;
#pragma unroll
                for (int j = 0; j < J; j++) x[k][j] = qkv_row[col + lane + 32 * j];
            }
        }
        const float* cs = a.post_cs + int64_t(pos) * HD;
#pragma unroll
        for (int j = 0; j < J; j++) {
            wq[j] = a.post_wn[lane + 32 * j];
            wk[j] = a.post_wn[HD + lane + 32 * j];
        }
#pragma unroll
        for (int j = 0; j < J / 2; j++) {
            co[j] = cs[2 * (lane + 32 * j)];
            sn[j] = cs[2 * (lane + 32 * j) + 1];
        }
#pragma unroll
        for (int k = 0; k < TMAX; k++) {
            const int t = warp + k * W;
            if (t >= tasks) break;  // warp-uniform
            const bool isq = t < G, isk = t == G;
            float* v = qs + (isq ? t : kMaxGroup + (isk ? 0 : 1)) * HD;
            float y[J];
#pragma unroll
            for (int j = 0; j < J; j++) y[j] = x[k][j];
            if (isq || isk) {  // per-head RMSNorm (sum of squares in double), then the NeoX rotation
                double ss = 0.0;
#pragma unroll
                for (int j = 0; j < J; j++) ss += double(y[j]) * y[j];
                const float sc = float(1.0 / sqrt(warp_sum_dbl(ss) / HD + double(a.post_eps)));
#pragma unroll
                for (int j = 0; j < J; j++) y[j] = __fmul_rn(__fmul_rn(y[j], sc), isq ? wq[j] : wk[j]);
#pragma unroll
                for (int j = 0; j < J / 2; j++) {
                    const float x0 = y[j], x1 = y[j + J / 2];
                    y[j] = __fsub_rn(__fmul_rn(x0, co[j]), __fmul_rn(x1, sn[j]));
                    y[j + J / 2] = __fadd_rn(__fmul_rn(x0, sn[j]), __fmul_rn(x1, co[j]));
                }
            }
#pragma unroll
            for (int j = 0; j < J; j++) v[lane + 32 * j] = y[j];
            if (!isq) {  // the new cache row
                uint16_t* dst = const_cast<uint16_t*>(isk ? a.kc : a.vc) + int64_t(slot) * a.slot_stride +
                                int64_t(pos) * a.pos_stride + int64_t(kvh) * a.head_stride;
#pragma unroll
                for (int j = 0; j < J; j++) dst[lane + 32 * j] = __half_as_ushort(__float2half_rn(y[j]));
            }
        }
        __syncthreads();
    }
    // shared-memory address of (row, 8-half piece q) of the key (v = 0) or value (v = 1) tile in buffer b
    auto tile_addr = [&](int b, int v, int row, int q) -> const void* {
        if constexpr (TMA)
            return smem + b * BUF + (v * NB + (q >> 3)) * kTmaBox + row * 128 + (((q & 7) ^ (row & 7)) << 4);
        else
            return kvb + (b * 2 + v) * CH * P + row * P + 8 * q;
    };

    // query fragments (row gr = query head gr of the group; rows 8..15 and heads past G are zero)
    uint32_t qh[KS][2], ql[KS][2];
    {
        const float* qrow = fused ? qs + gr * HD : a.q + int64_t(r) * a.q_stride + int64_t(kvh * G + gr) * HD;
#pragma unroll
        for (int ks = 0; ks < KS; ks++)
#pragma unroll
            for (int h = 0; h < 2; h++) {
                const int d = 16 * ks + 8 * h + 2 * c;
                const float x0 = gr < G ? qrow[d] : 0.0f, x1 = gr < G ? qrow[d + 1] : 0.0f;
                split_hilo(x0, x1, qh[ks][h], ql[ks][h]);
            }
    }
    // lane (g, c) keeps heads 2c, 2c + 1 of the group: their running max and its share of the running sum, and
    // the P.V accumulators O^T[dim][head] of dims 16t + g and 16t + g + 8
    float o[MT][4];
#pragma unroll
    for (int t = 0; t < MT; t++) o[t][0] = o[t][1] = o[t][2] = o[t][3] = 0.0f;
    float m_run[2] = {-INFINITY, -INFINITY}, l_part[2] = {0.0f, 0.0f};
    const int k0 = 16 * warp;

    for (int cc = 0; cc < nchunks; cc++) {
        const int b = cc % NBUF, n = min(CH, j_end - (j_begin + cc * CH));
        if constexpr (TMA) {
            if (tma_ok) mbar_wait(&bars[b], uint32_t(cc / NBUF) & 1u);  // chunk cc landed (bounded)
            if (n < CH) {  // value rows past the last key: zeros (0 x inf or NaN in stale rows would poison P.V)
                uint8_t* vz = smem + b * BUF + NB * kTmaBox;
                for (int i = tid; i < NB * (CH - n) * 8; i += NT) {
                    const int bx = i / ((CH - n) * 8), rem = i - bx * (CH - n) * 8;
                    *reinterpret_cast<uint4*>(vz + bx * kTmaBox + (n + (rem >> 3)) * 128 + 16 * (rem & 7)) =
                        make_uint4(0u, 0u, 0u, 0u);
                }
            }
            if (owns_new && pos - (j_begin + cc * CH) < CH) {  // the new key / value row, as the caches now hold
                const int jr = pos - (j_begin + cc * CH);
                for (int i = tid; i < 2 * (HD / 8); i += NT) {
                    const int vs = i / (HD / 8), q = i - vs * (HD / 8);
                    const float* src = qs + (kMaxGroup + vs) * HD + 8 * q;
                    uint4 pk;
                    pk.x = h2u(__floats2half2_rn(src[0], src[1]));
                    pk.y = h2u(__floats2half2_rn(src[2], src[3]));
                    pk.z = h2u(__floats2half2_rn(src[4], src[5]));
                    pk.w = h2u(__floats2half2_rn(src[6], src[7]));
                    *reinterpret_cast<uint4*>(const_cast<void*>(tile_addr(b, vs, jr, q))) = pk;
                }
            }
            __syncthreads();  // zeroed and new rows visible; every warp is done with chunk cc - 1's buffer
            if (tid == 0 && tma_ok && cc + NBUF - 1 < nchunks) issue(cc + NBUF - 1);
        } else {
            cp_wait<NBUF - 2>();  // chunk cc landed (this thread's pieces)
            __syncthreads();         // ... every thread's; and every warp is done with chunk cc - 1's buffer
            if (cc + NBUF - 1 < nchunks) issue(cc + NBUF - 1);
            cp_commit();
        }
        if (k0 < n) {
            // scores S^T[key][head] of keys k0..k0+15 (the MMA's rows) and the group's heads (its columns): A = key
            // rows by ldmatrix, B = the query fragments; hi and lo products of even and odd k-steps in four
            // independent accumulators
            float sa[4][4];
#pragma unroll
            for (int ks = 0; ks < KS; ks++) {
                uint32_t kf[4];
                ldsm_x4(kf, tile_addr(b, 0, k0 + (lane & 15), 2 * ks + (lane >> 4)));
                float(&sh)[4] = sa[2 * (ks & 1)];
                float(&sl)[4] = sa[2 * (ks & 1) + 1];
                if (ks < 2) {
                    mma16816_z(sh, kf, qh[ks][0], qh[ks][1]);
                    mma16816_z(sl, kf, ql[ks][0], ql[ks][1]);
                } else {
                    mma16816(sh, kf, qh[ks][0], qh[ks][1]);
                    mma16816(sl, kf, ql[ks][0], ql[ks][1]);
                }
            }
            // s4[0], s4[1]: key k0 + gr, heads 2c, 2c + 1; s4[2], s4[3]: key k0 + gr + 8
            float s4[4];
            const bool v0 = k0 + gr < n, v1 = k0 + gr + 8 < n;
#pragma unroll
            for (int e = 0; e < 4; e++) {
                const float t = (sa[0][e] + sa[1][e]) + (sa[2][e] + sa[3][e]);
                s4[e] = (e < 2 ? v0 : v1) ? t * a.scale : -INFINITY;
            }
            // online softmax per head over the warp's keys (the 8 lanes of a column hold them)
            float mx0 = fmaxf(s4[0], s4[2]), mx1 = fmaxf(s4[1], s4[3]);
#pragma unroll
            for (int off = 4; off < 32; off <<= 1) {
                mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, off));
                mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, off));
            }
            const float mn0 = fmaxf(m_run[0], mx0), mn1 = fmaxf(m_run[1], mx1);  // finite: key k0 < n
            const float c0 = expf(m_run[0] - mn0), c1 = expf(m_run[1] - mn1);    // 0 on the first keys
            l_part[0] *= c0;
            l_part[1] *= c1;
#pragma unroll
            for (int t = 0; t < MT; t++) {
                o[t][0] *= c0;
                o[t][2] *= c0;
                o[t][1] *= c1;
                o[t][3] *= c1;
            }
            const float p0 = expf(s4[0] - mn0), p1 = expf(s4[1] - mn1), p2 = expf(s4[2] - mn0),
                        p3 = expf(s4[3] - mn1);
            l_part[0] += p0 + p2;
            l_part[1] += p1 + p3;
            m_run[0] = mn0;
            m_run[1] = mn1;
            // P^T as the B fragment of P.V: lane (g, c) needs P[keys 2c, 2c+1, 2c+8, 2c+9][head g], held by lanes
            // (2c, g / 2) and (2c + 1, g / 2) in their head-(g & 1) registers
            const int sA = 8 * c + (gr >> 1), sB = sA + 4;
            const bool odd = gr & 1;
            const float e0 = __shfl_sync(0xffffffffu, p0, sA), q0 = __shfl_sync(0xffffffffu, p1, sA);
            const float e1 = __shfl_sync(0xffffffffu, p0, sB), q1 = __shfl_sync(0xffffffffu, p1, sB);
            const float e2 = __shfl_sync(0xffffffffu, p2, sA), q2 = __shfl_sync(0xffffffffu, p3, sA);
            const float e3 = __shfl_sync(0xffffffffu, p2, sB), q3 = __shfl_sync(0xffffffffu, p3, sB);
            uint32_t bh0, bl0, bh1, bl1;
            split_hilo(odd ? q0 : e0, odd ? q1 : e1, bh0, bl0);
            split_hilo(odd ? q2 : e2, odd ? q3 : e3, bh1, bl1);
            // O^T[dim][head] += V^T[dim][key] . P^T[key][head]: A = value rows, transposed by ldmatrix
#pragma unroll
            for (int t = 0; t < MT; t++) {
                uint32_t vf[4];
                ldsm_x4_trans(vf, tile_addr(b, 1, k0 + (lane & 7) + 8 * (lane >> 4), 2 * t + ((lane >> 3) & 1)));
                mma16816(o[t], vf, bh0, bh1);
                mma16816(o[t], vf, bl0, bl1);
            }
        }
    }

    // The next kernel may launch now: earlier, its CTAs (waiting on this grid) would take the shared memory that
    // lets four of these CTAs share an SM.
    pdl_trigger();
    // merge the warps (the buffers are free once every warp is past its last chunk)
    __syncthreads();
#pragma unroll
    for (int off = 4; off < 32; off <<= 1) {
        l_part[0] += __shfl_xor_sync(0xffffffffu, l_part[0], off);
        l_part[1] += __shfl_xor_sync(0xffffffffu, l_part[1], off);
    }
    float* wm = reinterpret_cast<float*>(smem);  // [W][8] max
    float* wl = wm + 8 * W;                      // [W][8] sum
    float* wo = wl + 8 * W;                      // [W][8][HD] acc
    static_assert((16 * W + 8 * W * HD) * 4 <= NBUF * BUF, "the warp merge fits the buffers");
#pragma unroll
    for (int e = 0; e < 2; e++) {
        const int h = 2 * c + e;
        if (h < G) {
            if (gr == 0) {
                wm[warp * 8 + h] = m_run[e];
                wl[warp * 8 + h] = l_part[e];
            }
#pragma unroll
            for (int t = 0; t < MT; t++) {
                wo[(warp * 8 + h) * HD + 16 * t + gr] = o[t][e];
                wo[(warp * 8 + h) * HD + 16 * t + gr + 8] = o[t][2 + e];
            }
        }
    }
    __syncthreads();
    const bool split_mode = active > 1;
    const int64_t rec = HD + 2;
    for (int i = tid; i < G * HD; i += NT) {
        const int g = i / HD, d = i - g * HD;
        float M = -INFINITY;
#pragma unroll
        for (int w = 0; w < W; w++) M = fmaxf(M, wm[w * 8 + g]);
        float num = 0.0f, den = 0.0f;
#pragma unroll
        for (int w = 0; w < W; w++) {
            const float f = expf(wm[w * 8 + g] - M);  // 0 for a warp that saw no keys (max -inf)
            num += f * wo[(w * 8 + g) * HD + d];
            den += f * wl[w * 8 + g];
        }
        if (!split_mode) {
            store_out(a, r, (kvh * G + g) * HD + d, num / den);
        } else {
            float* pr = a.part + ((int64_t(r) * a.n_head + kvh * G + g) * geo.splits + split) * rec;
            if (d == 0) {
                pr[0] = M;
                pr[1] = den;
            }
            pr[2 + d] = num;
        }
    }
    if (!split_mode) return;
    __threadfence();
    __syncthreads();
    if (tid == 0) {
        unsigned* t = a.tickets + int64_t(r) * a.n_kv + kvh;
        const unsigned ticket = atomicAdd(t, 1u);
        last = ticket == unsigned(active - 1);
        if (last) *t = 0u;  // every CTA of this (row, KV head) has taken its ticket: reset for the next launch
    }
    __syncthreads();
    if (!last) return;
    __threadfence();
    for (int i = tid; i < G * HD; i += NT) {
        const int g = i / HD, d = i - g * HD;
        const float* base = a.part + (int64_t(r) * a.n_head + kvh * G + g) * geo.splits * rec;
        float M = -INFINITY;
        for (int sp = 0; sp < active; sp++) M = fmaxf(M, __ldcg(base + sp * rec));
        float num = 0.0f, den = 0.0f;
        for (int sp = 0; sp < active; sp++) {
            const float w = expf(__ldcg(base + sp * rec) - M);
            den += __ldcg(base + sp * rec + 1) * w;
            num += __ldcg(base + sp * rec + 2 + d) * w;
        }
        store_out(a, r, (kvh * G + g) * HD + d, num / den);
    }
}

Geometry plan(int rows, int n_kv, int max_pos, int G, int hd, bool tma) {
    const int L = max_pos + 1;
    const int sms = num_sms();
    Geometry g;
    if (tma) {  // TMA tensor-core kernel: splits that fill the four CTAs per SM once, at least 128 keys each
        g.chunk = kTmaChunk;
        const int items = std::max(1, rows * n_kv);
        const int want = std::max(1, std::min(kTcCtasTma * sms / items, L / 128));
        g.span = std::max(g.chunk, ((L + want - 1) / want + g.chunk - 1) / g.chunk * g.chunk);
        g.splits = (L + g.span - 1) / g.span;
        g.smem = 0;
        return g;
    }
    g.chunk = chunk_for(hd);
    // about two CTAs per SM, at least two chunks of keys per split: a CTA's start-up and its share of the split
    // merge are fixed costs, so long splits win (measured at batch 64, position 512: 1 split per (row, KV head)
    // 3.25 ms per decode step, 2 splits 3.59 ms, 3 splits 3.72 ms)
    const int want = std::max(1, std::min((2 * sms + rows * n_kv - 1) / (rows * n_kv), L / (2 * g.chunk)));
    int span = (L + want - 1) / want;
    span = std::max(g.chunk, (span + g.chunk - 1) / g.chunk * g.chunk);
    g.span = span;
    g.splits = (L + span - 1) / span;
    g.smem = layout(G, hd, g.chunk).total;
    return g;
}

}  // namespace

void attention_scratch(int rows, int n_head, int n_kv, int hd, int max_pos, int64_t* part_floats, int64_t* tickets,
                       bool tma) {
    const int G = n_head / std::max(1, n_kv);
    int splits = plan(rows, n_kv, max_pos, G, hd, false).splits;
    if (tma && (hd == 64 || hd == 128) && G <= 8)
        splits = std::max(splits, plan(rows, n_kv, max_pos, G, hd, true).splits);
    *part_floats = splits > 1 ? int64_t(rows) * n_head * splits * (hd + 2) : 0;
    *tickets = int64_t(rows) * n_kv;
}

bool attention_shape_ok(int n_head, int n_kv, int hd) {
    return n_kv > 0 && n_head > 0 && n_head % n_kv == 0 && n_head / n_kv <= kMaxGroup && hd > 0 && hd <= kMaxHd &&
           hd % 8 == 0;
}

cudaError_t launch_attention(const AttnArgs& a, cudaStream_t st, bool pdl) {
    if (a.rows <= 0) return cudaSuccess;
    if (!attention_shape_ok(a.n_head, a.n_kv, a.hd)) return cudaErrorInvalidValue;
    // bulk copies need 16-byte aligned key rows
    if ((a.pos_stride % 8) || (a.head_stride % 8) || (a.slot_stride % 8) ||
        (reinterpret_cast<uintptr_t>(a.kc) & 15) || (reinterpret_cast<uintptr_t>(a.vc) & 15))
        return cudaErrorInvalidValue;
    const int G = a.n_head / a.n_kv;
    const bool tc_shape = (a.hd == 64 || a.hd == 128) && G <= 8;
    // TMA staging when every (slot, KV head) holds its positions as consecutive hd-element rows of a known
    // [cache_rows][hd] array, and both tensor maps encode
    CUtensorMap tk{}, tv{};
    static const bool tma_on = [] {
        const char* e = std::getenv("NEKO_ATTN_TMA");
        return !(e && e[0] == '0');
    }();
    const bool tma = tc_shape && tma_on && a.pos_stride == a.hd && a.cache_rows > 0 &&
                     a.cache_rows < (int64_t(1) << 31) && a.slot_stride % a.hd == 0 && a.head_stride % a.hd == 0 &&
                     encode_f16_2d_sw128(&tk, a.kc, uint64_t(a.hd), uint64_t(a.cache_rows), uint64_t(a.hd) * 2, 64,
                                         kTmaChunk) &&
                     encode_f16_2d_sw128(&tv, a.vc, uint64_t(a.hd), uint64_t(a.cache_rows), uint64_t(a.hd) * 2, 64,
                                         kTmaChunk);
    const Geometry g = plan(a.rows, a.n_kv, a.max_pos, G, a.hd, tma);
    if (g.splits > 1) {
        const int64_t need = int64_t(a.rows) * a.n_head * g.splits * (a.hd + 2);
        if (!a.part || !a.tickets || need > a.part_capacity || int64_t(a.rows) * a.n_kv > a.ticket_capacity)
            return cudaErrorInvalidValue;
    }
    const bool tc = tc_shape && (tma || kTcChunk == g.chunk);
    if (a.fuse_post && (!tma || !a.post_wn || !a.post_cs || a.k_off < 0 || a.v_off < 0)) return cudaErrorNotSupported;
    if (a.out_hi && (!tc || !a.out_lo || a.out_hl_stride < int64_t(a.n_head) * a.hd)) return cudaErrorInvalidValue;
    if (tc) {  // tensor-core kernel
        auto k = a.hd == 128 ? (tma ? attention_tc_kernel<128, true> : attention_tc_kernel<128, false>)
                             : (tma ? attention_tc_kernel<64, true> : attention_tc_kernel<64, false>);
        const int smem = a.hd == 128 ? (tma ? tc_attn_smem<128, true>() : tc_attn_smem<128, false>())
                                     : (tma ? tc_attn_smem<64, true>() : tc_attn_smem<64, false>());
        static int attr_tc[2][2][8] = {};  // per head_dim, staging, device < 8
        int dev = 0;
        cudaGetDevice(&dev);
        if (dev >= 8 || !attr_tc[a.hd == 128][tma][dev]) {
            if (cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
                e != cudaSuccess)
                return e;
            if (dev < 8) attr_tc[a.hd == 128][tma][dev] = 1;
        }
        return launch_ex(k, dim3(g.splits, a.n_kv, a.rows), dim3(32 * tc_warps(tma)), size_t(smem), st, pdl, a, g, tk,
                         tv);
    }
    static unsigned attr_done = 0u;  // bit d: device d (< 32); function attributes are per device
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 32 || !((attr_done >> dev) & 1u)) {
        if (cudaError_t e = cudaFuncSetAttribute(attention_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                 160 * 1024);
            e != cudaSuccess)
            return e;
        if (dev < 32) attr_done |= 1u << dev;
    }
    return launch_ex(attention_kernel, dim3(g.splits, a.n_kv, a.rows), dim3(kAttnThreads), size_t(g.smem), st, pdl, a,
                     g);
}

}  // namespace neko
