// Decode-step kernel: one persistent, cooperative launch runs a whole decode step of 1..4 sequences -- token
// embedding, every layer of Qwen3ForwardGpu / Gpt2ForwardGpu (qwen3_model.cpp:300-340, gpt2_model.cpp:180-215),
// the final norm, the tied LM head and the greedy argmax -- instead of ~6 dependent launches per layer.
//
// Why: at batch 1 each matrix of Qwen3-0.6B is 1-6 MB, under a microsecond of HBM time, while a dependent kernel
// launch plus its activation round trip costs several microseconds. Here the weights never wait for the math:
//  * one CTA per SM (all co-resident), 12 consumer warps + 1 producer warp;
//  * every CTA owns a fixed row range of every matrix; its producer warp streams those rows, phase after phase
//    and layer after layer, through a ring of shared-memory slots with cp.async.bulk (TMA), gated only by free
//    slots, so the next matrices are already on chip while the current phase waits for its inputs;
//  * phases hand their outputs over as tagged words: every output element is stored as one 64-bit word, the
//    float's bits in the low half and the exchange's tag (step epoch + layer + phase) in the high half, with a
//    single-copy-atomic 64-bit store. A consumer issues all of its loads at once and reloads only the words whose
//    tag is not the expected one yet, so the data carries its own readiness: one L2 round trip per hand-off, no
//    counters, fences or tickets (measured on B200: 1.2 us per grid-wide hand-off of a 1024-float vector, against
//    2.5 us for a release counter followed by the data reads);
//  * attention items (sequence, KV head, key span) fold in the per-head QK RMSNorm, RoPE and the f16 KV store;
//    when a head's keys are split over several items, their partial softmax states are merged by idle warps of
//    other CTAs in a separate hand-off;
//  * the residual stream: the CTA that owns rows of x (the o_proj / down rows) keeps them in shared memory and
//    publishes each update;
//  * Qwen3's RMSNorm before a matrix is applied in the GEMV epilogue: the staged activations are x * gamma and
//    the row's dot product is multiplied by rstd = 1 / sqrt(mean(x^2) + eps), which is the same RMSNorm since
//    W (x rstd gamma) = rstd (W (x gamma)); the sums of squares ride on the staging pass, so it needs one barrier.
// The dot products and activation layout are the GEMV kernel's (same summation order).
//
// Every wait is bounded (DecodeParams::wait_ns on %globaltimer, 2 s by default): on expiry the kernel records
// kErrMbarTimeout, raises an abort flag that makes every other wait return at once, and the producer waits
// (bounded) for its copies in flight before leaving. Waits that can fail are combined over the CTA's consumer
// threads with a reducing barrier, so the threads leave together. The last CTA to finish finalises the greedy
// tokens, resets the step counter and advances the epoch, so the launch replays from a CUDA graph.
#include <algorithm>

#include "gemv_core.cuh"
#include "mma_frag.cuh"
#include "neko_common.cuh"
#include "neko_internal.h"

namespace neko {

namespace {

constexpr int kW = 12;                 // consumer warps (12 + 1 warps: at most 128 registers a thread)
constexpr int kNT = kW * 32;           // consumer threads
constexpr int kThr = kNT + 32;         // + the producer warp
constexpr int kMaxSlots = 16;
constexpr int kSlotBytes = 32768;      // bigger stages stream faster (fewer producer / consumer hand-offs)
constexpr int kMaxGroupRows = kW * 4;  // rows the CTA consumes per pass, at most (kRows<1> warps x 4)
constexpr int kMaxStatSlots = 256;     // LayerNorm partial-sum slots (kGatherE * kW used)
constexpr int kChunk = 8192;           // bytes per bulk copy
constexpr int kMaxGq = 4;              // query heads per KV head
constexpr int kMaxSpan = 64;           // keys per attention item (staged in shared memory)
constexpr int kOwnRows = 32;           // residual rows a CTA owns, at most (C <= 32 * grid)
constexpr int kGatherE = 2;            // float4 groups a thread has in flight per gather batch
constexpr int kMergeS = 8;             // split states a merge warp has in flight per batch

enum Ph : int { kQkv = 0, kAttn = 1, kO = 2, kUp = 3, kDown = 4, kHead = 5 };
// Exchanges (tag offsets) per layer. The LM head reads x under layer L's kXIn.
enum Xch : unsigned { kXIn = 0, kXQkv = 1, kXPart = 2, kXAtt = 3, kXMid = 4, kXH = 5, kXPer = 8 };

__device__ unsigned g_dec_abort;  // raised by the first wait that gives up

__device__ __forceinline__ uint64_t gtimer() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}
__device__ __forceinline__ void csync() { asm volatile("bar.sync 1, %0;" ::"n"(kNT) : "memory"); }
// Consumer barrier that also ANDs a predicate over the consumer threads.
__device__ __forceinline__ bool csync_and(bool ok) {
    unsigned r;
    asm volatile(
        "{\n\t.reg .pred p, q;\n\t"
        "setp.ne.u32 q, %1, 0;\n\t"
        "bar.red.and.pred p, 1, %2, q;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(r)
        : "r"(ok ? 1u : 0u), "n"(kNT)
        : "memory");
    return r != 0;
}
__device__ __forceinline__ bool aborted() { return *reinterpret_cast<volatile unsigned*>(&g_dec_abort) != 0u; }
__device__ __forceinline__ void give_up() {
    set_device_error(kErrMbarTimeout);
    atomicExch(&g_dec_abort, 1u);
}
__device__ __forceinline__ double wsum_d(double v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// ---------------------------------------------------------------------------------------------- tagged words
__device__ __forceinline__ void tw_put(uint64_t* p, float v, unsigned tag) {
    const uint64_t w = (uint64_t(tag) << 32) | __float_as_uint(v);
    asm volatile("st.relaxed.gpu.global.u64 [%0], %1;" ::"l"(p), "l"(w) : "memory");
}
__device__ __forceinline__ void tw_ld2(const uint64_t* p, uint64_t& a, uint64_t& b) {  // 16-byte aligned pair
    asm volatile("ld.relaxed.gpu.global.v2.u64 {%0, %1}, [%2];" : "=l"(a), "=l"(b) : "l"(p) : "memory");
}
__device__ __forceinline__ uint64_t tw_ld(const uint64_t* p) {
    uint64_t w;
    asm volatile("ld.relaxed.gpu.global.u64 %0, [%1];" : "=l"(w) : "l"(p) : "memory");
    return w;
}
__device__ __forceinline__ bool tw_ok(uint64_t w, unsigned tag) { return unsigned(w >> 32) == tag; }
__device__ __forceinline__ float tw_val(uint64_t w) { return __uint_as_float(unsigned(w)); }

// Poll bookkeeping shared by the gathers: false once the wait has run past lim (reported) or another wait gave up.
// The clock is read at the first retry and checked with the abort flag (a global load) every 16th retry only, so
// a retry costs no more than the reload itself.
struct Poll {
    uint64_t t0 = 0;
    uint32_t n = 0;
    __device__ __forceinline__ bool keep_going(uint64_t lim) {
        if (n++ == 0u) {
            t0 = gtimer();
            return true;
        }
        if (n & 15u) return true;
        if (aborted()) return false;
        if (gtimer() - t0 > lim) {
            give_up();
            return false;
        }
        return true;
    }
};

// E groups of 4 consecutive tagged words (group q at src + 4 q, for the q of this thread that are < nq): every
// load in flight at once, then only the groups with a stale tag are reloaded. False on timeout or abort.
template <int E>
__device__ bool gather4(const uint64_t* src, const int (&q)[E], int nq, unsigned tag, float4 (&out)[E],
                        uint64_t lim) {
    uint64_t w[E][4];
#pragma unroll
    for (int e = 0; e < E; e++)
        if (q[e] < nq) {
            tw_ld2(src + 4 * int64_t(q[e]), w[e][0], w[e][1]);
            tw_ld2(src + 4 * int64_t(q[e]) + 2, w[e][2], w[e][3]);
        }
    Poll pl;
    for (;;) {
        unsigned miss = 0;
#pragma unroll
        for (int e = 0; e < E; e++)
            if (q[e] < nq && !(tw_ok(w[e][0], tag) && tw_ok(w[e][1], tag) && tw_ok(w[e][2], tag) && tw_ok(w[e][3], tag)))
                miss |= 1u << e;
        if (!miss) break;
        if (!pl.keep_going(lim)) return false;
#pragma unroll
        for (int e = 0; e < E; e++)
            if (miss >> e & 1u) {
                tw_ld2(src + 4 * int64_t(q[e]), w[e][0], w[e][1]);
                tw_ld2(src + 4 * int64_t(q[e]) + 2, w[e][2], w[e][3]);
            }
    }
#pragma unroll
    for (int e = 0; e < E; e++)
        out[e] = make_float4(tw_val(w[e][0]), tw_val(w[e][1]), tw_val(w[e][2]), tw_val(w[e][3]));
    return true;
}

// N tagged words src[stride * i], i < N, for one lane. False on timeout or abort.
template <int N>
__device__ bool gather_lane(const uint64_t* src, int stride, unsigned tag, float (&out)[N], uint64_t lim) {
    uint64_t w[N];
#pragma unroll
    for (int i = 0; i < N; i++) w[i] = tw_ld(src + int64_t(i) * stride);
    Poll pl;
    for (;;) {
        unsigned miss = 0;
#pragma unroll
        for (int i = 0; i < N; i++)
            if (!tw_ok(w[i], tag)) miss |= 1u << i;
        if (!miss) break;
        if (!pl.keep_going(lim)) return false;
#pragma unroll
        for (int i = 0; i < N; i++)
            if (miss >> i & 1u) w[i] = tw_ld(src + int64_t(i) * stride);
    }
#pragma unroll
    for (int i = 0; i < N; i++) out[i] = tw_val(w[i]);
    return true;
}

// try_wait with a suspend-time hint: the thread sleeps until the phase completes or hint_ns pass, instead of
// spinning (a spinning warp takes issue slots and instruction fetches from the warps doing the math).
__device__ __forceinline__ bool mbar_try_wait_sleep(uint64_t* bar, uint32_t parity, uint32_t hint_ns) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity), "r"(hint_ns)
        : "memory");
    return ok != 0;
}

// Bounded mbarrier wait for the decode kernel (gives up on abort or after lim ns). Out of line: callers try the
// barrier once first, and the kernel's code is kept small (instruction fetch is on its critical path).
__device__ __noinline__ bool dwait(uint64_t* bar, uint32_t parity, uint64_t lim, uint32_t hint_ns = 20000) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = gtimer();
    for (;;) {
        if (mbar_try_wait_sleep(bar, parity, hint_ns)) return true;
        if (aborted()) return false;
        if (gtimer() - t0 > lim) {
            give_up();
            return false;
        }
    }
}

// ---------------------------------------------------------------------------------------------- shared memory
// Shared-memory state of the kernel at fixed offsets of the dynamic region, so the phase functions address it
// directly (a struct of pointers passed around ends up in local memory and puts a load on every access):
// barriers | DShared | layer table | activations | keys/values | ring. The small arrays are not file-scope
// __shared__ variables: the device linker places those in one window shared with the other files' and the
// kernel's static shared memory would grow with them.
extern __shared__ __align__(128) uint8_t dsm[];
struct DShared {
    double part[2 * kMaxStatSlots];             // LayerNorm prologue partial sums
    double ss[kW][kDecodeMaxSeqs];              // RMSNorm: per-warp sums of squares of the staged rows
    float xown[kDecodeMaxSeqs][kOwnRows];       // the residual rows this CTA owns
    unsigned long long key[kDecodeMaxSeqs];     // LM head: the CTA's greedy argmax keys
    uint64_t attn_bar;                          // an attention item's keys / values have landed
    int last;
    int span;                                   // keys per attention split this step (p.span: the buffers' bound)
    unsigned epoch;
};
constexpr int kDHdr = 256 + int(sizeof(DShared) + 127) / 128 * 128;  // bytes before the layer table
__device__ __forceinline__ DShared& dsh() { return *reinterpret_cast<DShared*>(dsm + 256); }
__device__ __forceinline__ uint64_t* full_bar() { return reinterpret_cast<uint64_t*>(dsm); }
__device__ __forceinline__ uint64_t* empty_bar() { return reinterpret_cast<uint64_t*>(dsm) + kMaxSlots; }
__device__ __forceinline__ const DecodeLayer* layer_tab() { return reinterpret_cast<const DecodeLayer*>(dsm + kDHdr); }
__device__ __forceinline__ int tab_bytes(const DecodeParams& p) {
    return (p.layers * int(sizeof(DecodeLayer)) + 127) / 128 * 128;
}
__device__ __forceinline__ float* xs_buf(const DecodeParams& p) {
    return reinterpret_cast<float*>(dsm + kDHdr + tab_bytes(p));
}
__device__ __forceinline__ uint16_t* kv_buf(const DecodeParams& p) {
    return reinterpret_cast<uint16_t*>(dsm + kDHdr + tab_bytes(p) + p.xs_bytes);
}
__device__ __forceinline__ uint8_t* ring_buf(const DecodeParams& p) {
    return dsm + kDHdr + tab_bytes(p) + p.xs_bytes + p.kv_bytes;
}
__device__ __forceinline__ unsigned tag_of(int l, unsigned x) { return dsh().epoch + unsigned(l) * kXPer + x; }

// ---------------------------------------------------------------------------------------------- GEMV phases
struct GemvPh {
    const uint8_t* W;
    int64_t rb;
    int rows, K, pair;   // pair: SwiGLU, gate row n with up row n + rows
    const uint64_t* x;   // tagged input words [M][K]
    unsigned xtag;
    int embed;           // (LayerNorm path) unused
    int norm;
    const float *gamma, *beta, *bias;
    int flags;
    uint64_t* y;         // tagged output words [M][ys] (nullptr: the LM head's plain logits)
    unsigned ytag;
    int64_t ys;
    int resid;           // output rows are residual rows of x (o_proj, down): added to this CTA's copy
    int head;
    float* xout;         // plain output rows [M][ys] instead of tagged words (the last down with x_final)
};

template <int QW>
__device__ __forceinline__ GemvPh gemv_ph(const DecodeParams& p, int l, int kind) {
    GemvPh g{};
    const int lnk = QW ? kNormRms : kNormLayer;
    if (kind == kHead) {
        g.W = p.embed; g.rb = p.rb_c; g.rows = p.V; g.K = p.C;
        g.x = p.x_tw; g.xtag = tag_of(p.layers, kXIn); g.norm = lnk; g.gamma = p.normf; g.beta = p.normfb;
        g.ys = p.V; g.head = 1;
        return g;
    }
    const DecodeLayer& L = layer_tab()[l];
    if (kind == kQkv) {
        g.W = L.wqkv; g.rb = p.rb_c; g.rows = p.QW; g.K = p.C;
        g.x = p.x_tw; g.xtag = tag_of(l, kXIn); g.norm = lnk; g.gamma = L.ln1; g.beta = L.ln1b;
        g.bias = L.bqkv; g.flags = QW ? 0 : kBias; g.y = p.qkv_tw; g.ytag = tag_of(l, kXQkv); g.ys = p.QW;
    } else if (kind == kO) {
        g.W = L.wo; g.rb = p.rb_att; g.rows = p.C; g.K = p.H * p.hd;
        g.x = p.att_tw; g.xtag = tag_of(l, kXAtt);
        g.bias = L.bo; g.flags = QW ? 0 : kBias; g.y = p.x_tw; g.ytag = tag_of(l, kXMid); g.ys = p.C;
        g.resid = 1;
    } else if (kind == kUp) {
        g.W = L.wup; g.rb = p.rb_c; g.rows = p.F; g.K = p.C; g.pair = QW;
        g.x = p.x_tw; g.xtag = tag_of(l, kXMid); g.norm = lnk; g.gamma = L.ln2; g.beta = L.ln2b;
        g.bias = L.bup; g.flags = QW ? 0 : (kBias | kGelu); g.y = p.h_tw; g.ytag = tag_of(l, kXH); g.ys = p.F;
    } else {
        g.W = L.wdown; g.rb = p.rb_f; g.rows = p.C; g.K = p.F;
        g.x = p.h_tw; g.xtag = tag_of(l, kXH);
        g.bias = L.bdown; g.flags = QW ? 0 : kBias; g.y = p.x_tw; g.ytag = tag_of(l + 1, kXIn); g.ys = p.C;
        g.resid = 1;
        if (l == p.layers - 1) g.xout = p.x_final;
    }
    return g;
}

__device__ __forceinline__ void cta_rows(int rows, int grid, int& r0, int& r1) {
    const int rpc = (rows + grid - 1) / grid;
    r0 = min(rows, int(blockIdx.x) * rpc);
    r1 = min(rows, r0 + rpc);
}
// Rows (SwiGLU: gate / up pairs) per ring stage: as many as a slot holds, at most 16 per consumer warp (a stage's
// 16-row tiles are split over the warps along K).
__device__ __forceinline__ int stage_rows(const DecodeParams& p, const GemvPh& g) {
    return min(int(int64_t(p.slot_bytes) / (g.rb * (g.pair ? 2 : 1))), 16 * kW);
}
// GEMV phase kind of the k-th matrix of layer l (l == layers: the LM head).
__device__ __forceinline__ int mat_kind(const DecodeParams& p, int l, int k) {
    return l == p.layers ? kHead : k == 0 ? kQkv : k == 1 ? kO : k == 2 ? kUp : kDown;
}

// ---------------------------------------------------------------------------------------------- producer
template <int QW>
__device__ void producer(const DecodeParams& p, uint64_t* full, uint64_t* empty, uint8_t* ring, int lane) {
    uint32_t st = 0;
    bool ok = true;
    const int last = p.x_final ? p.layers - 1 : p.layers;  // the LM head's weights too unless it runs apart
    for (int l = 0; l <= last && ok; l++) {
        for (int k = 0; k < (l == p.layers ? 1 : 4) && ok; k++) {
            const GemvPh g = gemv_ph<QW>(p, l, mat_kind(p, l, k));
            int r0, r1;
            cta_rows(g.rows, p.grid, r0, r1);
            const int rps = stage_rows(p, g);
            for (int row = r0; row < r1; row += rps, st++) {
                const int slot = int(st % uint32_t(p.nslot));
                if (st >= uint32_t(p.nslot)) {
                    int good = 1;
                    if (lane == 0) good = dwait(&empty[slot], ((st / p.nslot) - 1) & 1, p.wait_ns);
                    if (!__shfl_sync(0xffffffffu, good, 0)) {
                        ok = false;
                        break;
                    }
                }
                const int n = min(rps, r1 - row);
                const uint32_t bytes = uint32_t(n * g.rb);
                uint8_t* dst = ring + size_t(slot) * p.slot_bytes;
                if (lane == 0) mbar_arrive_expect_tx(&full[slot], g.pair ? 2 * bytes : bytes);
                __syncwarp();
                const int nch = int((bytes + kChunk - 1) / kChunk);
                for (int c = lane; c < (g.pair ? 2 : 1) * nch; c += 32) {
                    const int half = c >= nch ? 1 : 0, cc = c - half * nch;
                    const uint32_t off = uint32_t(cc) * kChunk, sz = min(uint32_t(kChunk), bytes - off);
                    bulk_g2s(dst + (half ? bytes : 0) + off,
                             g.W + (int64_t(row) + (half ? g.rows : 0)) * g.rb + off, sz, &full[slot]);
                }
            }
        }
    }
    // Leave only when no copy of ours is in flight (on the abort path the consumers may be gone).
    if (lane == 0) {
        const uint32_t first = st > uint32_t(p.nslot) ? st - uint32_t(p.nslot) : 0u;
        const uint64_t t0 = gtimer();
        for (uint32_t s = first; s < st; s++) {
            while (!mbar_try_wait(&full[s % p.nslot], (s / p.nslot) & 1))
                if (gtimer() - t0 > p.wait_ns) return;
        }
    }
}

// ---------------------------------------------------------------------------------------------- activations
// Token id of sequence m (an id outside the vocabulary is reported and read as 0).
__device__ __forceinline__ int token_of(const DecodeParams& p, int m) {
    const int t = p.tokens[m];
    if (t < 0 || t >= p.V) {
        set_device_error(kErrBadIndex);
        return 0;
    }
    return t;
}

// 1 / sqrt(ss / n + eps) in double, rounded to float (the norms of cpu_ops.cpp:483-511), with CUDA's double
// reciprocal square root: its result differs from the reference's correctly rounded divide and square root by
// far less than the float rounding that follows.
__device__ __forceinline__ float inv_rms(double ss, double inv_n, float eps) {
    return float(rsqrt(ss * inv_n + double(eps)));
}

// rstd of row m from the staging pass's per-warp sums of squares (RMSNorm, cpu_ops.cpp:502-511).
__device__ __forceinline__ float rms_rstd(const DecodeParams& p, int m, int K) {
    double a = 0.0;
#pragma unroll
    for (int w = 0; w < kW; w++) a += dsh().ss[w][m];
    return inv_rms(a, 1.0 / K, p.eps);
}

// ---------------------------------------------------------------------------------------------- GEMV phases, one sequence
// Weight rows a warp walks together (independent load streams): more for one sequence, where the registers of
// the activation tiles are free.
template <int NM>
constexpr int kRows = NM == 1 ? 4 : 2;

// Stages the M input rows of a phase (tagged words) into the permuted layout of the dot products: RMSNorm phases
// store x * gamma and leave per-warp sums of squares in dsh().ss (the epilogue applies rstd); LayerNorm phases
// (GPT-2) normalise in place with the row mean and variance (cpu_ops.cpp:483-500, sums in double). `ok` false:
// this thread's earlier wait failed. Returns false, for every consumer thread alike, when any wait failed or an
// input never arrived.
template <int FMT, int NM>
__device__ bool stage_x(const DecodeParams& p, const GemvPh& g, float* xs, int warp, int lane, bool ok) {
    const int tid = threadIdx.x;
    const int K4 = g.K / 4, nq = p.M * K4, xrow = seg_count(FMT, g.K) * Seg<FMT>::W;
    const bool rms = g.norm == kNormRms, ln = g.norm == kNormLayer;
    double ss[NM];
#pragma unroll
    for (int m = 0; m < NM; m++) ss[m] = 0.0;
    for (int base = 0; base < nq && ok; base += kGatherE * kNT) {
        int q[kGatherE];
        float4 gm[kGatherE];
#pragma unroll
        for (int e = 0; e < kGatherE; e++) {
            q[e] = base + tid + e * kNT;
            if (rms && q[e] < nq) gm[e] = __ldg(reinterpret_cast<const float4*>(g.gamma + 4 * (q[e] % K4)));
        }
        float4 v[kGatherE];
        ok = gather4<kGatherE>(g.x, q, nq, g.xtag, v, p.wait_ns);
        if (!ok) break;
#pragma unroll
        for (int e = 0; e < kGatherE; e++) {
            if (q[e] >= nq) continue;
            const int m = q[e] / K4, k = 4 * (q[e] - m * K4);
            float4 y = v[e];
            if (rms) {
                const double sq = double(y.x) * y.x + double(y.y) * y.y + double(y.z) * y.z + double(y.w) * y.w;
#pragma unroll
                for (int mm = 0; mm < NM; mm++)
                    if (mm == m) ss[mm] += sq;
                y.x = __fmul_rn(y.x, gm[e].x);
                y.y = __fmul_rn(y.y, gm[e].y);
                y.z = __fmul_rn(y.z, gm[e].z);
                y.w = __fmul_rn(y.w, gm[e].w);
            }
            *reinterpret_cast<float4*>(xs + m * xrow + xperm<FMT>(k)) = y;
        }
    }
    if (rms) {
#pragma unroll
        for (int m = 0; m < NM; m++) {
            if (m >= p.M) break;
            const double t = wsum_d(ss[m]);
            if (lane == 0) dsh().ss[warp][m] = t;
        }
    }
    if (!csync_and(ok)) return false;
    if (!ln) return true;
    // LayerNorm: K % 128 == 0, so the 32 float4 of a warp in one pass share a row
    for (int base = 0; base < nq; base += kNT) {
        const int i = base + tid;
        double s1 = 0.0, s2 = 0.0;
        if (i < nq) {
            const int m = i / K4;
            const float4 v = *reinterpret_cast<const float4*>(xs + m * xrow + xperm<FMT>(4 * (i - m * K4)));
            s1 = double(v.x) + double(v.y) + double(v.z) + double(v.w);
            s2 = double(v.x) * v.x + double(v.y) * v.y + double(v.z) * v.z + double(v.w) * v.w;
        }
        if (base + warp * 32 < nq) {
            s1 = wsum_d(s1);
            s2 = wsum_d(s2);
            if (lane == 0) {
                const int qq = base / 32 + warp;
                dsh().part[2 * qq] = s1;
                dsh().part[2 * qq + 1] = s2;
            }
        }
    }
    csync();
    const int gpr = K4 / 32;  // partial slots per row
    for (int i = tid; i < nq; i += kNT) {
        const int m = i / K4, k = 4 * (i - m * K4);
        double a1 = 0.0, a2 = 0.0;
        for (int qq = m * gpr; qq < (m + 1) * gpr; qq++) {
            a1 += dsh().part[2 * qq];
            a2 += dsh().part[2 * qq + 1];
        }
        const double mu = a1 / g.K;
        const float mean = float(mu);
        const float r = float(1.0 / sqrt(a2 / g.K - mu * mu + double(p.eps)));
        float4* px = reinterpret_cast<float4*>(xs + m * xrow + xperm<FMT>(k));
        float4 y = *px;
        const float4 ga = __ldg(reinterpret_cast<const float4*>(g.gamma + k));
        const float4 be = __ldg(reinterpret_cast<const float4*>(g.beta + k));
        y.x = __fadd_rn(__fmul_rn(__fmul_rn(__fsub_rn(y.x, mean), r), ga.x), be.x);
        y.y = __fadd_rn(__fmul_rn(__fmul_rn(__fsub_rn(y.y, mean), r), ga.y), be.y);
        y.z = __fadd_rn(__fmul_rn(__fmul_rn(__fsub_rn(y.z, mean), r), ga.z), be.z);
        y.w = __fadd_rn(__fmul_rn(__fmul_rn(__fsub_rn(y.w, mean), r), ga.w), be.w);
        *px = y;
    }
    csync();
    return true;
}

// One GEMV phase of one sequence on CUDA cores: take the first weight stage, gather and stage the inputs,
// consume the producer's stages, store the outputs as tagged words. A pass of a warp takes RR rows (RR / 2 gate /
// up pairs for SwiGLU) spaced kW apart, so the CTA's warps walk the stages together and free them in order (no
// barrier per stage: at one sequence this beats the tensor-core phase below, 0.85 vs 0.92 ms per Qwen3-0.6B
// step). Returns false when the kernel must stop (a wait failed).
template <int FMT, int NM>
__device__ __forceinline__ bool gemv_run_cc(const DecodeParams& p, const GemvPh& g, uint32_t& st_base, uint32_t& seen,
                                         int warp, int lane) {
    constexpr int RR = kRows<NM>;
    int r0, r1;
    cta_rows(g.rows, p.grid, r0, r1);
    if (r0 >= r1) return true;
    const int n = r1 - r0, rps = stage_rows(p, g), nst = (n + rps - 1) / rps;
    const int cbytes = code_bytes(FMT, g.K), nseg = seg_count(FMT, g.K), xrow = nseg * Seg<FMT>::W;
    const int rpp = g.pair ? RR / 2 : RR;  // output rows per pass
    const bool rms = g.norm == kNormRms;
    constexpr float kF = FMT == kFP8 ? kFp8HwFactor : kFp4Factor;  // the dot products' decode factor
    RowWalk w{0, 0, int(st_base % uint32_t(p.nslot)), int((st_base / uint32_t(p.nslot)) & 1u)};
    w.advance(warp, rps, p.nslot);  // this warp's first row
    int released = 0;               // stages [0, released) of this phase that this warp has let go
    // A parity wait on a slot is only unambiguous while the slot is at most one phase ahead of the waiter, and a
    // warp need not have rows in every stage, so each warp observes the landing of every stage of the step in
    // order (`seen`: the next one), the ones it does not read included, and lets go of a stage only after
    // observing it. The landed ones cost one try_wait.
    auto observe = [&](uint32_t upto) -> bool {
        int ok = 1;
        for (; seen <= upto && ok; seen++) {
            const int slot = int(seen % uint32_t(p.nslot)), par = int((seen / uint32_t(p.nslot)) & 1u);
            if (lane == 0) ok = mbar_try_wait(&full_bar()[slot], par) || dwait(&full_bar()[slot], par, p.wait_ns);
            ok = __shfl_sync(0xffffffffu, ok, 0);
        }
        return ok != 0;
    };
    auto release_to = [&](int s) -> bool {
        if (s > released && !observe(st_base + uint32_t(s - 1))) return false;
        for (; released < s; released++)
            if (lane == 0) mbar_arrive(&empty_bar()[(st_base + uint32_t(released)) % uint32_t(p.nslot)]);
        return true;
    };
    unsigned long long best[NM];    // LM head: this warp's greedy argmax key per sequence
#pragma unroll
    for (int m = 0; m < NM; m++) best[m] = 0ull;
    const uint8_t* wr[RR];
    int nr = 0;
    RowWalk v = w;
    // Rows of the pass starting at i0: their stages waited for (one lane waits), their pointers in wr. False if
    // a wait gave up.
    auto setup = [&](int i0) -> bool {
        nr = 0;
        v = w;
#pragma unroll
        for (int r = 0; r < RR; r++) {
            if (r >= rpp) break;
            if (i0 + r * kW < n) {
                if (!observe(st_base + uint32_t(v.s))) return false;
                const uint8_t* b = ring_buf(p) + size_t(v.slot) * p.slot_bytes;
                wr[r] = b + int64_t(v.o) * g.rb;
                if (g.pair) wr[rpp + r] = b + int64_t(min(rps, n - v.s * rps) + v.o) * g.rb;
                nr = r + 1;
            } else {  // no row: repeat row 0 (never used) so every load of the pass is unconditional
                wr[r] = wr[0];
                if (g.pair) wr[rpp + r] = wr[rpp];
            }
            v.advance(kW, rps, p.nslot);
        }
        return true;
    };
    // The first pass's weights were streamed in during earlier phases: take them before the activations' wait.
    // A stage wait that gives up stops this warp's consumption; the failure reaches the other consumer threads
    // at the next reducing barrier (every consumer thread passes the same barriers), and they all leave.
    bool ok = warp < n ? setup(warp) : true;
    if (!stage_x<FMT, NM>(p, g, xs_buf(p), warp, lane, ok)) return false;
    float rstd[NM];
#pragma unroll
    for (int m = 0; m < NM; m++) rstd[m] = (rms && m < p.M) ? rms_rstd(p, m, g.K) : 1.0f;
    for (int i0 = warp; i0 < n; i0 += kW * rpp) {
        if (i0 != warp && !setup(i0)) {
            ok = false;
            break;
        }
        // SwiGLU: up row r sits at rpp + r (gate rows nr .. rpp - 1 are computed but unused)
        const int nrows = g.pair ? rpp + nr : nr;
        float acc[RR][NM];
        dot_rows<FMT, NM, RR>(wr, nrows, cbytes, nseg, xs_buf(p), xrow, p.M, lane, acc);
        // reductions of every row first (independent shuffle chains), then the lanes that own a row store it
        float red_[RR][NM];
#pragma unroll
        for (int r = 0; r < RR; r++)
#pragma unroll
            for (int m = 0; m < NM; m++) red_[r][m] = (r < nrows && m < p.M) ? warp_sum(acc[r][m]) * kF : 0.0f;
#pragma unroll
        for (int r = 0; r < RR; r++) {
            if (r >= rpp) break;
#pragma unroll
            for (int m = 0; m < NM; m++) {
                if (m >= p.M) break;
                if (r >= nr || lane != ((r * NM + m) & 31)) continue;
                const int row = r0 + i0 + r * kW;
                const float rs = rstd[m];
                float val;
                if (g.pair) {
                    const float gs = __fmul_rn(red_[r][m], rs);
                    const float us = __fmul_rn(red_[rpp + r < RR ? rpp + r : 0][m], rs);
                    val = __fdividef(gs, 1.0f + expf(-gs)) * us;  // cpu::siluMul (cpu_ops.cpp:526-533)
                } else {
                    val = rms ? __fmul_rn(red_[r][m], rs) : red_[r][m];
                    if (g.flags & kBias) val += g.bias[row];
                    if (g.flags & kGelu) val = gelu(val);
                    if (g.resid) {
                        float& xo = dsh().xown[m][row - r0];
                        val += xo;
                        xo = val;
                    }
                }
                if (g.head) {
                    p.logits[int64_t(m) * g.ys + row] = val;
                    best[m] = max(best[m], argmax_key(val, row));
                } else if (g.xout) {
                    g.xout[int64_t(m) * g.ys + row] = val;
                } else {
                    tw_put(g.y + int64_t(m) * g.ys + row, val, g.ytag);
                }
            }
        }
        __syncwarp();
        w = v;  // the first row of this warp's next pass
        if (!release_to(i0 + kW * rpp < n ? w.s : nst)) {
            ok = false;
            break;
        }
    }
    __syncwarp();
    if (ok) ok = release_to(nst);
    if (g.head) {  // one shared atomic per warp and sequence
#pragma unroll
        for (int m = 0; m < NM; m++) {
            if (m >= p.M) break;
            unsigned long long k = best[m];
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) k = max(k, __shfl_xor_sync(0xffffffffu, k, o));
            if (lane == 0 && k) atomicMax(&dsh().key[m], k);
        }
    }
    st_base += uint32_t(nst);
    // the next phase's staging overwrites the activations this phase's warps may still be reading
    return csync_and(ok);
}

// ---------------------------------------------------------------------------------------------- GEMV phases, 2..4 sequences
// The dot products run on the tensor cores (mma.sync m16n8k16, f16 x f16 -> fp32): 16 weight rows of a ring
// stage are the A operand, converted from their codes in registers (FP8: the hardware e4m3 -> f16 conversion;
// FP4: bit arithmetic; both exact in f16); the activations are the B operand, column 2m the f16 rounding hi of
// sequence m's row, column 2m + 1 the rounding lo of the remainder (about 22 bits together), each 32-element block
// divided by a power of two s_b that puts its largest magnitude in [2^14, 2^15) (so f16's range holds any row).
// Per block: acc += sw(row, block) * s_b * (D[hi] + D[lo]) in fp32, then the norm's rstd and the format's decode
// factor in the epilogue, as in the CUDA-core kernels.
//
// B layout: row n of the staging area = column n ([2M][K] halves), then the block scales [M][K / 32] floats. Within
// a block, lane t of an MMA reads its 8 values at halves 8t .. 8t + 7: FP8 in natural order (lane t holds code
// bytes 8t .. 8t + 7 of the block); FP4 as weights 4t .. 4t + 3 then 16 + 4t .. 16 + 4t + 3 (code bytes 4t .. 4t
// + 3 hold those as low / high nibbles).
template <int FMT>
__device__ __forceinline__ int bpos(int k) {  // half index within the row of activation k (k % 4 == 0)
    if (FMT == kFP8) return k;
    const int kk = k & 31;
    return (k & ~31) + (kk < 16 ? 2 * kk : 2 * (kk - 16) + 4);
}
__device__ __forceinline__ int b_bytes(int M, int K) { return 4 * M * K + M * (K / 32) * 4; }

// Writes 4 activations of sequence m at k (y = x / s_b is formed by the caller's block-scale exponent) as hi / lo.
template <int FMT>
__device__ __forceinline__ void put_hilo(__half* bx, int K, int m, int k, float4 y, float inv) {
    uint32_t h0, l0, h1, l1;
    split_hilo(y.x * inv, y.y * inv, h0, l0);
    split_hilo(y.z * inv, y.w * inv, h1, l1);
    const int o = bpos<FMT>(k);
    *reinterpret_cast<uint2*>(bx + int64_t(2 * m) * K + o) = make_uint2(h0, h1);
    *reinterpret_cast<uint2*>(bx + int64_t(2 * m + 1) * K + o) = make_uint2(l0, l1);
}

// The block's power-of-two scale from the 8 lanes (lanes 8j .. 8j + 7) that hold its 32 values: s (stored) and
// 1 / s (applied). Every lane of the warp calls it.
__device__ __forceinline__ void block_scale(float4 y, float& s, float& inv) {
    float v = fmaxf(fmaxf(fabsf(y.x), fabsf(y.y)), fmaxf(fabsf(y.z), fabsf(y.w)));
    v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, 1));
    v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, 2));
    v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, 4));
    const int F = int((__float_as_uint(v) >> 23) & 0xFF) - 127;  // v in [2^F, 2^(F+1))
    const int e = max(-126, min(127, F - 14)), ie = max(-126, min(127, -e));
    s = __uint_as_float(uint32_t(e + 127) << 23);
    inv = __uint_as_float(uint32_t(ie + 127) << 23);
}

// Stages the M input rows of a phase (tagged words) as the B operand: RMSNorm phases stage x * gamma and leave
// per-warp sums of squares in dsh().ss (the epilogue applies rstd); LayerNorm phases (GPT-2) gather x into an f32
// area first, then normalise with the row mean and variance (cpu_ops.cpp:483-500, sums in double). `ok` false:
// this thread's earlier wait failed. Returns false, for every consumer thread alike, when any wait failed or an
// input never arrived. A thread's float4 groups are base + tid + e * kNT; the 8 lanes of a block are consecutive.
template <int FMT, int NM>
__device__ bool stage_b(const DecodeParams& p, const GemvPh& g, int warp, int lane, bool ok) {
    const int tid = threadIdx.x, K = g.K, K4 = K / 4, nq = p.M * K4;
    const bool rms = g.norm == kNormRms, ln = g.norm == kNormLayer;
    __half* bx = reinterpret_cast<__half*>(xs_buf(p));
    float* bsc = reinterpret_cast<float*>(xs_buf(p)) + p.M * K;  // after the 2M half rows
    float* xr = bsc + p.M * (K / 32);                             // LayerNorm: raw rows [M][K]
    double ss[NM], s1[NM];
#pragma unroll
    for (int m = 0; m < NM; m++) ss[m] = s1[m] = 0.0;
    for (int base = 0; base < nq && ok; base += kGatherE * kNT) {
        int q[kGatherE];
        float4 gm[kGatherE];
#pragma unroll
        for (int e = 0; e < kGatherE; e++) {
            q[e] = base + tid + e * kNT;
            if (rms && q[e] < nq) gm[e] = __ldg(reinterpret_cast<const float4*>(g.gamma + 4 * (q[e] % K4)));
        }
        float4 v[kGatherE];
        ok = __all_sync(0xffffffffu, gather4<kGatherE>(g.x, q, nq, g.xtag, v, p.wait_ns));  // the block scales
        if (!ok) break;                                                                     // shuffle the warp
#pragma unroll
        for (int e = 0; e < kGatherE; e++) {
            const bool has = q[e] < nq;
            const int m = has ? q[e] / K4 : 0, k = has ? 4 * (q[e] - m * K4) : 0;
            float4 y = has ? v[e] : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
            const double sq = double(y.x) * y.x + double(y.y) * y.y + double(y.z) * y.z + double(y.w) * y.w;
            const double sm = double(y.x) + double(y.y) + double(y.z) + double(y.w);
#pragma unroll
            for (int mm = 0; mm < NM; mm++)
                if (has && mm == m) {
                    ss[mm] += sq;
                    s1[mm] += sm;
                }
            if (ln) {
                if (has) *reinterpret_cast<float4*>(xr + int64_t(m) * K + k) = y;
                continue;
            }
            if (rms) {
                y.x = __fmul_rn(y.x, gm[e].x);
                y.y = __fmul_rn(y.y, gm[e].y);
                y.z = __fmul_rn(y.z, gm[e].z);
                y.w = __fmul_rn(y.w, gm[e].w);
            }
            float sb, inv;
            block_scale(y, sb, inv);  // every lane (groups past nq hold zeros)
            if (has) {
                put_hilo<FMT>(bx, K, m, k, y, inv);
                if ((k & 31) == 0) bsc[m * (K / 32) + k / 32] = sb;
            }
        }
    }
#pragma unroll
    for (int m = 0; m < NM; m++) {
        if (m >= p.M) break;
        const double t2 = wsum_d(ss[m]);
        if (ln) {
            const double t1 = wsum_d(s1[m]);
            if (lane == 0) dsh().part[2 * (warp * NM + m)] = t1;
        }
        if (lane == 0) dsh().ss[warp][m] = t2;
    }
    if (!csync_and(ok)) return false;
    if (!ln) return true;
    // LayerNorm: the rows' mean and rstd from the per-warp sums, then the normalised values as the B operand
    float mean[NM], r[NM];
#pragma unroll
    for (int m = 0; m < NM; m++) {
        double a1 = 0.0, a2 = 0.0;
        if (m < p.M)
            for (int w = 0; w < kW; w++) {
                a1 += dsh().part[2 * (w * NM + m)];
                a2 += dsh().ss[w][m];
            }
        const double mu = a1 / K;
        mean[m] = float(mu);
        r[m] = m < p.M ? float(1.0 / sqrt(a2 / K - mu * mu + double(p.eps))) : 0.0f;
    }
    for (int base = 0; base < nq; base += kNT) {
        const int qq = base + tid;
        const bool has = qq < nq;
        const int m = has ? qq / K4 : 0, k = has ? 4 * (qq - m * K4) : 0;
        float4 y = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        if (has) {
            float mm = mean[0], rr = r[0];
#pragma unroll
            for (int q2 = 1; q2 < NM; q2++)
                if (q2 == m) {
                    mm = mean[q2];
                    rr = r[q2];
                }
            const float4 x = *reinterpret_cast<const float4*>(xr + int64_t(m) * K + k);
            const float4 ga = __ldg(reinterpret_cast<const float4*>(g.gamma + k));
            const float4 be = __ldg(reinterpret_cast<const float4*>(g.beta + k));
            y.x = __fadd_rn(__fmul_rn(__fmul_rn(__fsub_rn(x.x, mm), rr), ga.x), be.x);
            y.y = __fadd_rn(__fmul_rn(__fmul_rn(__fsub_rn(x.y, mm), rr), ga.y), be.y);
            y.z = __fadd_rn(__fmul_rn(__fmul_rn(__fsub_rn(x.z, mm), rr), ga.z), be.z);
            y.w = __fadd_rn(__fmul_rn(__fmul_rn(__fsub_rn(x.w, mm), rr), ga.w), be.w);
        }
        float sb, inv;
        block_scale(y, sb, inv);
        if (has) {
            put_hilo<FMT>(bx, K, m, k, y, inv);
            if ((k & 31) == 0) bsc[m * (K / 32) + k / 32] = sb;
        }
    }
    csync();
    return true;
}

// Lane (g, t)'s sums over spans [s0, s1) (64 weights: two blocks) of the 16 rows whose codes start at wg (row g)
// and wh (row g + 8) in a ring stage: c0 (row g), c1 (row g + 8), for sequence t (B columns 2t, 2t + 1). xb: this
// lane's B row (column g; nullptr past 2M), bs: sequence t's block scales.
template <int FMT>
__device__ __forceinline__ void tile_dot(const uint8_t* wg, const uint8_t* wh, int cbytes, int s0, int s1,
                                         const __half* xb, const float* bs, int t, float& c0, float& c1) {
#pragma unroll 2
    for (int sp = s0; sp < s1; sp++) {
        const __half2 swg = *reinterpret_cast<const __half2*>(wg + cbytes + 4 * sp);  // blocks 2sp, 2sp + 1
        const __half2 swh = *reinterpret_cast<const __half2*>(wh + cbytes + 4 * sp);
        const float2 fg = __half22float2(swg), fh = __half22float2(swh);
        const float2 sb = *reinterpret_cast<const float2*>(bs + 2 * sp);
#pragma unroll
        for (int k = 0; k < 2; k++) {
            const int blk = 2 * sp + k;
            uint4 xv = make_uint4(0u, 0u, 0u, 0u);
            if (xb) xv = *reinterpret_cast<const uint4*>(xb + 32 * blk + 8 * t);
            uint32_t ga[4], ha[4];  // (MMA j, k slots 2t, 2t + 1 | 2t + 8, 2t + 9) of rows g / g + 8
            if (FMT == kFP8) {
                const uint2 cg = *reinterpret_cast<const uint2*>(wg + 32 * blk + 8 * t);
                const uint2 ch = *reinterpret_cast<const uint2*>(wh + 32 * blk + 8 * t);
                __half2 a, b, c, d;
                e4m3x4_to_half2(cg.x, a, b);
                e4m3x4_to_half2(cg.y, c, d);
                ga[0] = h2u(a), ga[1] = h2u(b), ga[2] = h2u(c), ga[3] = h2u(d);
                e4m3x4_to_half2(ch.x, a, b);
                e4m3x4_to_half2(ch.y, c, d);
                ha[0] = h2u(a), ha[1] = h2u(b), ha[2] = h2u(c), ha[3] = h2u(d);
            } else {  // code bytes 4t .. 4t + 3: low nibbles = weights 4t .., high nibbles = weights 16 + 4t ..
                const uint32_t wdg = *reinterpret_cast<const uint32_t*>(wg + 16 * blk + 4 * t);
                const uint32_t wdh = *reinterpret_cast<const uint32_t*>(wh + 16 * blk + 4 * t);
                auto unpack = [](uint32_t wd, uint32_t (&o)[4]) {
                    const __half2 e0 = fp4x2_to_half2(wd & 0x000F000Fu), o0 = fp4x2_to_half2((wd >> 8) & 0x000F000Fu);
                    const __half2 e1 = fp4x2_to_half2((wd >> 4) & 0x000F000Fu);
                    const __half2 o1 = fp4x2_to_half2((wd >> 12) & 0x000F000Fu);
                    o[0] = h2u(__halves2half2(__low2half(e0), __low2half(o0)));    // weights 4t, 4t + 1
                    o[1] = h2u(__halves2half2(__high2half(e0), __high2half(o0)));  // 4t + 2, 4t + 3
                    o[2] = h2u(__halves2half2(__low2half(e1), __low2half(o1)));    // 16 + 4t, 16 + 4t + 1
                    o[3] = h2u(__halves2half2(__high2half(e1), __high2half(o1)));  // 16 + 4t + 2, + 3
                };
                unpack(wdg, ga);
                unpack(wdh, ha);
            }
            float d[4];
            const uint32_t a0[4] = {ga[0], ha[0], ga[1], ha[1]}, a1[4] = {ga[2], ha[2], ga[3], ha[3]};
            mma16816_z(d, a0, xv.x, xv.y);
            mma16816(d, a1, xv.z, xv.w);
            const float sbk = k ? sb.y : sb.x;
            c0 = fmaf((k ? fg.y : fg.x) * sbk, d[0] + d[1], c0);
            c1 = fmaf((k ? fh.y : fh.x) * sbk, d[2] + d[3], c1);
        }
    }
}

// One GEMV phase on this CTA's rows: gather and stage the inputs (the B operand), then stage by stage of the
// producer's ring: every warp observes the stage, the stage's T tiles of 16 rows are split over the 12 warps
// along K (Q = 12 / T warps per tile), the partial sums meet in shared memory (buffers alternate by stage) and,
// after one barrier, one thread per (row, sequence) adds them in K order and stores the output as a tagged word.
// Returns false when the kernel must stop (a wait failed).
template <int FMT, int NM>
__device__ __forceinline__ bool gemv_run_tc(const DecodeParams& p, const GemvPh& g, uint32_t& st_base, uint32_t& seen,
                                            uint32_t& red_par, int warp, int lane) {
    __shared__ float s_red[2][kW][2][NM][16];  // [stage parity][warp][gate | up][sequence][tile row]
    int r0, r1;
    cta_rows(g.rows, p.grid, r0, r1);
    if (r0 >= r1) return true;
    const int n = r1 - r0, rps = stage_rows(p, g), nst = (n + rps - 1) / rps;
    const int tid = threadIdx.x, gq = lane >> 2, t = lane & 3;
    const int cbytes = code_bytes(FMT, g.K), nsp = g.K / 64;
    const bool rms = g.norm == kNormRms;
    constexpr float kF = FMT == kFP8 ? kFp8HwFactor : kFp4Factor;  // the dot products' decode factor
    // Every warp observes the landing of every stage of the step in order (`seen`: the next one) before it lets
    // go of it: an mbarrier parity wait is only unambiguous while the slot is at most one phase ahead.
    auto observe = [&](uint32_t upto) -> bool {
        int ok = 1;
        for (; seen <= upto && ok; seen++) {
            const int slot = int(seen % uint32_t(p.nslot)), par = int((seen / uint32_t(p.nslot)) & 1u);
            if (lane == 0) ok = mbar_try_wait(&full_bar()[slot], par) || dwait(&full_bar()[slot], par, p.wait_ns);
            ok = __shfl_sync(0xffffffffu, ok, 0);
        }
        return ok != 0;
    };
    // The first stage's weights were streamed in during earlier phases: take them before the activations' wait.
    // A stage wait that gives up stops this warp's consumption; the failure reaches the other consumer threads at
    // the next reducing barrier (every consumer thread passes the same barriers), and they all leave.
    bool ok = observe(st_base);
    if (!stage_b<FMT, NM>(p, g, warp, lane, ok)) return false;
    float rstd[NM];
#pragma unroll
    for (int m = 0; m < NM; m++) rstd[m] = (rms && m < p.M) ? rms_rstd(p, m, g.K) : 1.0f;
    const __half* bx = reinterpret_cast<const __half*>(xs_buf(p));
    const float* bsc = reinterpret_cast<const float*>(xs_buf(p)) + p.M * g.K;
    const __half* xb = gq < 2 * p.M ? bx + int64_t(gq) * g.K : nullptr;
    const float* bs = bsc + min(t, p.M - 1) * (g.K / 32);
    unsigned long long best[NM];  // LM head: this thread's greedy argmax key per sequence
#pragma unroll
    for (int m = 0; m < NM; m++) best[m] = 0ull;
    for (int s = 0; s < nst; s++) {
        // a wait that gives up skips this warp's work but not the barrier below, which every consumer thread
        // reaches once per stage and which then returns false to all of them
        if (ok && !observe(st_base + uint32_t(s))) ok = false;
        const int rows_s = min(rps, n - s * rps), T = (rows_s + 15) / 16, Q = kW / T;
        const int tile = warp / Q, ks = warp % Q;
        const uint8_t* base = ring_buf(p) + size_t((st_base + uint32_t(s)) % uint32_t(p.nslot)) * p.slot_bytes;
        float c[2][2] = {{0.0f, 0.0f}, {0.0f, 0.0f}};
        if (ok && tile < T) {
            const int rg = min(16 * tile + gq, rows_s - 1), rh = min(16 * tile + gq + 8, rows_s - 1);
            const int s0 = ks * nsp / Q, s1 = (ks + 1) * nsp / Q;
#pragma unroll
            for (int u = 0; u < 2; u++) {
                if (u == 1 && !g.pair) break;
                const uint8_t* hb = base + int64_t(u ? rows_s : 0) * g.rb;  // SwiGLU: the up rows follow
                tile_dot<FMT>(hb + int64_t(rg) * g.rb, hb + int64_t(rh) * g.rb, cbytes, s0, s1, xb, bs, t, c[u][0],
                              c[u][1]);
            }
        }
        if (t < p.M && t < NM) {
#pragma unroll
            for (int u = 0; u < 2; u++) {
                s_red[red_par][warp][u][t][gq] = c[u][0];
                s_red[red_par][warp][u][t][gq + 8] = c[u][1];
            }
        }
        __syncwarp();
        if (ok && lane == 0) mbar_arrive(&empty_bar()[(st_base + uint32_t(s)) % uint32_t(p.nslot)]);
        // every warp's partial sums of this stage are in; the other buffer is free (its readers passed this)
        if (!csync_and(ok)) return false;
        for (int i = tid; i < rows_s * p.M; i += kNT) {
            const int m = i % p.M, q = i / p.M, tq = q >> 4, a = q & 15;
            float red_[2];
#pragma unroll
            for (int u = 0; u < 2; u++) {
                float acc = 0.0f;
                for (int k = 0; k < Q; k++) acc += s_red[red_par][tq * Q + k][u][m][a];
                red_[u] = acc * kF;
            }
            const int row = r0 + s * rps + q;
            const float rs = rstd[0];
            float rsm = rs;
#pragma unroll
            for (int mm = 1; mm < NM; mm++)
                if (mm == m) rsm = rstd[mm];
            float val;
            if (g.pair) {
                const float gs = __fmul_rn(red_[0], rsm), us = __fmul_rn(red_[1], rsm);
                val = __fdividef(gs, 1.0f + expf(-gs)) * us;  // cpu::siluMul (cpu_ops.cpp:526-533)
            } else {
                val = rms ? __fmul_rn(red_[0], rsm) : red_[0];
                if (g.flags & kBias) val += g.bias[row];
                if (g.flags & kGelu) val = gelu(val);
                if (g.resid) {
                    float& xo = dsh().xown[m][row - r0];
                    val += xo;
                    xo = val;
                }
            }
            if (g.head) {
                p.logits[int64_t(m) * g.ys + row] = val;
                const unsigned long long key = argmax_key(val, row);
#pragma unroll
                for (int mm = 0; mm < NM; mm++)
                    if (mm == m) best[mm] = max(best[mm], key);
            } else if (g.xout) {
                g.xout[int64_t(m) * g.ys + row] = val;
            } else {
                tw_put(g.y + int64_t(m) * g.ys + row, val, g.ytag);
            }
        }
        red_par ^= 1u;
    }
    if (g.head) {  // one shared atomic per thread and sequence; the barrier orders them before the CTA's read
#pragma unroll
        for (int m = 0; m < NM; m++)
            if (m < p.M && best[m]) atomicMax(&dsh().key[m], best[m]);
        csync();
    }
    st_base += uint32_t(nst);
    return ok;
}

template <int FMT, int NM>
__device__ __forceinline__ bool gemv_run(const DecodeParams& p, const GemvPh& g, uint32_t& st_base, uint32_t& seen,
                                         uint32_t& red_par, int warp, int lane) {
    if constexpr (NM == 1)
        return gemv_run_cc<FMT, 1>(p, g, st_base, seen, warp, lane);
    else
        return gemv_run_tc<FMT, NM>(p, g, st_base, seen, red_par, warp, lane);
}

// ---------------------------------------------------------------------------------------------- attention
// DL consecutive f16 values of a staged key / value row.
template <int DL>
__device__ __forceinline__ void load_half_row(const uint16_t* src, float (&out)[DL]) {
    if constexpr (DL == 4) {
        const uint2 w = *reinterpret_cast<const uint2*>(src);
        const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&w.x));
        const float2 b = __half22float2(*reinterpret_cast<const __half2*>(&w.y));
        out[0] = a.x;
        out[1] = a.y;
        out[2] = b.x;
        out[3] = b.y;
    } else {
        const unsigned w = *reinterpret_cast<const unsigned*>(src);
        const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&w));
        out[0] = a.x;
        out[1] = a.y;
    }
}

struct AttnItem {
    int m, g, j, ns, pos, slot, k0, n;
};

// Item it of this step: sequence m, KV head g, split j of ns, keys [k0, k0 + n).
__device__ __forceinline__ AttnItem attn_item(const DecodeParams& p, const int (&Sm)[kDecodeMaxSeqs],
                                              const int (&Pm)[kDecodeMaxSeqs], int it) {
    AttnItem a;
    int rem = it, m = 0, ns = Sm[0], pos = Pm[0];
#pragma unroll
    for (int mm = 0; mm < kDecodeMaxSeqs - 1; mm++) {  // unrolled walk (no dynamic indexing of the arrays)
        if (rem >= p.KV * ns) {
            rem -= p.KV * ns;
            m = mm + 1;
            ns = Sm[mm + 1];
            pos = Pm[mm + 1];
        }
    }
    a.m = m;
    a.ns = ns;
    a.g = rem / ns;
    a.j = rem - a.g * ns;
    a.pos = pos;
    a.slot = p.slots[m];
    a.k0 = a.j * dsh().span;
    a.n = min(a.pos + 1, a.k0 + dsh().span) - a.k0;
    return a;
}

// Attention items of the step: Sm[m] splits of sequence m, Pm[m] its (clamped) position; returns the count.
__device__ __forceinline__ int attn_items(const DecodeParams& p, int (&Sm)[kDecodeMaxSeqs], int (&Pm)[kDecodeMaxSeqs]) {
    int total = 0;
#pragma unroll
    for (int m = 0; m < kDecodeMaxSeqs; m++) {
        Sm[m] = 1;
        Pm[m] = 0;
        if (m >= p.M) continue;
        const int pos = max(0, min(p.pos[m], p.context - 1));  // out of range: reported at kernel start
        Pm[m] = pos;
        Sm[m] = (pos + dsh().span) / dsh().span;
        total += p.KV * Sm[m];
    }
    return total;
}

// One thread: copies the item's cached keys and values (positions below pos; the newest comes from this step)
// into shared memory with two bulk copies (a head's positions are contiguous in the cache), completing on
// dsh().attn_bar. The cache rows are from earlier steps, so this is issued long before the item runs.
__device__ __forceinline__ void attn_issue(const DecodeParams& p, int l, const AttnItem& a) {
    const DecodeLayer& Ly = layer_tab()[l];
    const int nold = min(a.n, a.pos - a.k0);  // rows that are in the cache already
    const uint32_t bytes = uint32_t(nold) * uint32_t(p.hd) * 2u;
    const int64_t base = int64_t(a.slot) * p.kv_slot + int64_t(a.g) * p.kv_head + int64_t(a.k0) * p.hd;
    mbar_arrive_expect_tx(&dsh().attn_bar, 2u * bytes);
    if (bytes) {
        bulk_g2s(kv_buf(p), Ly.kc + base, bytes, &dsh().attn_bar);
        bulk_g2s(kv_buf(p) + dsh().span * p.hd, Ly.vc + base, bytes, &dsh().attn_bar);
    }
}

// Items (sequence m, KV head g, split j) over keys [j * span, min(L, (j + 1) * span)), L = pos + 1. Each item
// rebuilds the group's query heads (QK-norm + RoPE, qwen3_model.cpp:249-262) and the new key / value
// (f16-rounded, as the cache holds them); split 0 stores them at pos (cpu::storeKv). The older keys and values
// were copied to shared memory when the layer started. Lane l owns dims [l * DL, l * DL + DL) of a key / value
// row for scores (cpu_ops.cpp:558) and P.V. A sequence with one split writes its heads' output; with several,
// each item writes its partial softmax state (max, sum, unnormalised P.V) for merge_run.
template <int DL, int QW>
__device__ __noinline__ bool attn_run(const DecodeParams& p, int l, int& issued, int warp, int lane) {
    const int Gq = p.H / p.KV, hd = p.hd, span = dsh().span;
    int Sm[kDecodeMaxSeqs], Pm[kDecodeMaxSeqs];
    const int total = attn_items(p, Sm, Pm);
    if (int(blockIdx.x) >= total) return true;
    const DecodeLayer& Ly = layer_tab()[l];
    float* sq = xs_buf(p);            // [Gq][hd]
    float* snk = sq + Gq * hd;        // [hd]
    float* snv = snk + hd;            // [hd]
    float* sc = snv + hd;             // [Gq][span]
    float* red = sc + Gq * span;      // [kW][Gq][hd]
    float* sst = red + kW * Gq * hd;  // [Gq](max, sum)
    const uint16_t* kbuf = kv_buf(p);  // [span][hd]
    const uint16_t* vbuf = kv_buf(p) + span * hd;
    // stall_test: the queries wait for a tag no phase writes (timeout path test)
    const unsigned qtag = tag_of(l, kXQkv) ^ (p.stall_test ? 0x80000000u : 0u);

    AttnItem a = attn_item(p, Sm, Pm, blockIdx.x);
    float cs_c[DL / 2], cs_s[DL / 2], wn[DL];
    auto load_rot = [&](const AttnItem& it) {
        if (QW && warp <= Gq) {
            const float* cs = p.rope + int64_t(it.pos) * hd;
#pragma unroll
            for (int i = 0; i < DL / 2; i++) {
                cs_c[i] = cs[2 * (lane + 32 * i)];
                cs_s[i] = cs[2 * (lane + 32 * i) + 1];
            }
#pragma unroll
            for (int i = 0; i < DL; i++) wn[i] = Ly.qknorm[(warp == Gq ? hd : 0) + lane + 32 * i];
        }
    };
    load_rot(a);

    for (int it = blockIdx.x; it < total; it += p.grid) {
        if (it != int(blockIdx.x)) {  // later items of this CTA (long contexts): requested after the previous
            a = attn_item(p, Sm, Pm, it);
            load_rot(a);
        }
        const int L = a.pos + 1, n = a.n, g = a.g, m = a.m;
        const bool has_new = a.k0 + n == L;
        bool ok = true;
        // 1. query heads of the group, the new key and value: one warp per head, straight from the tagged words
        if (warp < Gq + 2) {
            const int which = warp < Gq ? 0 : warp == Gq ? 1 : 2;
            const int col = which == 0 ? (g * Gq + warp) * hd : which == 1 ? (p.H + g) * hd : (p.H + p.KV + g) * hd;
            float e[DL];
            ok = gather_lane<DL>(p.qkv_tw + int64_t(m) * p.QW + col + lane, 32, qtag, e, p.wait_ns);
            if (ok) {
                if (QW && which != 2) {
                    double ss = 0.0;
#pragma unroll
                    for (int i = 0; i < DL; i++) ss += double(e[i]) * e[i];
                    ss = wsum_d(ss);
                    const float sn = inv_rms(ss, 1.0 / hd, p.eps);
#pragma unroll
                    for (int i = 0; i < DL; i++) e[i] = __fmul_rn(__fmul_rn(e[i], sn), wn[i]);
#pragma unroll
                    for (int i = 0; i < DL / 2; i++) {  // NeoX pairs (d, d + hd / 2), cpu::rope
                        const float x0 = e[i], x1 = e[i + DL / 2];
                        e[i] = __fsub_rn(__fmul_rn(x0, cs_c[i]), __fmul_rn(x1, cs_s[i]));
                        e[i + DL / 2] = __fadd_rn(__fmul_rn(x0, cs_s[i]), __fmul_rn(x1, cs_c[i]));
                    }
                }
                if (which == 0) {
#pragma unroll
                    for (int i = 0; i < DL; i++) sq[warp * hd + lane + 32 * i] = e[i];
                } else {
                    uint16_t* cache = (which == 1 ? Ly.kc : Ly.vc) + int64_t(a.slot) * p.kv_slot +
                                      int64_t(g) * p.kv_head + int64_t(a.pos) * hd;
                    float* dst = which == 1 ? snk : snv;
#pragma unroll
                    for (int i = 0; i < DL; i++) {
                        const __half hv = __float2half_rn(e[i]);
                        dst[lane + 32 * i] = __half2float(hv);
                        if (a.j == 0 && p.pos[m] == a.pos) cache[lane + 32 * i] = __half_as_ushort(hv);
                    }
                }
            }
        }
        if (threadIdx.x == 0 && !dwait(&dsh().attn_bar, uint32_t(issued - 1) & 1u, p.wait_ns)) ok = false;
        if (!csync_and(ok)) return false;  // the inputs or the keys never arrived: leave together
        // 2. scores, four keys x four query heads (heads past Gq are zero) per warp pass: the 16 lane partial
        // sums are reduced together by a transposed butterfly (halves exchange 8 values, then 4, 2, 1, then one
        // xor step), 16 shuffles instead of 5 per dot product
        static_assert(kMaxGq == 4, "16 values per pass");
        for (int grp = warp; 4 * grp < n; grp += kW) {
            float v[16];
#pragma unroll
            for (int j = 0; j < 4; j++) {
                const int t = 4 * grp + j;
                float kv[DL];
                if (t < n && has_new && a.k0 + t == L - 1) {
#pragma unroll
                    for (int i = 0; i < DL; i++) kv[i] = snk[lane * DL + i];
                } else if (t < n) {
                    load_half_row<DL>(kbuf + t * hd + lane * DL, kv);
                } else {
#pragma unroll
                    for (int i = 0; i < DL; i++) kv[i] = 0.0f;
                }
#pragma unroll
                for (int gq = 0; gq < kMaxGq; gq++) {
                    float d = 0.0f;
                    if (gq < Gq)
#pragma unroll
                        for (int i = 0; i < DL; i++) d = fmaf(sq[gq * hd + lane * DL + i], kv[i], d);
                    v[4 * j + gq] = d;
                }
            }
#pragma unroll
            for (int w = 8; w >= 1; w >>= 1) {  // exchange halves: lane bit (16 >> k) picks which half it keeps
                const bool up = lane & (2 * w);
#pragma unroll
                for (int i = 0; i < w; i++) {
                    const float keep = up ? v[i + w] : v[i], send = up ? v[i] : v[i + w];
                    v[i] = keep + __shfl_xor_sync(0xffffffffu, send, 2 * w);
                }
            }
            v[0] += __shfl_xor_sync(0xffffffffu, v[0], 1);
            // lane L holds value ((L >> 4) & 1) 8 + ((L >> 3) & 1) 4 + ((L >> 2) & 1) 2 + ((L >> 1) & 1)
            const int idx = ((lane >> 4) & 1) * 8 + ((lane >> 3) & 1) * 4 + ((lane >> 2) & 1) * 2 + ((lane >> 1) & 1);
            const int t = 4 * grp + (idx >> 2), gq = idx & 3;
            if (!(lane & 1) && gq < Gq && t < n) sc[gq * span + t] = v[0] * p.scale;
        }
        csync();
        // 3. softmax of each query head over the item's keys
        if (warp < Gq) {
            float mx = -INFINITY;
            for (int t = lane; t < n; t += 32) mx = fmaxf(mx, sc[warp * span + t]);
            mx = warp_max(mx);
            float sum = 0.0f;
            for (int t = lane; t < n; t += 32) {
                const float e = expf(sc[warp * span + t] - mx);
                sc[warp * span + t] = e;
                sum += e;
            }
            sum = warp_sum(sum);
            if (lane == 0) {
                sst[2 * warp] = mx;
                sst[2 * warp + 1] = sum;
            }
        }
        csync();
        // 4. P.V
        float acc[kMaxGq][DL];
#pragma unroll
        for (int gq = 0; gq < kMaxGq; gq++)
#pragma unroll
            for (int i = 0; i < DL; i++) acc[gq][i] = 0.0f;
        for (int t = warp; t < n; t += kW) {
            float vv[DL];
            if (has_new && a.k0 + t == L - 1) {
#pragma unroll
                for (int i = 0; i < DL; i++) vv[i] = snv[lane * DL + i];
            } else {
                load_half_row<DL>(vbuf + t * hd + lane * DL, vv);
            }
#pragma unroll
            for (int gq = 0; gq < kMaxGq; gq++) {
                if (gq >= Gq) break;
                const float pr = sc[gq * span + t];
#pragma unroll
                for (int i = 0; i < DL; i++) acc[gq][i] = fmaf(pr, vv[i], acc[gq][i]);
            }
        }
#pragma unroll
        for (int gq = 0; gq < kMaxGq; gq++) {
            if (gq >= Gq) break;
#pragma unroll
            for (int i = 0; i < DL; i++) red[(warp * Gq + gq) * hd + lane * DL + i] = acc[gq][i];
        }
        csync();
        if (it + p.grid < total) {  // the staged keys / values are consumed: request the next item's
            if (threadIdx.x == 0) attn_issue(p, l, attn_item(p, Sm, Pm, it + p.grid));
            issued++;
        }
        // 5. merge the warps; one split: the heads' output, else this split's partial state
        const int outs = Gq * hd;
        for (int o = threadIdx.x; o < outs; o += kNT) {
            float sacc = 0.0f;
#pragma unroll
            for (int w = 0; w < kW; w++) sacc += red[w * outs + o];
            const int gq = o / hd, d = o - gq * hd;
            if (a.ns == 1) {
                tw_put(p.att_tw + int64_t(m) * p.H * hd + int64_t(g) * outs + o, __fdividef(sacc, sst[2 * gq + 1]),
                       tag_of(l, kXAtt));
            } else {
                uint64_t* pr = p.part_tw + (((int64_t(m) * p.KV + g) * p.max_splits + a.j) * Gq + gq) * (hd + 2);
                tw_put(pr + 2 + d, sacc, tag_of(l, kXPart));
                if (d == 0) {
                    tw_put(pr, sst[2 * gq], tag_of(l, kXPart));
                    tw_put(pr + 1, sst[2 * gq + 1], tag_of(l, kXPart));
                }
            }
        }
        csync();  // the scores and partial buffers are reused by the next item
    }
    return true;
}

// Split-KV merge: one warp per (sequence, KV head, query head, block of 32 dims) of a sequence with several
// splits, on warps of CTAs that hold no attention item when there are enough of them; lane l owns dim 32 b + l.
// The splits are merged in order with the softmax rescaling of their states (max m_s, sum l_s, unnormalised
// P.V a_s): out = sum_s exp(m_s - M) a_s / sum_s exp(m_s - M) l_s, M = max_s m_s (cpu_ops.cpp:556-572 over all
// keys). A merge that cannot finish (timeout or abort) is skipped: the next phase's inputs then never arrive and
// every CTA leaves through its own failed wait.
__device__ __noinline__ void merge_run(const DecodeParams& p, int l, int warp, int lane) {
    const int Gq = p.H / p.KV, hd = p.hd, nb = hd / 32;
    int Sm[kDecodeMaxSeqs], Pm[kDecodeMaxSeqs];
    const int total = attn_items(p, Sm, Pm);
    const int per_seq = p.KV * Gq * nb;
    int units = 0;
#pragma unroll
    for (int m = 0; m < kDecodeMaxSeqs; m++)
        if (m < p.M && Sm[m] > 1) units += per_seq;
    if (!units) return;
    // CTAs without an attention item first (the last ones), then all CTAs; unit u on warp u / ctas
    const int idle = max(0, p.grid - total);
    const int ctas = idle * kW >= units ? idle : p.grid;
    const int first = idle * kW >= units ? total : 0;
    const int cta = int(blockIdx.x) - first;
    if (cta < 0) return;
    const unsigned ptag = tag_of(l, kXPart), atag = tag_of(l, kXAtt);
    for (int u = cta + warp * ctas; u < units; u += kW * ctas) {
        // unit u -> (m, g, gq, b) over the sequences that have several splits
        int rem = u, m = 0;
#pragma unroll
        for (int mm = 0; mm < kDecodeMaxSeqs; mm++) {
            const int c = (mm < p.M && Sm[mm] > 1) ? per_seq : 0;
            if (m == mm && rem >= c) {
                rem -= c;
                m = mm + 1;
            }
        }
        int ns = Sm[0];
#pragma unroll
        for (int mm = 1; mm < kDecodeMaxSeqs; mm++)
            if (m == mm) ns = Sm[mm];
        const int gh = rem / nb, b = rem - gh * nb, g = gh / Gq, gq = gh - g * Gq;
        const uint64_t* base = p.part_tw + ((int64_t(m) * p.KV + g) * p.max_splits * Gq + gq) * (hd + 2);
        const int64_t sstride = int64_t(Gq) * (hd + 2);
        const int d = 32 * b + lane;
        float M = -INFINITY, den = 0.0f, num = 0.0f;
        bool ok = true;
        for (int s0 = 0; s0 < ns && ok; s0 += kMergeS) {
            // kMergeS splits at a time, every load in flight at once: lane j < kMergeS also holds the (max, sum)
            // of split s0 + j
            const int cnt = min(kMergeS, ns - s0);
            const bool have = lane < cnt;
            const int64_t so = int64_t(s0 + (have ? lane : 0)) * sstride;
            uint64_t w[kMergeS], wm = tw_ld(base + so), wl = tw_ld(base + so + 1);
#pragma unroll
            for (int j = 0; j < kMergeS; j++) w[j] = j < cnt ? tw_ld(base + int64_t(s0 + j) * sstride + 2 + d) : 0ull;
            Poll pl;
            for (;;) {
                unsigned miss = 0;
#pragma unroll
                for (int j = 0; j < kMergeS; j++)
                    if (j < cnt && !tw_ok(w[j], ptag)) miss |= 1u << j;
                const bool stm = have && !(tw_ok(wm, ptag) && tw_ok(wl, ptag));
                if (!__any_sync(0xffffffffu, miss || stm)) break;
                if (!pl.keep_going(p.wait_ns)) {
                    ok = false;
                    break;
                }
                if (stm) {
                    wm = tw_ld(base + so);
                    wl = tw_ld(base + so + 1);
                }
#pragma unroll
                for (int j = 0; j < kMergeS; j++)
                    if (miss >> j & 1u) w[j] = tw_ld(base + int64_t(s0 + j) * sstride + 2 + d);
            }
            if (!ok) break;
            const float ms = tw_val(wm), ls = tw_val(wl);
            // in split order: the running max, then the rescaled sums
            float wv[kMergeS];
#pragma unroll
            for (int j = 0; j < kMergeS; j++) wv[j] = tw_val(w[j]);
#pragma unroll 1
            for (int j = 0; j < cnt; j++) {
                const float mj = __shfl_sync(0xffffffffu, ms, j), lj = __shfl_sync(0xffffffffu, ls, j);
                const float Mn = fmaxf(M, mj);
                const float a = expf(M - Mn), e = expf(mj - Mn);  // exp(-inf) = 0 for the first split
                den = den * a + lj * e;
                num = num * a + wv[j] * e;
                M = Mn;
            }
        }
        if (!ok) return;
        tw_put(p.att_tw + int64_t(m) * p.H * hd + int64_t(g * Gq + gq) * hd + d, __fdividef(num, den), atag);
    }
}

// ---------------------------------------------------------------------------------------------- the kernel
template <int FMT, int NM, int QW, int DL>
__global__ void __launch_bounds__(kThr, 1) decode_kernel(const __grid_constant__ DecodeParams p) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (threadIdx.x == 0) {
        for (int s = 0; s < p.nslot; s++) {
            mbar_init(&full_bar()[s], 1);
            mbar_init(&empty_bar()[s], kW);
        }
        mbar_init(&dsh().attn_bar, 1);
        fence_barrier_init();
        dsh().epoch = *reinterpret_cast<volatile const unsigned*>(p.epoch);
        // keys per attention split: the smallest multiple of 32 (up to p.span) whose items fit the grid, one item
        // per CTA (more, smaller items finish sooner: the phase waits for its slowest item)
        int sp = 32;
        for (;; sp += 32) {
            int items = 0;
            for (int m = 0; m < p.M; m++) items += p.KV * ((max(0, min(p.pos[m], p.context - 1)) + sp) / sp);
            if (items <= p.grid || sp >= p.span) break;
        }
        dsh().span = sp;
    }
    // the per-layer pointers, once, into shared memory (indexing the parameter block by layer would go through
    // the constant cache on every phase)
    {
        const int words = p.layers * int(sizeof(DecodeLayer) / 8);
        const uint64_t* src = reinterpret_cast<const uint64_t*>(p.layer);
        uint64_t* dst = reinterpret_cast<uint64_t*>(dsm + kDHdr);
        for (int i = threadIdx.x; i < words; i += blockDim.x) dst[i] = src[i];
    }
    if (threadIdx.x < kDecodeMaxSeqs) dsh().key[threadIdx.x] = 0ull;
    __syncthreads();
    if (warp == kW) {
        producer<QW>(p, full_bar(), empty_bar(), ring_buf(p), lane);
        return;
    }

    for (int m = threadIdx.x; m < p.M; m += kNT)
        if (p.pos[m] < 0 || p.pos[m] >= p.context) set_device_error(kErrBadIndex);
    // The residual stream starts as the token embeddings (+ positions): each CTA computes the rows it owns (the
    // o_proj / down rows), keeps them and publishes them for layer 0.
    {
        int n0, n1;
        cta_rows(p.C, p.grid, n0, n1);
        const int w = n1 - n0;
        for (int i = threadIdx.x; i < p.M * w; i += kNT) {
            const int m = i / w, c = n0 + (i - m * w);
            float v = dequant_one(p.fmt, p.embed + int64_t(token_of(p, m)) * p.rb_c, p.C, c);
            if (p.wpe) v += p.wpe[int64_t(p.pos[m]) * p.C + c];
            dsh().xown[m][c - n0] = v;
            tw_put(p.x_tw + int64_t(m) * p.C + c, v, tag_of(0, kXIn));
        }
    }
    // Phases in order: per layer qkv, attention, split merge, o_proj, up, down; then the LM head.
    uint32_t st = 0, seen = 0;  // weight stages of the step: consumed by the phases so far, landings observed
    uint32_t red_par = 0;       // the GEMV phases' partial-sum buffer in use (alternates by stage)
    int issued = 0;  // attention copies requested so far (the parity of dsh().attn_bar)
    int Sm[kDecodeMaxSeqs], Pm[kDecodeMaxSeqs];
    const bool attn_cta = int(blockIdx.x) < attn_items(p, Sm, Pm);
    // Leaving early (a wait gave up): no attention copy of ours may still be landing in shared memory.
    auto drain = [&]() {
        if (threadIdx.x == 0 && issued > 0) {
            const uint64_t t0 = gtimer();
            while (!mbar_try_wait(&dsh().attn_bar, uint32_t(issued - 1) & 1u) && gtimer() - t0 < p.wait_ns) {
            }
        }
    };
    const int last = p.x_final ? p.layers - 1 : p.layers;  // the LM head runs apart when x_final is set
    for (int l = 0; l <= last; l++) {
        for (int k = 0; k < (l == p.layers ? 1 : 5); k++) {
            if (k == kQkv && l < p.layers && attn_cta) {  // this layer's first attention item: keys / values now
                if (threadIdx.x == 0) attn_issue(p, l, attn_item(p, Sm, Pm, blockIdx.x));
                issued++;
            }
            if (k == kAttn) {
                const bool ok = attn_run<DL, QW>(p, l, issued, warp, lane);
                if (!ok) {
                    drain();
                    return;
                }
                merge_run(p, l, warp, lane);
                continue;
            }
            const int kind = l == p.layers ? int(kHead) : k;
            if (!gemv_run<FMT, NM>(p, gemv_ph<QW>(p, l, kind), st, seen, red_par, warp, lane)) {
                drain();
                return;
            }
        }
    }
    if (threadIdx.x < p.M && dsh().key[threadIdx.x]) atomicMax(p.keys + threadIdx.x, dsh().key[threadIdx.x]);
    // (No early trigger of the dependent LM-head launch: releasing it here measured 60 us slower per step.)
    __threadfence();
    csync();
    if (threadIdx.x == 0) dsh().last = atomicAdd(p.sync, 1u) == unsigned(p.grid - 1) ? 1 : 0;
    csync();
    if (!dsh().last) return;
    // Last CTA: every other CTA has passed its last wait. Greedy token per sequence (argmax_finalize_kernel
    // semantics), then reset the step counter and advance the epoch for the next launch.
    __threadfence();
    if (threadIdx.x < p.M && !p.x_final) {  // (with x_final the separate LM head and its finalize do this)
        const int m = threadIdx.x;
        const unsigned long long key = atomicExch(p.keys + m, 0ull);
        int idx = int(0xFFFFFFFFu - unsigned(key & 0xFFFFFFFFull));
        if (idx < 0 || idx >= p.V) {  // no logit was reduced (cannot happen unless the head phase was skipped)
            set_device_error(kErrBadIndex);
            idx = 0;
        }
        p.argmax[m] = idx;
        if (p.advance) {
            p.tokens[m] = idx;
            if (p.pos[m] + 1 < p.context) p.pos[m] += 1;
            else set_device_error(kErrBadIndex);
        }
    }
    if (threadIdx.x == 0) {
        *p.sync = 0u;
        *p.epoch = dsh().epoch + decode_epoch_stride(p.layers);
    }
}

using DecodeFn = void (*)(const DecodeParams);

// One instantiation per weight format, sequence count (1, or up to 4), model family and head dim (hd 128: four
// dims a lane, 64: two), so each holds only the code its model executes.
template <int QW, int DL>
DecodeFn pick_fm(int fmt, int M) {
    if (fmt == kFP8) return M == 1 ? decode_kernel<kFP8, 1, QW, DL> : decode_kernel<kFP8, kDecodeMaxSeqs, QW, DL>;
    return M == 1 ? decode_kernel<kFP4, 1, QW, DL> : decode_kernel<kFP4, kDecodeMaxSeqs, QW, DL>;
}
DecodeFn pick(const DecodeParams& p) {
    if (!p.qwen) return p.hd == 64 ? pick_fm<0, 2>(p.fmt, p.M) : nullptr;
    return p.hd == 128 ? pick_fm<1, 4>(p.fmt, p.M) : p.hd == 64 ? pick_fm<1, 2>(p.fmt, p.M) : nullptr;
}

int64_t padded_x_bytes(int fmt, int M, int K) { return gemv_x_bytes(fmt, M, K); }

int attn_scratch_floats(const DecodeParams& p) {
    const int Gq = p.H / p.KV;
    return Gq * p.hd + 2 * p.hd + Gq * p.span + kW * Gq * p.hd + 2 * Gq;
}

int64_t table_bytes(const DecodeParams& p) { return (int64_t(p.layers) * int64_t(sizeof(DecodeLayer)) + 127) / 128 * 128; }

size_t smem_bytes(const DecodeParams& p) {
    return kDHdr + size_t(table_bytes(p)) + size_t(p.xs_bytes) + size_t(p.kv_bytes) + size_t(p.nslot) * p.slot_bytes;
}

}  // namespace

bool plan_decode(DecodeParams& p, std::string* why) {
    auto no = [&](const char* w) {
        if (why) *why = w;
        return false;
    };
    if (p.M < 1 || p.M > kDecodeMaxSeqs) return no("1..4 sequences");
    if (p.fmt != kFP8 && p.fmt != kFP4) return no("FP8 or FP4 weights");
    if (p.layers < 1 || p.layers > kDecodeMaxLayers) return no("layer count");
    if (p.hd != 64 && p.hd != 128) return no("head_dim 64 or 128");
    if (p.KV < 1 || p.H % p.KV || p.H / p.KV > kMaxGq) return no("at most 4 query heads per KV head");
    if (p.C % 128 || p.F % 32 || (p.H * p.hd) % 32) return no("embd % 128, ff % 32");
    if (int64_t(p.M) * p.C / 128 > kMaxStatSlots) return no("norm partials");
    if (p.span < 32 || p.span > kMaxSpan || p.span % 32 || p.max_splits < (p.context + p.span - 1) / p.span)
        return no("attention split");
    p.grid = num_sms();
    if ((p.C + p.grid - 1) / p.grid > kOwnRows) return no("residual rows per CTA");
    if (!p.x_tw || !p.qkv_tw || !p.att_tw || !p.h_tw || !p.part_tw || !p.epoch || !p.sync)
        return no("exchange buffers");
    // GEMV inputs: one sequence, f32 rows in the CUDA-core kernel's permuted layout; 2..4, the tensor-core B
    // operand: 2M f16 rows + block scales (+ LayerNorm's raw f32 rows)
    auto bxs = [&](int64_t K) {
        return p.M == 1 ? padded_x_bytes(p.fmt, p.M, int(K))
                        : 4 * p.M * K + p.M * (K / 32) * 4 + (p.qwen ? 0 : 4 * p.M * K);
    };
    int64_t xs = std::max({bxs(p.C), bxs(int64_t(p.H) * p.hd), bxs(p.F), int64_t(attn_scratch_floats(p)) * 4});
    xs = (xs + 127) / 128 * 128;
    const int64_t rb_max = std::max({p.rb_c * (p.qwen ? 2 : 1), p.rb_att, p.rb_f});
    int64_t slot = std::max<int64_t>(kSlotBytes, (rb_max + 1023) / 1024 * 1024);
    // One sequence: a warp's pass touches rows up to kMaxGroupRows - 1 apart; while it waits for the last of their
    // stages it holds the first, so the ring must hold every stage a pass can span plus one being refilled (fewer
    // when the CTA's share of the matrix has fewer stages). 2..4 sequences: every warp takes every stage of a
    // phase in order and lets it go before the next, so two slots keep the ring moving. Every warp walks every
    // stage in order, so no warp waits on a slot more than one phase ahead of it.
    auto need_for = [&](int64_t rows, int64_t rbe) {
        const int64_t rps = std::min<int64_t>(slot / rbe, 16 * kW), share = (rows + p.grid - 1) / p.grid;
        const int64_t nst = (share + rps - 1) / rps, span = (kMaxGroupRows - 1) / rps + 2;
        return int(std::min(nst, span) + 1);
    };
    const int need = p.M > 1 ? 2
                             : std::max({need_for(p.QW, p.rb_c), need_for(p.C, p.rb_att),
                                         need_for(p.F, p.rb_c * (p.qwen ? 2 : 1)), need_for(p.C, p.rb_f),
                                         need_for(p.V, p.rb_c), 2});
    const int64_t kvb = int64_t(2) * kMaxSpan * p.hd * 2;
    DecodeFn k = pick(p);
    if (!k) return no("GPT-2 with head_dim 64, Qwen3 with head_dim 64 or 128");
    // the instantiation's own static shared memory against the device's per-block opt-in limit
    cudaFuncAttributes fa{};
    int dev = 0, optin = 0;
    if (cudaFuncGetAttributes(&fa, k) != cudaSuccess || cudaGetDevice(&dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev) != cudaSuccess) {
        cudaGetLastError();
        return no("kernel attributes");
    }
    const int64_t budget = int64_t(optin) - int64_t(fa.sharedSizeBytes) - kDHdr - table_bytes(p) - xs - kvb;
    const int nslot = int(std::min<int64_t>(kMaxSlots, budget / slot));
    if (nslot < need) return no("shared memory: weight rows too wide for the slot ring");
    p.xs_bytes = int(xs);
    p.kv_bytes = int(kvb);
    p.slot_bytes = int(slot);
    p.nslot = nslot;
    const size_t smem = smem_bytes(p);
    int per_sm = 0;
    cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
    if (e == cudaSuccess) e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, k, kThr, smem);
    if (e != cudaSuccess || per_sm < 1) {
        cudaGetLastError();
        if (why)
            *why = std::string("the kernel does not fit one CTA per SM (") + cudaGetErrorString(e) + ", " +
                   std::to_string(smem) + " B of dynamic shared memory)";
        return false;
    }
    return true;
}

cudaError_t decode_clear_abort() {
    const unsigned zero = 0u;
    return cudaMemcpyToSymbol(g_dec_abort, &zero, sizeof(zero));
}

void decode_scratch(const DecodeParams& p, DecodeScratch* s) {
    const int Gq = p.H / std::max(1, p.KV);
    s->part_words = int64_t(p.M) * p.KV * p.max_splits * Gq * (p.hd + 2);
    s->x_words = int64_t(p.M) * p.C;
    s->qkv_words = int64_t(p.M) * p.QW;
    s->att_words = int64_t(p.M) * p.H * p.hd;
    s->h_words = int64_t(p.M) * p.F;
}

cudaError_t launch_decode(const DecodeParams& p, cudaStream_t st) {
    DecodeFn k = pick(p);
    if (!k) return cudaErrorInvalidValue;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(p.grid);
    cfg.blockDim = dim3(kThr);
    cfg.dynamicSmemBytes = smem_bytes(p);
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, k, p);
}

}  // namespace neko
