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
//  * phases (qkv, attention, o_proj, gate/up, down, LM head) hand their activations over through global memory;
//    a phase waits on a counter that the producing phase's CTAs bump after their writes (release / acquire at
//    GPU scope), so a step costs one on-chip hand-off per phase instead of a launch;
//  * attention folds in the per-head QK RMSNorm, RoPE and the f16 KV store (split-KV items, merged by the last
//    item of a (sequence, KV head) through a ticket).
// The dot products, activation staging, norm prologue and epilogues are the ones of the GEMV kernel (same
// summation order), so both paths give the same logits.
//
// Every wait is bounded (DecodeParams::wait_ns on %globaltimer, 2 s by default): on expiry the kernel records
// kErrMbarTimeout, raises an abort flag that makes every other wait return at once, and the producer waits (bounded) for its copies in flight
// before leaving. The last CTA to finish resets the counters, so the launch can be replayed from a CUDA graph.
#include <algorithm>

#include "gemv_core.cuh"
#include "neko_common.cuh"
#include "neko_internal.h"

namespace neko {

namespace {

constexpr int kW = 12;                 // consumer warps (12 + 1 warps: at most 128 registers a thread)
constexpr int kNT = kW * 32;           // consumer threads
constexpr int kThr = kNT + 32;         // + the producer warp
constexpr int kMaxGroupRows = kW * 4;  // rows the CTA consumes per pass, at most (kRows<1> warps x 4)
constexpr int kMaxSlots = 16;
constexpr int kSlotBytes = 32768;      // bigger stages stream faster (fewer producer / consumer hand-offs)
constexpr int kMaxStatSlots = 256;     // 32-float4 groups with a norm partial (M * C / 128)
constexpr int kChunk = 8192;           // bytes per bulk copy
constexpr int kPhases = 5;             // per layer: qkv, attention, o_proj, up, down
constexpr int kMaxGq = 4;              // query heads per KV head
constexpr int kMaxSpan = 64;           // keys per attention item (staged in shared memory)
constexpr int kStaticSmem = 8192;      // upper bound of the kernel's static shared memory

enum Ph : int { kQkv = 0, kAttn = 1, kO = 2, kUp = 3, kDown = 4, kHead = 5 };

__device__ unsigned g_dec_abort;  // raised by the first wait that gives up

__device__ __forceinline__ uint64_t gtimer() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}
__device__ __forceinline__ void csync() { asm volatile("bar.sync 1, %0;" ::"n"(kNT) : "memory"); }
__device__ __forceinline__ unsigned ld_acquire(const unsigned* p) {
    unsigned v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
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

// Bounded mbarrier wait for the decode kernel (gives up on abort or after lim ns).
__device__ bool dwait(uint64_t* bar, uint32_t parity, uint64_t lim, uint32_t hint_ns = 20000) {
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

// Consumer-side wait until *ctr >= target: thread 0 polls with acquire loads, then a consumer barrier.
__device__ bool wait_count(const unsigned* ctr, unsigned target, int* flag, const int* abort, uint64_t lim) {
    if (threadIdx.x == 0) {
        int ok = *reinterpret_cast<const volatile int*>(abort) == 0 ? 1 : 0;
        if (ok && ld_acquire(ctr) < target) {
            const uint64_t t0 = gtimer();
            for (uint32_t i = 1;; i++) {
                if (ld_acquire(ctr) >= target) break;
                if ((i & 63) == 0) {
                    if (aborted()) {
                        ok = 0;
                        break;
                    }
                    if (gtimer() - t0 > lim) {
                        give_up();
                        ok = 0;
                        break;
                    }
                }
            }
        }
        *flag = ok;
    }
    csync();
    return *reinterpret_cast<volatile int*>(flag) != 0;
}

// All consumer warps are done with the phase's writes: publish them.
__device__ __forceinline__ void signal(unsigned* ctr) {
    csync();
    if (threadIdx.x == 0) asm volatile("red.release.gpu.global.add.u32 [%0], 1;" ::"l"(ctr) : "memory");
}

// One GEMV phase of the step.
struct GemvPh {
    const uint8_t* W;
    int64_t rb;
    int rows, K, pair;  // pair: SwiGLU, gate row n with up row n + rows
    const float* x;
    int64_t xs;
    int embed_src;      // activations are the token embeddings (layer 0)
    int norm;
    const float *gamma, *beta, *bias;
    int flags;
    float* y;
    int64_t ys;
    int head;
};

__device__ __forceinline__ GemvPh gemv_ph(const DecodeParams& p, int l, int kind) {
    GemvPh g{};
    const int lnk = p.qwen ? kNormRms : kNormLayer;
    if (kind == kHead) {
        g.W = p.embed; g.rb = p.rb_c; g.rows = p.V; g.K = p.C;
        g.x = p.x; g.xs = p.C; g.norm = lnk; g.gamma = p.normf; g.beta = p.normfb;
        g.y = p.logits; g.ys = p.V; g.head = 1;
        return g;
    }
    const DecodeLayer& L = p.layer[l];
    if (kind == kQkv) {
        g.W = L.wqkv; g.rb = p.rb_c; g.rows = p.QW; g.K = p.C;
        g.x = p.x; g.xs = p.C; g.embed_src = l == 0; g.norm = lnk; g.gamma = L.ln1; g.beta = L.ln1b;
        g.bias = L.bqkv; g.flags = p.qwen ? 0 : kBias; g.y = p.qkv; g.ys = p.QW;
    } else if (kind == kO) {
        g.W = L.wo; g.rb = p.rb_att; g.rows = p.C; g.K = p.H * p.hd;
        g.x = p.att; g.xs = int64_t(p.H) * p.hd;
        g.bias = L.bo; g.flags = kAccumulate | (p.qwen ? 0 : kBias); g.y = p.x; g.ys = p.C;
    } else if (kind == kUp) {
        g.W = L.wup; g.rb = p.rb_c; g.rows = p.F; g.K = p.C; g.pair = p.qwen;
        g.x = p.x; g.xs = p.C; g.norm = lnk; g.gamma = L.ln2; g.beta = L.ln2b;
        g.bias = L.bup; g.flags = p.qwen ? 0 : (kBias | kGelu); g.y = p.h; g.ys = p.F;
    } else {
        g.W = L.wdown; g.rb = p.rb_f; g.rows = p.C; g.K = p.F;
        g.x = p.h; g.xs = p.F;
        g.bias = L.bdown; g.flags = kAccumulate | (p.qwen ? 0 : kBias); g.y = p.x; g.ys = p.C;
    }
    return g;
}

__device__ __forceinline__ void cta_rows(int rows, int grid, int& r0, int& r1) {
    const int rpc = (rows + grid - 1) / grid;
    r0 = min(rows, int(blockIdx.x) * rpc);
    r1 = min(rows, r0 + rpc);
}
__device__ __forceinline__ int stage_rows(const DecodeParams& p, const GemvPh& g) {
    return int(int64_t(p.slot_bytes) / (g.rb * (g.pair ? 2 : 1)));
}
// GEMV phase kind of the k-th matrix of layer l (l == layers: the LM head).
__device__ __forceinline__ int mat_kind(const DecodeParams& p, int l, int k) {
    return l == p.layers ? kHead : k == 0 ? kQkv : k == 1 ? kO : k == 2 ? kUp : kDown;
}

// ---------------------------------------------------------------------------------------------- producer
__device__ void producer(const DecodeParams& p, uint64_t* full, uint64_t* empty, uint8_t* ring, int lane) {
    uint32_t st = 0;
    bool ok = true;
    for (int l = 0; l <= p.layers && ok; l++) {
        for (int k = 0; k < (l == p.layers ? 1 : 4) && ok; k++) {
            const GemvPh g = gemv_ph(p, l, mat_kind(p, l, k));
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

__device__ __forceinline__ float4 embed4(const DecodeParams& p, int m, int k) {
    const uint8_t* row = p.embed + int64_t(token_of(p, m)) * p.rb_c;
    float4 r = make_float4(dequant_one(p.fmt, row, p.C, k), dequant_one(p.fmt, row, p.C, k + 1),
                           dequant_one(p.fmt, row, p.C, k + 2), dequant_one(p.fmt, row, p.C, k + 3));
    if (p.wpe) {  // GPT-2 learned positions (f32, like the CPU path)
        const float4 w = *reinterpret_cast<const float4*>(p.wpe + int64_t(p.pos[m]) * p.C + k);
        r.x += w.x;
        r.y += w.y;
        r.z += w.z;
        r.w += w.w;
    }
    return r;
}

// Weight rows a warp walks together (independent load streams): more for one sequence, where the registers of
// the activation tiles are free.
template <int NM>
constexpr int kRows = NM == 1 ? 4 : 2;

// Norm weights a consumer thread loads before the phase's wait (they do not depend on the previous phase).
constexpr int kNormPre = 2;
struct NormPre {
    float4 g[kNormPre], b[kNormPre];
};

__device__ __forceinline__ void norm_prefetch(const DecodeParams& p, const GemvPh& g, NormPre& pre) {
    if (g.norm == kNormNone) return;
    const int K4 = g.K / 4, total = p.M * K4;
#pragma unroll
    for (int j = 0; j < kNormPre; j++) {
        const int i = threadIdx.x + j * kNT;
        if (i < total) {
            const int k = 4 * (i % K4);
            pre.g[j] = __ldg(reinterpret_cast<const float4*>(g.gamma + k));
            if (g.norm == kNormLayer) pre.b[j] = __ldg(reinterpret_cast<const float4*>(g.beta + k));
        }
    }
}

// Stages the M activation rows of a phase into the permuted layout, with the norm prologue (RMSNorm /
// LayerNorm over K, sums in double, cpu_ops.cpp:483-511). The rows come straight from L2 into shared memory
// with cp.async (no registers held, every copy of the thread in flight at once); the token embeddings of layer
// 0 are dequantised on the way instead.
template <int FMT>
__device__ void stage_x(const DecodeParams& p, const GemvPh& g, const NormPre& pre, float* xs, double* spart,
                        float* snorm, int warp, int lane) {
    const int tid = threadIdx.x;
    const int K4 = g.K / 4, total = p.M * K4, xrow = seg_count(FMT, g.K) * Seg<FMT>::W;
    const bool norm = g.norm != kNormNone;
    if (g.embed_src) {
        for (int i = tid; i < total; i += kNT) {
            const int m = i / K4, k = 4 * (i - m * K4);
            *reinterpret_cast<float4*>(xs + m * xrow + xperm<FMT>(k)) = embed4(p, m, k);
        }
    } else {
        for (int i = tid; i < total; i += kNT) {
            const int m = i / K4, k = 4 * (i - m * K4);
            asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(xs + m * xrow + xperm<FMT>(k))),
                         "l"(g.x + int64_t(m) * g.xs + k)
                         : "memory");
        }
        asm volatile("cp.async.wait_all;" ::: "memory");
    }
    if (!norm) {
        csync();
        return;
    }
    // K % 128 == 0: the 32 float4 of a warp in one pass share a row
    for (int base = 0; base < total; base += kNT) {
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
                const int q = base / 32 + warp;
                spart[2 * q] = s1;
                spart[2 * q + 1] = s2;
            }
        }
    }
    csync();
    // Every thread totals the partials of the rows it normalises (fixed order), so no second barrier.
    const int gpr = K4 / 32;  // partial slots per row
    for (int i = tid, j = 0; i < total; i += kNT, j++) {
        const int m = i / K4, k = 4 * (i - m * K4);
        double a1 = 0.0, a2 = 0.0;
        for (int q = m * gpr; q < (m + 1) * gpr; q++) {
            a1 += spart[2 * q];
            a2 += spart[2 * q + 1];
        }
        float mean = 0.0f, r;
        if (g.norm == kNormRms) {
            r = float(1.0 / sqrt(a2 / g.K + double(p.eps)));
        } else {
            const double mu = a1 / g.K;
            mean = float(mu);
            r = float(1.0 / sqrt(a2 / g.K - mu * mu + double(p.eps)));
        }
        float4* px = reinterpret_cast<float4*>(xs + m * xrow + xperm<FMT>(k));
        float4 y = *px;
        float4 ga, be;
        if (j < kNormPre) {
            ga = j == 0 ? pre.g[0] : pre.g[kNormPre - 1];
            be = j == 0 ? pre.b[0] : pre.b[kNormPre - 1];
        } else {
            ga = __ldg(reinterpret_cast<const float4*>(g.gamma + k));
            if (g.norm == kNormLayer) be = __ldg(reinterpret_cast<const float4*>(g.beta + k));
        }
        if (g.norm == kNormRms) {
            y.x = __fmul_rn(__fmul_rn(y.x, r), ga.x);
            y.y = __fmul_rn(__fmul_rn(y.y, r), ga.y);
            y.z = __fmul_rn(__fmul_rn(y.z, r), ga.z);
            y.w = __fmul_rn(__fmul_rn(y.w, r), ga.w);
        } else {
            y.x = __fadd_rn(__fmul_rn(__fmul_rn(__fsub_rn(y.x, mean), r), ga.x), be.x);
            y.y = __fadd_rn(__fmul_rn(__fmul_rn(__fsub_rn(y.y, mean), r), ga.y), be.y);
            y.z = __fadd_rn(__fmul_rn(__fmul_rn(__fsub_rn(y.z, mean), r), ga.z), be.z);
            y.w = __fadd_rn(__fmul_rn(__fmul_rn(__fsub_rn(y.w, mean), r), ga.w), be.w);
        }
        *px = y;
    }
    csync();
}

// Shared-memory state of the kernel at file scope, so the phase functions address it directly (a struct of
// pointers passed around ends up in local memory and puts a load on every access).
extern __shared__ __align__(128) uint8_t dsm[];  // barriers | activations | attention keys/values | weight ring
__shared__ double s_part[2 * kMaxStatSlots];      // norm prologue partial sums
__shared__ float s_norm[2 * kDecodeMaxSeqs];
__shared__ unsigned long long s_key[kDecodeMaxSeqs];  // LM head: the CTA's greedy argmax keys
__shared__ int s_flag, s_ticket, s_last, s_abort;      // s_abort: a stage wait of this CTA gave up
__shared__ __align__(8) uint64_t s_attn_bar;           // an attention item's keys / values have landed
__device__ __forceinline__ uint64_t* full_bar() { return reinterpret_cast<uint64_t*>(dsm); }
__device__ __forceinline__ uint64_t* empty_bar() { return reinterpret_cast<uint64_t*>(dsm) + kMaxSlots; }
__device__ __forceinline__ float* xs_buf() { return reinterpret_cast<float*>(dsm + 256); }
__device__ __forceinline__ uint16_t* kv_buf(const DecodeParams& p) {
    return reinterpret_cast<uint16_t*>(dsm + 256 + p.xs_bytes);
}
__device__ __forceinline__ uint8_t* ring_buf(const DecodeParams& p) { return dsm + 256 + p.xs_bytes + p.kv_bytes; }



// One GEMV phase on this CTA's rows: wait for the inputs, stage them, consume the producer's stages. A pass of a
// warp takes RR rows (RR / 2 gate / up pairs for SwiGLU) spaced kW apart, so the CTA's warps walk the stages
// together and free them in order.
template <int FMT, int NM>
__device__ __forceinline__ bool gemv_run(const DecodeParams& p, const GemvPh& g, const unsigned* dep,
                                         unsigned target, uint32_t& st_base, int warp, int lane) {
    constexpr int RR = kRows<NM>;
    int r0, r1;
    cta_rows(g.rows, p.grid, r0, r1);
    if (r0 >= r1) return true;
    NormPre pre;
    norm_prefetch(p, g, pre);
    constexpr float kF = FMT == kFP8 ? kFp8HwFactor : kFp4Factor;
    const int n = r1 - r0, rps = stage_rows(p, g), nst = (n + rps - 1) / rps;
    const int cbytes = code_bytes(FMT, g.K), nseg = seg_count(FMT, g.K), xrow = nseg * Seg<FMT>::W;
    const int rpp = g.pair ? RR / 2 : RR;  // output rows per pass
    RowWalk w{0, 0, int(st_base % uint32_t(p.nslot)), int((st_base / uint32_t(p.nslot)) & 1u)};
    w.advance(warp, rps, p.nslot);  // this warp's first row
    int released = 0;               // stages [0, released) of this phase that this warp has let go
    int waited = -1;                // last stage of this phase this warp has waited for
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
                if (v.s != waited) {
                    int ok = 1;
                    if (lane == 0)
                        ok = mbar_try_wait(&full_bar()[v.slot], v.par) || dwait(&full_bar()[v.slot], v.par, p.wait_ns);
                    if (!__shfl_sync(0xffffffffu, ok, 0)) return false;
                    waited = v.s;
                }
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
    // A wait that gives up stops the consumption but keeps the CTA's barriers in step; the next wait_count (or
    // the end of the step) sees the flag and every consumer warp leaves together.
    if (warp < n && !setup(warp)) {
        if (lane == 0) s_abort = 1;
        return true;
    }
    if (dep && !wait_count(dep, target, &s_flag, &s_abort, p.wait_ns)) return false;
    stage_x<FMT>(p, g, pre, xs_buf(), s_part, s_norm, warp, lane);
    for (int i0 = warp; i0 < n; i0 += kW * rpp) {
        if (i0 != warp && !setup(i0)) {
            if (lane == 0) s_abort = 1;
            return true;
        }
        // SwiGLU: up row r sits at rpp + r (gate rows nr .. rpp - 1 are computed but unused)
        const int nrows = g.pair ? rpp + nr : nr;
        float acc[RR][NM];
        dot_rows<FMT, NM, RR>(wr, nrows, cbytes, nseg, xs_buf(), xrow, p.M, lane, acc);
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
                float* dst = g.y + int64_t(m) * g.ys + row;
                const float gs = red_[r][m];
                float val;
                if (g.pair) {
                    const float us = red_[rpp + r < RR ? rpp + r : 0][m];
                    val = gs / (1.0f + expf(-gs)) * us;  // cpu::siluMul (cpu_ops.cpp:526-533)
                } else {
                    val = gs;
                    if (g.flags & kBias) val += g.bias[row];
                    if (g.flags & kGelu) val = gelu(val);
                    if (g.flags & kAccumulate) val += *dst;
                }
                *dst = val;
                if (g.head) best[m] = max(best[m], argmax_key(val, row));
            }
        }
        __syncwarp();
        w = v;  // the first row of this warp's next pass
        const int s_next = i0 + kW * rpp < n ? w.s : nst;
        for (; released < s_next; released++)
            if (lane == 0) mbar_arrive(&empty_bar()[(st_base + uint32_t(released)) % uint32_t(p.nslot)]);
    }
    __syncwarp();
    for (; released < nst; released++)
        if (lane == 0) mbar_arrive(&empty_bar()[(st_base + uint32_t(released)) % uint32_t(p.nslot)]);
    if (g.head) {  // one shared atomic per warp and sequence
#pragma unroll
        for (int m = 0; m < NM; m++) {
            if (m >= p.M) break;
            unsigned long long k = best[m];
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) k = max(k, __shfl_xor_sync(0xffffffffu, k, o));
            if (lane == 0 && k) atomicMax(&s_key[m], k);
        }
    }
    st_base += uint32_t(nst);
    return true;
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
    int m = 0, rem = it;
    while (rem >= p.KV * Sm[m]) {
        rem -= p.KV * Sm[m];
        m++;
    }
    a.m = m;
    a.ns = Sm[m];
    a.g = rem / a.ns;
    a.j = rem - a.g * a.ns;
    a.pos = Pm[m];
    a.slot = p.slots[m];
    a.k0 = a.j * p.span;
    a.n = min(a.pos + 1, a.k0 + p.span) - a.k0;
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
        Sm[m] = (pos + 1 + p.span - 1) / p.span;
        total += p.KV * Sm[m];
    }
    return total;
}

// One thread: copies the item's cached keys and values (positions below pos; the newest comes from this step)
// into shared memory with two bulk copies (a head's positions are contiguous in the cache), completing on
// s_attn_bar. The cache rows are from earlier steps, so this is issued long before the item runs.
__device__ __forceinline__ void attn_issue(const DecodeParams& p, int l, const AttnItem& a) {
    const DecodeLayer& Ly = p.layer[l];
    const int nold = min(a.n, a.pos - a.k0);  // rows that are in the cache already
    const uint32_t bytes = uint32_t(nold) * uint32_t(p.hd) * 2u;
    const int64_t base = int64_t(a.slot) * p.kv_slot + int64_t(a.g) * p.kv_head + int64_t(a.k0) * p.hd;
    mbar_arrive_expect_tx(&s_attn_bar, 2u * bytes);
    if (bytes) {
        bulk_g2s(kv_buf(p), Ly.kc + base, bytes, &s_attn_bar);
        bulk_g2s(kv_buf(p) + p.span * p.hd, Ly.vc + base, bytes, &s_attn_bar);
    }
}

// Items (sequence m, KV head g, split j) over keys [j * span, min(L, (j + 1) * span)), L = pos + 1. Each item
// rebuilds the group's query heads (QK-norm + RoPE, qwen3_model.cpp:249-262) and the new key / value
// (f16-rounded, as the cache holds them); split 0 stores them at pos (cpu::storeKv). The older keys and values
// are copied to shared memory before the wait for this step's qkv. Lane l owns dims [l * DL, l * DL + DL) of a
// key / value row for scores (cpu_ops.cpp:558) and P.V.
template <int DL>
__device__ __noinline__ bool attn_run(const DecodeParams& p, int l, int& issued, int warp, int lane) {
    const int Gq = p.H / p.KV, hd = p.hd, span = p.span;
    int Sm[kDecodeMaxSeqs], Pm[kDecodeMaxSeqs];
    const int total = attn_items(p, Sm, Pm);
    if (int(blockIdx.x) >= total) return true;
    unsigned* sy = p.sync + l * kPhases;
    const DecodeLayer& Ly = p.layer[l];
    float* sq = xs_buf();             // [Gq][hd]
    float* snk = sq + Gq * hd;        // [hd]
    float* snv = snk + hd;            // [hd]
    float* sc = snv + hd;             // [Gq][span]
    float* red = sc + Gq * span;      // [kW][Gq][hd]
    float* sst = red + kW * Gq * hd;  // [Gq](max, sum)
    const uint16_t* kbuf = kv_buf(p);  // [span][hd]
    const uint16_t* vbuf = kv_buf(p) + span * hd;

    // The first item's keys / values were requested at the start of the layer (attn_issue); before the wait,
    // the rotation and norm weights it needs.
    AttnItem a = attn_item(p, Sm, Pm, blockIdx.x);
    float cs_c[DL / 2], cs_s[DL / 2], wn[DL];
    auto load_rot = [&](const AttnItem& it) {
        if (p.qwen && warp <= Gq) {
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
    // stall_test: wait for one CTA more than there are, so the wait runs out (timeout path test)
    if (!wait_count(sy + kQkv, unsigned(p.grid + (p.stall_test ? 1 : 0)), &s_flag, &s_abort, p.wait_ns))
        return false;

    for (int it = blockIdx.x; it < total; it += p.grid) {
        if (it != int(blockIdx.x)) {  // later items of this CTA (long contexts): requested after the previous
            a = attn_item(p, Sm, Pm, it);
            load_rot(a);
        }
        const int L = a.pos + 1, n = a.n, g = a.g, m = a.m;
        const bool has_new = a.k0 + n == L;
        const float* row = p.qkv + int64_t(m) * p.QW;
        // 1. query heads of the group, the new key and value
        if (warp < Gq + 2) {
            const int which = warp < Gq ? 0 : warp == Gq ? 1 : 2;
            const int col = which == 0 ? (g * Gq + warp) * hd : which == 1 ? (p.H + g) * hd : (p.H + p.KV + g) * hd;
            float e[DL];
#pragma unroll
            for (int i = 0; i < DL; i++) e[i] = __ldcg(row + col + lane + 32 * i);
            if (p.qwen && which != 2) {
                double ss = 0.0;
#pragma unroll
                for (int i = 0; i < DL; i++) ss += double(e[i]) * e[i];
                ss = wsum_d(ss);
                const float sn = float(1.0 / sqrt(ss / hd + double(p.eps)));
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
                float* dsm = which == 1 ? snk : snv;
#pragma unroll
                for (int i = 0; i < DL; i++) {
                    const __half hv = __float2half_rn(e[i]);
                    dsm[lane + 32 * i] = __half2float(hv);
                    if (a.j == 0 && p.pos[m] == a.pos) cache[lane + 32 * i] = __half_as_ushort(hv);
                }
            }
        }
        if (!dwait(&s_attn_bar, uint32_t(issued - 1) & 1u, p.wait_ns)) {
            // the keys never landed: leave (the consumers' barriers stay in step: every thread is here)
            if (threadIdx.x == 0) s_abort = 1;
            csync();
            return false;
        }
        csync();
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
        // 5. merge the warps; one split: the output, else a partial for the ticket merge
        const int outs = Gq * hd;
        float* att = p.att + int64_t(m) * p.H * hd + int64_t(g) * Gq * hd;
        for (int o = threadIdx.x; o < outs; o += kNT) {
            float sacc = 0.0f;
#pragma unroll
            for (int w = 0; w < kW; w++) sacc += red[w * outs + o];
            const int gq = o / hd;
            if (a.ns == 1) {
                att[o] = sacc / sst[2 * gq + 1];
            } else {
                float* pr = p.part + (((int64_t(m) * p.KV + g) * p.max_splits + a.j) * Gq + gq) * (hd + 2);
                pr[2 + (o - gq * hd)] = sacc;
                if (o - gq * hd == 0) {
                    pr[0] = sst[2 * gq];
                    pr[1] = sst[2 * gq + 1];
                }
            }
        }
        if (a.ns == 1) {
            signal(sy + kAttn);
            csync();
            continue;
        }
        __threadfence();
        csync();
        if (threadIdx.x == 0) {
            unsigned* tk = p.tickets + m * p.KV + g;
            const unsigned t = atomicAdd(tk, 1u);
            s_ticket = t == unsigned(a.ns - 1) ? 1 : 0;
            if (t == unsigned(a.ns - 1)) *tk = 0u;  // every item of (m, g) has its ticket: ready for the next layer
        }
        csync();
        if (*reinterpret_cast<volatile int*>(&s_ticket)) {
            __threadfence();
            for (int o = threadIdx.x; o < outs; o += kNT) {
                const int gq = o / hd, d = o - gq * hd;
                const float* base = p.part + ((int64_t(m) * p.KV + g) * p.max_splits * Gq + gq) * (hd + 2);
                const int64_t sstride = int64_t(Gq) * (hd + 2);
                float mx = -INFINITY;
                for (int sp = 0; sp < a.ns; sp++) mx = fmaxf(mx, __ldcg(base + sp * sstride));
                float num = 0.0f, den = 0.0f;
                for (int sp = 0; sp < a.ns; sp++) {
                    const float w = expf(__ldcg(base + sp * sstride) - mx);
                    den += __ldcg(base + sp * sstride + 1) * w;
                    num += __ldcg(base + sp * sstride + 2 + d) * w;
                }
                att[o] = num / den;
            }
            signal(sy + kAttn);
        }
        csync();
    }
    return true;
}

// ---------------------------------------------------------------------------------------------- the kernel
template <int FMT, int NM>
__global__ void __launch_bounds__(kThr, 1) decode_kernel(const __grid_constant__ DecodeParams p) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (threadIdx.x == 0) {
        for (int s = 0; s < p.nslot; s++) {
            mbar_init(&full_bar()[s], 1);
            mbar_init(&empty_bar()[s], kW);
        }
        mbar_init(&s_attn_bar, 1);
        fence_barrier_init();
    }
    if (threadIdx.x < kDecodeMaxSeqs) s_key[threadIdx.x] = 0ull;
    if (threadIdx.x == 0) s_abort = 0;
    __syncthreads();
    if (warp == kW) {
        producer(p, full_bar(), empty_bar(), ring_buf(p), lane);
        return;
    }

    for (int m = threadIdx.x; m < p.M; m += kNT)
        if (p.pos[m] < 0 || p.pos[m] >= p.context) set_device_error(kErrBadIndex);
    // The residual stream starts as the token embeddings (+ positions); each CTA writes the rows it owns in the
    // o_proj / down phases, which are the only phases that read them back.
    {
        int n0, n1;
        cta_rows(p.C, p.grid, n0, n1);
        const int w = n1 - n0;
        for (int i = threadIdx.x; i < p.M * w; i += kNT) {
            const int m = i / w, c = n0 + (i - m * w);
            float v = dequant_one(p.fmt, p.embed + int64_t(token_of(p, m)) * p.rb_c, p.C, c);
            if (p.wpe) v += p.wpe[int64_t(p.pos[m]) * p.C + c];
            p.x[int64_t(m) * p.C + c] = v;
        }
    }
    // Phases in order: per layer qkv, attention, o_proj, up, down; then the LM head. Each GEMV phase waits for the
    // counter of the phase that produced its activations (the attention counter counts (sequence, KV head)
    // merges, the others CTAs) and bumps its own.
    uint32_t st = 0;
    int issued = 0;  // attention copies requested so far (the parity of s_attn_bar)
    int Sm[kDecodeMaxSeqs], Pm[kDecodeMaxSeqs];
    const bool attn_cta = int(blockIdx.x) < attn_items(p, Sm, Pm);
    for (int l = 0; l <= p.layers; l++) {
        unsigned* sy = p.sync + l * kPhases;
        for (int k = 0; k < (l == p.layers ? 1 : kPhases); k++) {
            if (k == kQkv && l < p.layers && attn_cta) {  // this layer's first attention item: keys / values now
                if (threadIdx.x == 0) attn_issue(p, l, attn_item(p, Sm, Pm, blockIdx.x));
                issued++;
            }
            // Leaving early (a wait gave up): no attention copy of ours may still be landing in shared memory.
            auto drain = [&]() {
                if (threadIdx.x == 0 && issued > 0) {
                    const uint64_t t0 = gtimer();
                    while (!mbar_try_wait(&s_attn_bar, uint32_t(issued - 1) & 1u) && gtimer() - t0 < p.wait_ns) {
                    }
                }
            };
            if (k == kAttn) {
                const bool ok = p.hd == 128 ? attn_run<4>(p, l, issued, warp, lane)
                                            : attn_run<2>(p, l, issued, warp, lane);
                if (!ok) {
                    drain();
                    return;
                }
                continue;
            }
            const int kind = l == p.layers ? int(kHead) : k;
            const unsigned* dep = kind == kQkv ? (l ? sy - kPhases + kDown : nullptr)
                                : kind == kHead ? sy - kPhases + kDown : sy + k - 1;
            const unsigned target = kind == kO ? unsigned(p.M * p.KV) : unsigned(p.grid);
            if (!gemv_run<FMT, NM>(p, gemv_ph(p, l, kind), dep, target, st, warp, lane)) {
                drain();
                return;
            }
            if (kind != kHead) signal(sy + k);
        }
    }
    csync();
    if (*reinterpret_cast<volatile int*>(&s_abort)) return;
    if (threadIdx.x < p.M && s_key[threadIdx.x]) atomicMax(p.keys + threadIdx.x, s_key[threadIdx.x]);
    __threadfence();
    csync();
    if (threadIdx.x == 0) s_last = atomicAdd(p.sync + p.layers * kPhases, 1u) == unsigned(p.grid - 1) ? 1 : 0;
    csync();
    if (!s_last) return;
    // Last CTA: every other CTA has passed its last wait. Greedy token per sequence (argmax_finalize_kernel
    // semantics), then reset the counters for the next launch.
    __threadfence();
    if (threadIdx.x < p.M) {
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
    for (int i = threadIdx.x; i <= p.layers * kPhases; i += kNT) p.sync[i] = 0u;
}

using DecodeFn = void (*)(const DecodeParams);

DecodeFn pick(int fmt, int M) {
    if (fmt == kFP8) return M == 1 ? decode_kernel<kFP8, 1> : decode_kernel<kFP8, kDecodeMaxSeqs>;
    return M == 1 ? decode_kernel<kFP4, 1> : decode_kernel<kFP4, kDecodeMaxSeqs>;
}

int64_t padded_x_bytes(int fmt, int M, int K) { return gemv_x_bytes(fmt, M, K); }

int attn_scratch_floats(const DecodeParams& p) {
    const int Gq = p.H / p.KV;
    return Gq * p.hd + 2 * p.hd + Gq * p.span + kW * Gq * p.hd + 2 * Gq;
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
    int64_t xs = std::max({padded_x_bytes(p.fmt, p.M, p.C), padded_x_bytes(p.fmt, p.M, p.H * p.hd),
                           padded_x_bytes(p.fmt, p.M, p.F), int64_t(attn_scratch_floats(p)) * 4});
    xs = (xs + 127) / 128 * 128;
    const int64_t rb_max = std::max({p.rb_c * (p.qwen ? 2 : 1), p.rb_att, p.rb_f});
    int64_t slot = std::max<int64_t>(kSlotBytes, (rb_max + 1023) / 1024 * 1024);
    // A warp's pass touches rows up to kMaxGroupRows - 1 apart; while it waits for the last of their stages it
    // holds the first, so the ring must hold every stage a pass can span plus one being refilled (fewer when the
    // CTA's share of the matrix has fewer stages).
    auto need_for = [&](int64_t rows, int64_t rbe) {
        const int64_t rps = slot / rbe, share = (rows + p.grid - 1) / p.grid;
        const int64_t nst = (share + rps - 1) / rps, span = (kMaxGroupRows - 1) / rps + 2;
        return int(std::min(nst, span) + 1);
    };
    const int need = std::max({need_for(p.QW, p.rb_c), need_for(p.C, p.rb_att),
                               need_for(p.F, p.rb_c * (p.qwen ? 2 : 1)), need_for(p.C, p.rb_f),
                               need_for(p.V, p.rb_c), 2});
    const int64_t kvb = int64_t(2) * kMaxSpan * p.hd * 2;
    const int64_t budget = 227 * 1024 - kStaticSmem - 256 - xs - kvb;
    const int nslot = int(std::min<int64_t>(kMaxSlots, budget / slot));
    if (nslot < need) return no("shared memory: weight rows too wide for the slot ring");
    p.xs_bytes = int(xs);
    p.kv_bytes = int(kvb);
    p.slot_bytes = int(slot);
    p.nslot = nslot;
    DecodeFn k = pick(p.fmt, p.M);
    const size_t smem = 256 + size_t(p.xs_bytes) + size_t(p.kv_bytes) + size_t(p.nslot) * p.slot_bytes;
    int per_sm = 0;
    if (cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem)) != cudaSuccess ||
        cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, k, kThr, smem) != cudaSuccess || per_sm < 1) {
        cudaGetLastError();
        return no("the kernel does not fit one CTA per SM");
    }
    return true;
}

cudaError_t decode_clear_abort() {
    const unsigned zero = 0u;
    return cudaMemcpyToSymbol(g_dec_abort, &zero, sizeof(zero));
}

void decode_scratch(const DecodeParams& p, int64_t* part_floats, int64_t* tickets, int64_t* counters) {
    const int Gq = p.H / std::max(1, p.KV);
    if (part_floats) *part_floats = int64_t(p.M) * p.KV * p.max_splits * Gq * (p.hd + 2);
    if (tickets) *tickets = int64_t(p.M) * p.KV;
    if (counters) *counters = int64_t(p.layers) * kPhases + 1;
}

cudaError_t launch_decode(const DecodeParams& p, cudaStream_t st) {
    DecodeFn k = pick(p.fmt, p.M);
    const size_t smem = 256 + size_t(p.xs_bytes) + size_t(p.kv_bytes) + size_t(p.nslot) * p.slot_bytes;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(p.grid);
    cfg.blockDim = dim3(kThr);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, k, p);
}

}  // namespace neko
