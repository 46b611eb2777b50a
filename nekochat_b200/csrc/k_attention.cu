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

#include "neko_common.cuh"
#include "neko_internal.h"

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

Geometry plan(int rows, int n_kv, int max_pos, int G, int hd) {
    const int L = max_pos + 1;
    const int sms = num_sms();
    Geometry g;
    g.chunk = chunk_for(hd);
    // enough CTAs for two waves over the SMs, at least one chunk of keys per split
    const int want = std::max(1, (2 * sms + rows * n_kv - 1) / (rows * n_kv));
    int span = (L + want - 1) / want;
    span = std::max(g.chunk, (span + g.chunk - 1) / g.chunk * g.chunk);
    g.span = span;
    g.splits = (L + span - 1) / span;
    g.smem = layout(G, hd, g.chunk).total;
    return g;
}

}  // namespace

void attention_scratch(int rows, int n_head, int n_kv, int hd, int max_pos, int64_t* part_floats, int64_t* tickets) {
    const Geometry g = plan(rows, n_kv, max_pos, n_head / std::max(1, n_kv), hd);
    *part_floats = g.splits > 1 ? int64_t(rows) * n_head * g.splits * (hd + 2) : 0;
    *tickets = int64_t(rows) * n_kv;
}

cudaError_t launch_attention(const AttnArgs& a, cudaStream_t st, bool pdl) {
    if (a.rows <= 0) return cudaSuccess;
    if (a.n_kv <= 0 || a.n_head % a.n_kv != 0 || a.n_head / a.n_kv > kMaxGroup || a.hd > kMaxHd || (a.hd % 8))
        return cudaErrorInvalidValue;
    // bulk copies need 16-byte aligned key rows
    if ((a.pos_stride % 8) || (a.head_stride % 8) || (a.slot_stride % 8) ||
        (reinterpret_cast<uintptr_t>(a.kc) & 15) || (reinterpret_cast<uintptr_t>(a.vc) & 15))
        return cudaErrorInvalidValue;
    const Geometry g = plan(a.rows, a.n_kv, a.max_pos, a.n_head / a.n_kv, a.hd);
    if (g.splits > 1) {
        const int64_t need = int64_t(a.rows) * a.n_head * g.splits * (a.hd + 2);
        if (!a.part || !a.tickets || need > a.part_capacity || int64_t(a.rows) * a.n_kv > a.ticket_capacity)
            return cudaErrorInvalidValue;
    }
    static bool attr = false;
    if (!attr) {
        cudaFuncSetAttribute(attention_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 160 * 1024);
        attr = true;
    }
    return launch_ex(attention_kernel, dim3(g.splits, a.n_kv, a.rows), dim3(kAttnThreads), size_t(g.smem), st, pdl, a,
                     g);
}

}  // namespace neko
