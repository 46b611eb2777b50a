// Causal grouped-query attention over f16 KV caches: cpu::attention (app/architecture/shared/cpp/cpu_ops.cpp:
// 544-575) and the Attention kernel (gpu/shaders/attention.comp), written for sm_100a.
//
// Each activation row r (one token of some sequence) attends to cache positions [0, pos_r] of its sequence.
// Work unit = (row, KV head, split): the CTA serves the whole GQA group of the KV head (n_head / n_kv query
// heads), so each K/V byte is read once per row. Keys of a split are walked in chunks of kChunk with an online
// softmax (running max and sum, fp32), scores first (one thread per key, 16-byte loads of the key row), then
// P.V (threads own value-dimension pairs). When a row needs several splits (long context, few rows) the
// partial (max, sum, acc) go to scratch and the last CTA of the (row, KV head) to finish merges them: it is
// elected with a ticket counter that it resets, so the kernel can be replayed from a CUDA graph.
#include <algorithm>

#include "neko_common.cuh"
#include "neko_internal.h"

namespace neko {

namespace {

constexpr int kAttnThreads = 128;
constexpr int kChunk = 256;     // keys per chunk (scores kept in shared memory)
constexpr int kMaxGroup = 8;    // query heads per KV head
constexpr int kMaxHd = 256;     // head dim (attention.comp limit)

struct Geometry {
    int splits;    // CTAs per (row, KV head)
    int span;      // keys per split (multiple of kChunk)
};

__device__ __forceinline__ float dot_key(const float* q, const uint16_t* k, int hd) {
    float s = 0.0f;
    if ((hd & 7) == 0) {
        const uint4* k4 = reinterpret_cast<const uint4*>(k);
#pragma unroll 4
        for (int i = 0; i < hd / 8; i++) {
            const uint4 w = k4[i];
            const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&w.x));
            const float2 b = __half22float2(*reinterpret_cast<const __half2*>(&w.y));
            const float2 c = __half22float2(*reinterpret_cast<const __half2*>(&w.z));
            const float2 d = __half22float2(*reinterpret_cast<const __half2*>(&w.w));
            const float* qq = q + 8 * i;
            s = fmaf(qq[0], a.x, s);
            s = fmaf(qq[1], a.y, s);
            s = fmaf(qq[2], b.x, s);
            s = fmaf(qq[3], b.y, s);
            s = fmaf(qq[4], c.x, s);
            s = fmaf(qq[5], c.y, s);
            s = fmaf(qq[6], d.x, s);
            s = fmaf(qq[7], d.y, s);
        }
    } else {
        const __half2* k2 = reinterpret_cast<const __half2*>(k);
        for (int i = 0; i < hd / 2; i++) {
            const float2 a = __half22float2(k2[i]);
            s = fmaf(q[2 * i], a.x, s);
            s = fmaf(q[2 * i + 1], a.y, s);
        }
    }
    return s;
}

__global__ void __launch_bounds__(kAttnThreads) attention_kernel(const AttnArgs a, const Geometry geo) {
    __shared__ float sq[kMaxGroup * kMaxHd];          // query heads of the group
    __shared__ float sc[kMaxGroup * kChunk];          // chunk scores -> probabilities
    __shared__ float red[kMaxGroup][kAttnThreads / 32];
    __shared__ float stage[kMaxGroup * kMaxHd];       // P.V partials of one key group
    __shared__ int last;

    const int split = blockIdx.x, kvh = blockIdx.y, r = blockIdx.z;
    const int G = a.n_head / a.n_kv, hd = a.hd;
    pdl_wait();
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
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;

    for (int i = tid; i < G * hd; i += kAttnThreads)
        sq[i] = a.q[int64_t(r) * a.q_stride + int64_t(kvh * G + i / hd) * hd + (i % hd)];
    const uint16_t* kbase = a.kc + int64_t(slot) * a.slot_stride + int64_t(kvh) * a.head_stride;
    const uint16_t* vbase = a.vc + int64_t(slot) * a.slot_stride + int64_t(kvh) * a.head_stride;

    // value-dimension ownership: half2 pair dp, keys kg, kg + kgroups, ...
    const int dpairs = hd / 2;
    const int kgroups = kAttnThreads / dpairs;  // >= 1 since hd <= 256
    const int dp = tid % dpairs, kg = tid / dpairs;
    const bool pv_active = kg < kgroups;

    float m_run[kMaxGroup], l_run[kMaxGroup], acc[kMaxGroup][2];
#pragma unroll
    for (int g = 0; g < kMaxGroup; g++) {
        m_run[g] = -INFINITY;
        l_run[g] = 0.0f;
        acc[g][0] = acc[g][1] = 0.0f;
    }
    __syncthreads();

    for (int j0 = j_begin; j0 < j_end; j0 += kChunk) {
        const int n = min(kChunk, j_end - j0);
        // scores: s = (q . k) * scale   (cpu_ops.cpp:558)
        float cmax[kMaxGroup];
#pragma unroll
        for (int g = 0; g < kMaxGroup; g++) cmax[g] = -INFINITY;
        for (int jj = tid; jj < n; jj += kAttnThreads) {
            const uint16_t* k = kbase + int64_t(j0 + jj) * a.pos_stride;
#pragma unroll
            for (int g = 0; g < kMaxGroup; g++) {
                if (g >= G) break;
                const float s = dot_key(sq + g * hd, k, hd) * a.scale;
                sc[g * kChunk + jj] = s;
                cmax[g] = fmaxf(cmax[g], s);
            }
        }
        // chunk max per head, then new running max
#pragma unroll
        for (int g = 0; g < kMaxGroup; g++) {
            if (g >= G) break;
            const float w = warp_max(cmax[g]);
            if (lane == 0) red[g][warp] = w;
        }
        __syncthreads();
        float m_new[kMaxGroup], corr[kMaxGroup];
#pragma unroll
        for (int g = 0; g < kMaxGroup; g++) {
            if (g >= G) break;
            float w = red[g][0];
            for (int i = 1; i < kAttnThreads / 32; i++) w = fmaxf(w, red[g][i]);
            m_new[g] = fmaxf(m_run[g], w);
            corr[g] = expf(m_run[g] - m_new[g]);  // 0 on the first chunk (m_run = -inf)
        }
        // probabilities and their chunk sums
        float lsum[kMaxGroup];
#pragma unroll
        for (int g = 0; g < kMaxGroup; g++) lsum[g] = 0.0f;
        for (int jj = tid; jj < n; jj += kAttnThreads) {
#pragma unroll
            for (int g = 0; g < kMaxGroup; g++) {
                if (g >= G) break;
                const float e = expf(sc[g * kChunk + jj] - m_new[g]);
                sc[g * kChunk + jj] = e;
                lsum[g] += e;
            }
        }
        __syncthreads();  // red reused; probabilities visible
#pragma unroll
        for (int g = 0; g < kMaxGroup; g++) {
            if (g >= G) break;
            const float w = warp_sum(lsum[g]);
            if (lane == 0) red[g][warp] = w;
        }
        __syncthreads();
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
        // P.V
        if (pv_active) {
            const uint16_t* v = vbase + 2 * dp;
            for (int jj = kg; jj < n; jj += kgroups) {
                const float2 vv = __half22float2(*reinterpret_cast<const __half2*>(v + int64_t(j0 + jj) * a.pos_stride));
#pragma unroll
                for (int g = 0; g < kMaxGroup; g++) {
                    if (g >= G) break;
                    const float p = sc[g * kChunk + jj];
                    acc[g][0] = fmaf(p, vv.x, acc[g][0]);
                    acc[g][1] = fmaf(p, vv.y, acc[g][1]);
                }
            }
        }
        __syncthreads();  // sc and red are rewritten by the next chunk
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

Geometry plan(int rows, int n_kv, int max_pos) {
    const int L = max_pos + 1;
    const int sms = num_sms();
    // enough CTAs for two waves over the SMs, but at least one chunk of keys per split
    const int want = std::max(1, (2 * sms + rows * n_kv - 1) / (rows * n_kv));
    int span = (L + want - 1) / want;
    span = std::max(kChunk, (span + kChunk - 1) / kChunk * kChunk);
    Geometry g;
    g.span = span;
    g.splits = (L + span - 1) / span;
    return g;
}

}  // namespace

void attention_scratch(int rows, int n_head, int n_kv, int hd, int max_pos, int64_t* part_floats, int64_t* tickets) {
    const Geometry g = plan(rows, n_kv, max_pos);
    *part_floats = g.splits > 1 ? int64_t(rows) * n_head * g.splits * (hd + 2) : 0;
    *tickets = int64_t(rows) * n_kv;
}

cudaError_t launch_attention(const AttnArgs& a, cudaStream_t st, bool pdl) {
    if (a.rows <= 0) return cudaSuccess;
    if (a.n_kv <= 0 || a.n_head % a.n_kv != 0 || a.n_head / a.n_kv > kMaxGroup || a.hd > kMaxHd || (a.hd & 1))
        return cudaErrorInvalidValue;
    const Geometry g = plan(a.rows, a.n_kv, a.max_pos);
    if (g.splits > 1) {
        const int64_t need = int64_t(a.rows) * a.n_head * g.splits * (a.hd + 2);
        if (!a.part || !a.tickets || need > a.part_capacity || int64_t(a.rows) * a.n_kv > a.ticket_capacity)
            return cudaErrorInvalidValue;
    }
    return launch_ex(attention_kernel, dim3(g.splits, a.n_kv, a.rows), dim3(kAttnThreads), 0, st, pdl, a, g);
}

}  // namespace neko
