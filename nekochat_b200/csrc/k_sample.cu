// Token sampling on the device: Sampler::sample (sampler.cpp:14-55) for each row of logits, with the uniform draw
// supplied by the caller (u in [0, 1) per row), so the choice is a deterministic function of the logits, the
// history and u:
//  * repetition penalty over the distinct ids of the last repeat_last_n history tokens, applied to the logits in
//    place (x / penalty above zero, x * penalty otherwise; ids outside [0, V) skipped);
//  * temperature <= 0: the first index of the maximum (std::max_element);
//  * else the k = top_k (0: V) largest logits, in descending order (ties by index: std::partial_sort leaves them
//    unspecified), exp((x - max) / temperature) in float, their sum in double, the nucleus cut where the double
//    cumulative share first reaches top_p, and the token where r = u x (the kept candidates' sum) first drops to
//    or below zero when the candidates' weights are subtracted in order.
// One CTA of 1024 threads per row. The k-th largest logit is found by a radix select over order-preserving 32-bit
// keys (4 passes of 8-bit histograms); the candidates above it, plus the equal ones of lowest index, are sorted
// in shared memory (bitonic, k <= kMaxTopK); one thread then runs the sequential arithmetic above.
#include <algorithm>
#include <cstdint>

#include "neko_common.cuh"
#include "neko_internal.h"

namespace neko {

namespace {

constexpr int kSampleThreads = 1024;

__device__ __forceinline__ uint32_t order_key(float v) {
    const uint32_t b = __float_as_uint(v);
    return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}
__device__ __forceinline__ float key_value(uint32_t k) {
    return __uint_as_float((k & 0x80000000u) ? (k & 0x7FFFFFFFu) : ~k);
}

// Exclusive prefix sum of one value per thread over the CTA; returns the CTA total in *total.
__device__ int block_scan(int v, int* warp_tot, int* total) {
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    int incl = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int t = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += t;
    }
    __syncthreads();
    if (lane == 31) warp_tot[w] = incl;
    __syncthreads();
    if (w == 0) {
        int s = warp_tot[lane];
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int t = __shfl_up_sync(0xffffffffu, s, o);
            if (lane >= o) s += t;
        }
        warp_tot[lane] = s;  // inclusive over warps
    }
    __syncthreads();
    const int before = w ? warp_tot[w - 1] : 0;
    *total = warp_tot[kSampleThreads / 32 - 1];
    return before + incl - v;
}

__global__ void __launch_bounds__(kSampleThreads) sample_kernel(float* __restrict__ logits, int V,
                                                                const int* __restrict__ hist, const int* hist_len,
                                                                int hist_stride, const double* __restrict__ u,
                                                                const neko_sampling sp, int* __restrict__ out) {
    __shared__ unsigned bins[256];
    __shared__ unsigned long long cand[kMaxTopK];  // (key << 32) | (~index): descending = value desc, index asc
    __shared__ float wgt[kMaxTopK];
    __shared__ int warp_tot[kSampleThreads / 32];
    __shared__ unsigned s_prefix, s_mask, s_need;
    __shared__ int s_count;
    __shared__ unsigned long long s_best[kSampleThreads / 32];
    const int r = blockIdx.x, tid = threadIdx.x, lane = tid & 31, w = tid >> 5;
    float* x = logits + int64_t(r) * V;
    pdl_wait();

    // 1. repetition penalty (sampler.cpp:15-23): the first occurrence of each id in the window
    if (sp.repeat_penalty != 1.0f && sp.repeat_last_n > 0 && hist && hist_len) {
        const int* h = hist + int64_t(r) * hist_stride;
        const int L = min(hist_len[r], hist_stride), start = max(0, L - sp.repeat_last_n);
        for (int i = start + tid; i < L; i += kSampleThreads) {
            const int id = h[i];
            if (id < 0 || id >= V) continue;
            bool first = true;
            for (int j = start; j < i && first; j++)
                if (h[j] == id) first = false;
            if (first) {
                const float v = x[id];
                x[id] = v > 0 ? v / sp.repeat_penalty : v * sp.repeat_penalty;
            }
        }
        __syncthreads();  // the CTA's global writes are visible to its own later reads
    }

    // 2. greedy: the first index of the maximum
    if (sp.temperature <= 0.0f) {
        unsigned long long best = 0ull;
        for (int i = tid; i < V; i += kSampleThreads)
            best = max(best, (static_cast<unsigned long long>(order_key(x[i])) << 32) | (0xFFFFFFFFu - unsigned(i)));
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) best = max(best, __shfl_xor_sync(0xffffffffu, best, o));
        if (lane == 0) s_best[w] = best;
        __syncthreads();
        if (tid == 0) {
            unsigned long long b = 0ull;
            for (int q = 0; q < kSampleThreads / 32; q++) b = max(b, s_best[q]);
            out[r] = int(0xFFFFFFFFu - unsigned(b & 0xFFFFFFFFull));
        }
        return;
    }

    // 3. the k-th largest key: radix select from the top byte down
    const int k = sp.top_k > 0 ? min(sp.top_k, V) : V;  // <= kMaxTopK (the host checks)
    if (tid == 0) {
        s_prefix = 0u;
        s_mask = 0u;
        s_need = unsigned(k);
        s_count = 0;
    }
    for (int pass = 3; pass >= 0; pass--) {
        if (tid < 256) bins[tid] = 0u;
        __syncthreads();
        const unsigned pre = s_prefix, msk = s_mask;
        for (int i = tid; i < V; i += kSampleThreads) {
            const uint32_t key = order_key(x[i]);
            if ((key & msk) == pre) atomicAdd(&bins[(key >> (8 * pass)) & 255u], 1u);
        }
        __syncthreads();
        if (tid == 0) {
            unsigned cum = 0, need = s_need;
            int d = 255;
            for (; d > 0; d--) {
                if (cum + bins[d] >= need) break;
                cum += bins[d];
            }
            s_need = need - cum;  // still to take among keys with this digit
            s_prefix = pre | (unsigned(d) << (8 * pass));
            s_mask = msk | (0xFFu << (8 * pass));
        }
        __syncthreads();
    }
    const uint32_t T = s_prefix;
    const int need_eq = int(s_need);  // keys equal to T to take (lowest indices first)

    // 4. the candidates: every key above T, then the first need_eq keys equal to T in index order
    for (int i = tid; i < V; i += kSampleThreads) {
        const uint32_t key = order_key(x[i]);
        if (key > T) {
            const int slot = atomicAdd(&s_count, 1);
            cand[slot] = (static_cast<unsigned long long>(key) << 32) | (0xFFFFFFFFu - unsigned(i));
        }
    }
    __syncthreads();
    const int above = s_count;  // == k - need_eq
    int taken = 0;
    for (int base = 0; base < V && taken < need_eq; base += kSampleThreads) {
        const int i = base + tid;
        const int eq = (i < V && order_key(x[i]) == T) ? 1 : 0;
        int tile = 0;
        const int pos = taken + block_scan(eq, warp_tot, &tile);
        if (eq && pos < need_eq) cand[above + pos] = (static_cast<unsigned long long>(T) << 32) | (0xFFFFFFFFu - unsigned(i));
        taken += tile;
        __syncthreads();
    }
    // pad to a power of two and sort descending (bitonic)
    int np2 = 1;
    while (np2 < k) np2 <<= 1;
    for (int i = k + tid; i < np2; i += kSampleThreads) cand[i] = 0ull;
    __syncthreads();
    for (int size = 2; size <= np2; size <<= 1) {
        for (int stride = size >> 1; stride > 0; stride >>= 1) {
            for (int i = tid; i < np2; i += kSampleThreads) {
                const int j = i ^ stride;
                if (j > i) {
                    const bool desc = (i & size) == 0;
                    const unsigned long long a = cand[i], b = cand[j];
                    if (desc ? a < b : a > b) {
                        cand[i] = b;
                        cand[j] = a;
                    }
                }
            }
            __syncthreads();
        }
    }

    // 5. temperature, nucleus and the draw (sampler.cpp:32-54), sequentially in the reference's order
    if (tid == 0) {
        const float mx = key_value(uint32_t(cand[0] >> 32));
        double sum = 0.0;
        for (int i = 0; i < k; i++) {
            const float e = expf((key_value(uint32_t(cand[i] >> 32)) - mx) / sp.temperature);
            wgt[i] = e;
            sum += e;
        }
        double cum = 0.0;
        int keep = k;
        for (int i = 0; i < k; i++) {
            cum += wgt[i] / sum;
            if (cum >= sp.top_p) {
                keep = i + 1;
                break;
            }
        }
        double total = 0.0;
        for (int i = 0; i < keep; i++) total += wgt[i];
        double rr = u[r] * total;
        int pick = int(0xFFFFFFFFu - unsigned(cand[keep - 1] & 0xFFFFFFFFull));
        for (int i = 0; i < keep; i++) {
            rr -= wgt[i];
            if (rr <= 0) {
                pick = int(0xFFFFFFFFu - unsigned(cand[i] & 0xFFFFFFFFull));
                break;
            }
        }
        out[r] = pick;
    }
}

}  // namespace

cudaError_t launch_sample(float* logits, int rows, int V, const int* hist, const int* hist_len, int hist_stride,
                          const double* u, const neko_sampling& sp, int* out, cudaStream_t st) {
    if (rows <= 0) return cudaSuccess;
    if (sp.temperature > 0.0f && (sp.top_k <= 0 ? V : std::min(sp.top_k, V)) > kMaxTopK) return cudaErrorNotSupported;
    return launch_ex(sample_kernel, dim3(rows), dim3(kSampleThreads), 0, st, false, logits, V, hist, hist_len,
                     hist_stride, u, sp, out);
}

}  // namespace neko
