// Elementwise and reduction kernels around the matmuls: LayerNorm/RMSNorm, row softmax, argmax, embedding
// gather, Qwen3 QK-norm + RoPE + KV-cache store, KV store, SwiGLU. All memory-bound; each reads its inputs
// once where the row fits on chip and keeps fp32 (fp64 for the norm sums, like cpu_ops.cpp) arithmetic.
#include <cooperative_groups.h>

#include <algorithm>
#include <cfloat>

#include "neko_common.cuh"
#include "neko_internal.h"

namespace neko {

namespace {

constexpr int kNormThreads = 256;
constexpr int kRowCacheFloats = 24 * 1024;  // rows up to 96 KB are read once, into shared memory

__device__ __forceinline__ double warp_sum_d(double v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

__device__ double block_sum_d(double v, double* red) {
    v = warp_sum_d(v);
    const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
    __syncthreads();
    if (l == 0) red[w] = v;
    __syncthreads();
    double t = l < int(blockDim.x >> 5) ? red[l] : 0.0;
    return warp_sum_d(t);
}

// cpu::layerNorm / cpu::rmsNorm (cpu_ops.cpp:483-511), one block per row; layernorm.comp's rowOffset is
// folded into x by the caller. Sums in double like the CPU; the row is cached in shared memory if it fits.
__global__ void __launch_bounds__(kNormThreads) norm_kernel(const float* __restrict__ x, int64_t xs,
                                                            float* __restrict__ y, int64_t ys,
                                                            const float* __restrict__ g,
                                                            const float* __restrict__ b, int C, float eps, int rms) {
    extern __shared__ float row[];
    __shared__ double red[kNormThreads / 32];
    pdl_wait();
    const float* xr = x + int64_t(blockIdx.x) * xs;
    float* yr = y + int64_t(blockIdx.x) * ys;
    const bool cached = C <= kRowCacheFloats;
    double s1 = 0.0, s2 = 0.0;
    for (int c = threadIdx.x; c < C; c += blockDim.x) {
        const float v = xr[c];
        if (cached) row[c] = v;
        s1 += v;
        s2 += double(v) * v;
    }
    float r, m = 0.0f;
    if (rms) {
        s2 = block_sum_d(s2, red);
        r = float(1.0 / sqrt(s2 / C + double(eps)));
    } else {
        const double mean = block_sum_d(s1, red) / C;
        double var = 0.0;
        for (int c = threadIdx.x; c < C; c += blockDim.x) {
            const double d = (cached ? row[c] : xr[c]) - mean;
            var += d * d;
        }
        var = block_sum_d(var, red) / C;
        r = float(1.0 / sqrt(var + double(eps)));
        m = float(mean);
    }
    pdl_trigger();
    for (int c = threadIdx.x; c < C; c += blockDim.x) {
        const float v = cached ? row[c] : xr[c];
        yr[c] = rms ? __fmul_rn(__fmul_rn(v, r), g[c]) : __fadd_rn(__fmul_rn(__fmul_rn(__fsub_rn(v, m), r), g[c]), b[c]);
    }
}

// Row softmax: max, exp(x - max), float sum, times 1 / sum (the softmax inside cpu::attention,
// cpu_ops.cpp:556-572). Rows that fit are read once into shared memory.
__global__ void __launch_bounds__(kNormThreads) softmax_kernel(const float* __restrict__ x, float* __restrict__ y,
                                                               int C) {
    extern __shared__ float row[];
    __shared__ float red[kNormThreads / 32];
    const float* xr = x + int64_t(blockIdx.x) * C;
    float* yr = y + int64_t(blockIdx.x) * C;
    const bool cached = C <= kRowCacheFloats;
    float mx = -INFINITY;
    for (int c = threadIdx.x * 4; c < C; c += blockDim.x * 4) {
        if (c + 3 < C && (C & 3) == 0) {
            const float4 v = *reinterpret_cast<const float4*>(xr + c);
            if (cached) *reinterpret_cast<float4*>(row + c) = v;
            mx = fmaxf(mx, fmaxf(fmaxf(v.x, v.y), fmaxf(v.z, v.w)));
        } else {
            for (int k = c; k < min(C, c + 4); k++) {
                const float v = xr[k];
                if (cached) row[k] = v;
                mx = fmaxf(mx, v);
            }
        }
    }
    mx = warp_max(mx);
    const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
    if (l == 0) red[w] = mx;
    __syncthreads();
    mx = l < kNormThreads / 32 ? red[l] : -INFINITY;
    mx = warp_max(mx);
    float s = 0.0f;
    for (int c = threadIdx.x; c < C; c += blockDim.x) {
        const float e = expf((cached ? row[c] : xr[c]) - mx);
        if (cached) row[c] = e;
        s += e;
    }
    s = block_sum<kNormThreads>(s, red);
    const float inv = 1.0f / s;
    for (int c = threadIdx.x; c < C; c += blockDim.x) yr[c] = (cached ? row[c] : expf(xr[c] - mx)) * inv;
}

// Narrow rows (C <= kWarpRowMaxC): one warp per row, 8 rows per CTA, reductions by warp shuffles only (no block
// barrier); the row is re-read from L1 / L2 for the later passes. Same formulas as norm_kernel / softmax_kernel.
constexpr int kWarpRowMaxC = 4096;
__global__ void __launch_bounds__(kNormThreads) rows_warp_kernel(const float* __restrict__ x, int64_t xs,
                                                                 float* __restrict__ y, int64_t ys,
                                                                 const float* __restrict__ g,
                                                                 const float* __restrict__ b, int rows, int C,
                                                                 float eps, int kind) {  // 0 rms, 1 layer, 2 softmax
    pdl_wait();
    const int lane = threadIdx.x & 31, r = blockIdx.x * (kNormThreads / 32) + (threadIdx.x >> 5);
    if (r >= rows) return;
    const float* xr = x + int64_t(r) * xs;
    float* yr = y + int64_t(r) * ys;
    if (kind == 2) {
        float mx = -INFINITY;
#pragma unroll 4
        for (int c = lane; c < C; c += 32) mx = fmaxf(mx, xr[c]);
        mx = warp_max(mx);
        float s = 0.0f;
#pragma unroll 4
        for (int c = lane; c < C; c += 32) s += expf(xr[c] - mx);
        const float inv = 1.0f / warp_sum(s);
        pdl_trigger();
#pragma unroll 4
        for (int c = lane; c < C; c += 32) yr[c] = expf(xr[c] - mx) * inv;
        return;
    }
    double s1 = 0.0, s2 = 0.0;
#pragma unroll 4
    for (int c = lane; c < C; c += 32) {
        const float v = xr[c];
        s1 += v;
        s2 += double(v) * v;
    }
    float rs, m = 0.0f;
    if (kind == 0) {
        rs = float(1.0 / sqrt(warp_sum_d(s2) / C + double(eps)));
    } else {
        const double mean = warp_sum_d(s1) / C;
        double var = 0.0;
#pragma unroll 4
    #pragma unroll 4
    for (int c = lane; c < C; c += 32) {
            const double d = xr[c] - mean;
            var += d * d;
        }
        rs = float(1.0 / sqrt(warp_sum_d(var) / C + double(eps)));
        m = float(mean);
    }
    pdl_trigger();
#pragma unroll 4
    for (int c = lane; c < C; c += 32) {
        const float v = xr[c];
        yr[c] = kind == 0 ? __fmul_rn(__fmul_rn(v, rs), g[c])
                          : __fadd_rn(__fmul_rn(__fmul_rn(__fsub_rn(v, m), rs), g[c]), b[c]);
    }
}

// Rows wider than the row cache, sms or more of them: a thread-block cluster of CL CTAs per row, each caching its
// chunk (at most kRowCacheFloats) in shared memory; the chunks' partial statistics go through distributed shared
// memory and every CTA sums them in rank order (deterministic), so x is read from memory once. kind: 0 RMSNorm,
// 1 LayerNorm (mean, then the centred sum of squares), 2 softmax (max, then the float sum of exp(x - max)).
__device__ __forceinline__ float block_max_f(float v, float* red) {
    v = warp_max(v);
    const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
    __syncthreads();
    if (l == 0) red[w] = v;
    __syncthreads();
    v = l < kNormThreads / 32 ? red[l] : -INFINITY;
    return warp_max(v);
}

__global__ void __launch_bounds__(kNormThreads) rows_cluster_kernel(const float* __restrict__ x, int64_t xs,
                                                                    float* __restrict__ y, int64_t ys,
                                                                    const float* __restrict__ g,
                                                                    const float* __restrict__ b, int C, int chunk,
                                                                    float eps, int kind, int bulk) {
    namespace cg = cooperative_groups;
    extern __shared__ __align__(16) float cache[];
    __shared__ double red[kNormThreads / 32];
    __shared__ float redf[kNormThreads / 32];
    __shared__ double xch[2];  // this CTA's partial of exchange round 0 / 1
    __shared__ __align__(8) uint64_t bar;
    pdl_wait();
    cg::cluster_group cl = cg::this_cluster();
    const int CL = int(cl.num_blocks()), rank = int(cl.block_rank()), r = blockIdx.y;
    const float* xr = x + int64_t(r) * xs;
    float* yr = y + int64_t(r) * ys;
    const int c0 = rank * chunk, n = max(0, min(C, c0 + chunk) - c0);
    // 1. the chunk into shared memory (bulk: one asynchronous copy of n floats, 16-byte aligned, multiple of 4)
    if (bulk) {
        if (threadIdx.x == 0) {
            mbar_init(&bar, 1);
            fence_barrier_init();
            mbar_arrive_expect_tx(&bar, uint32_t(n) * 4u);
            if (n > 0) bulk_g2s(cache, xr + c0, uint32_t(n) * 4u, &bar);
        }
        __syncthreads();
        mbar_wait(&bar, 0);  // bounded; a timeout is recorded
    } else {
#pragma unroll 4
        for (int i = threadIdx.x; i < n; i += kNormThreads) cache[i] = xr[c0 + i];
        __syncthreads();
    }
    // the first partial
    double p1 = 0.0;
    float pm = -INFINITY;
#pragma unroll 4
    for (int i = threadIdx.x; i < n; i += kNormThreads) {
        const float v = cache[i];
        if (kind == 2) pm = fmaxf(pm, v);
        else p1 += kind == 0 ? double(v) * v : double(v);
    }
    if (kind == 2) pm = block_max_f(pm, redf);
    else p1 = block_sum_d(p1, red);
    if (threadIdx.x == 0) xch[0] = kind == 2 ? double(pm) : p1;
    cl.sync();
    // 2. the row's first statistic from every rank's partial, in rank order
    double s0 = kind == 2 ? -INFINITY : 0.0;
    for (int k = 0; k < CL; k++) {
        const double v = *cl.map_shared_rank(&xch[0], k);
        s0 = kind == 2 ? fmax(s0, v) : s0 + v;
    }
    float rs = 0.0f, mean = 0.0f, mx = 0.0f, inv = 0.0f;
    if (kind == 0) {
        rs = float(1.0 / sqrt(s0 / C + double(eps)));
    } else {
        // second partial: centred squares (LayerNorm) or exp sums (softmax)
        const double mu = s0 / C;
        mx = float(s0);
        double p2 = 0.0;
        float ps = 0.0f;
#pragma unroll 4
        for (int i = threadIdx.x; i < n; i += kNormThreads) {
            if (kind == 1) {
                const double d = cache[i] - mu;
                p2 += d * d;
            } else {
                ps += expf(cache[i] - mx);
            }
        }
        if (kind == 1) p2 = block_sum_d(p2, red);
        else ps = block_sum<kNormThreads>(ps, redf);
        if (threadIdx.x == 0) xch[1] = kind == 1 ? p2 : double(ps);
        cl.sync();
        if (kind == 1) {
            double v2 = 0.0;
            for (int k = 0; k < CL; k++) v2 += *cl.map_shared_rank(&xch[1], k);
            rs = float(1.0 / sqrt(v2 / C + double(eps)));
            mean = float(mu);
        } else {
            float t = 0.0f;
            for (int k = 0; k < CL; k++) t += float(*cl.map_shared_rank(&xch[1], k));
            inv = 1.0f / t;
        }
    }
    // reads of the peers' partials are done: arrive now, wait before leaving (a peer may still read ours)
    cl.barrier_arrive();
    pdl_trigger();
    auto out = [&](float v, int c) {
        return kind == 0   ? __fmul_rn(__fmul_rn(v, rs), g[c])
               : kind == 1 ? __fadd_rn(__fmul_rn(__fmul_rn(__fsub_rn(v, mean), rs), g[c]), b[c])
                           : expf(v - mx) * inv;
    };
    if (bulk) {  // y rows are 16-byte aligned too (the host checks): float4 stores
        for (int i = 4 * threadIdx.x; i < n; i += 4 * kNormThreads) {
            const float4 v = *reinterpret_cast<const float4*>(cache + i);
            const int c = c0 + i;
            *reinterpret_cast<float4*>(yr + c) = make_float4(out(v.x, c), out(v.y, c + 1), out(v.z, c + 2), out(v.w, c + 3));
        }
    } else {
        for (int i = threadIdx.x; i < n; i += kNormThreads) yr[c0 + i] = out(cache[i], c0 + i);
    }
    cl.barrier_wait();
}

// Wide rows, few of them (the LM-head width at 1..sms rows): one CTA per row leaves most SMs idle, so each row is
// split into S chunks over CTAs across the GPU, in two kernels: per-chunk partial statistics (RMS: the sum of
// squares in double; softmax: the chunk's max and float sum of exp(x - max)), then every chunk CTA combines its
// row's partials in chunk order (deterministic) and writes its outputs. The second pass re-reads x from L2.
__global__ void __launch_bounds__(kNormThreads) wide_partial_kernel(const float* __restrict__ x, int64_t xs, int C,
                                                                    int chunk, int softmax, double* __restrict__ part) {
    __shared__ double red[kNormThreads / 32];
    __shared__ float redf[kNormThreads / 32];
    pdl_wait();
    const int j = blockIdx.x, r = blockIdx.y, S = gridDim.x;
    const float* xr = x + int64_t(r) * xs;
    const int c0 = j * chunk, c1 = min(C, c0 + chunk);
    double* pr = part + (int64_t(r) * S + j) * 2;
    if (!softmax) {
        double s2 = 0.0;
#pragma unroll 4
        for (int c = c0 + threadIdx.x; c < c1; c += kNormThreads) {
            const float v = xr[c];
            s2 += double(v) * v;
        }
        s2 = block_sum_d(s2, red);
        if (threadIdx.x == 0) pr[0] = s2;
    } else {
        float mx = -INFINITY;
#pragma unroll 4
        for (int c = c0 + threadIdx.x; c < c1; c += kNormThreads) mx = fmaxf(mx, xr[c]);
        mx = warp_max(mx);
        const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
        if (l == 0) redf[w] = mx;
        __syncthreads();
        mx = l < kNormThreads / 32 ? redf[l] : -INFINITY;
        mx = warp_max(mx);
        float sum = 0.0f;
#pragma unroll 4
        for (int c = c0 + threadIdx.x; c < c1; c += kNormThreads) sum += expf(xr[c] - mx);
        sum = block_sum<kNormThreads>(sum, redf);
        if (threadIdx.x == 0) {
            pr[0] = mx;
            pr[1] = sum;
        }
    }
    pdl_trigger();
}

__global__ void __launch_bounds__(kNormThreads) wide_apply_kernel(const float* __restrict__ x, int64_t xs,
                                                                  float* __restrict__ y, int64_t ys,
                                                                  const float* __restrict__ g, int C, int chunk,
                                                                  int softmax, float eps,
                                                                  const double* __restrict__ part) {
    __shared__ float stat[2];
    pdl_wait();
    const int j = blockIdx.x, r = blockIdx.y, S = gridDim.x;
    const double* pr = part + int64_t(r) * S * 2;
    if (threadIdx.x < 32) {  // the row statistic from its S partials: lanes take chunks l, l + 32, ... in order
        const int l = threadIdx.x;
        if (!softmax) {
            double t = 0.0;
            for (int k = l; k < S; k += 32) t += pr[2 * k];
            t = warp_sum_d(t);
            if (l == 0) stat[0] = float(1.0 / sqrt(t / C + double(eps)));
        } else {
            float M = -INFINITY;
            for (int k = l; k < S; k += 32) M = fmaxf(M, float(pr[2 * k]));
            M = warp_max(M);
            float t = 0.0f;
            for (int k = l; k < S; k += 32) t += float(pr[2 * k + 1]) * expf(float(pr[2 * k]) - M);
            t = warp_sum(t);
            if (l == 0) {
                stat[0] = M;
                stat[1] = 1.0f / t;
            }
        }
    }
    __syncthreads();
    pdl_trigger();
    const float* xr = x + int64_t(r) * xs;
    float* yr = y + int64_t(r) * ys;
    const int c0 = j * chunk, c1 = min(C, c0 + chunk);
    if (!softmax) {
        const float rs = stat[0];
#pragma unroll 4
        for (int c = c0 + threadIdx.x; c < c1; c += kNormThreads) yr[c] = __fmul_rn(__fmul_rn(xr[c], rs), g[c]);
    } else {
        const float M = stat[0], inv = stat[1];
#pragma unroll 4
        for (int c = c0 + threadIdx.x; c < c1; c += kNormThreads) yr[c] = expf(xr[c] - M) * inv;
    }
}

// First index of the maximum of each row (std::max_element: strict '<' keeps the earliest).
__global__ void __launch_bounds__(kNormThreads) argmax_kernel(const float* __restrict__ x, int64_t stride, int C,
                                                              int* __restrict__ out) {
    __shared__ float bv[kNormThreads / 32];
    __shared__ int bi[kNormThreads / 32];
    pdl_wait();
    const float* xr = x + int64_t(blockIdx.x) * stride;
    float v = -INFINITY;
    int idx = 0x7fffffff;
    for (int c = threadIdx.x; c < C; c += blockDim.x) {
        const float t = xr[c];
        if (t > v) {  // strided scan visits increasing c, so '>' keeps this thread's first maximum
            v = t;
            idx = c;
        }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, v, o);
        const int oi = __shfl_xor_sync(0xffffffffu, idx, o);
        if (ov > v || (ov == v && oi < idx)) {
            v = ov;
            idx = oi;
        }
    }
    const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
    if (l == 0) {
        bv[w] = v;
        bi[w] = idx;
    }
    __syncthreads();
    if (w == 0) {
        v = l < kNormThreads / 32 ? bv[l] : -INFINITY;
        idx = l < kNormThreads / 32 ? bi[l] : 0x7fffffff;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, v, o);
            const int oi = __shfl_xor_sync(0xffffffffu, idx, o);
            if (ov > v || (ov == v && oi < idx)) {
                v = ov;
                idx = oi;
            }
        }
        if (l == 0) out[blockIdx.x] = idx == 0x7fffffff ? 0 : idx;
    }
}

// cpu::siluMul (cpu_ops.cpp:526-533) / silu_mul.comp.
__global__ void silu_mul_kernel(const float* __restrict__ h, float* __restrict__ g, int T, int I) {
    const int64_t idx = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
    if (idx >= int64_t(T) * I) return;
    const int t = int(idx / I), i = int(idx % I);
    const float a = h[int64_t(t) * 2 * I + i];
    const float b = h[int64_t(t) * 2 * I + I + i];
    g[idx] = a / (1.0f + expf(-a)) * b;
}

// embed.comp + QMatrix::dequantizeRow for the token rows (+ position row).
__global__ void embed_kernel(const int* __restrict__ tokens, int T, int C, int fmt, const uint8_t* __restrict__ table,
                             int64_t rb, int row_base, int nrows, const uint16_t* __restrict__ wpe16,
                             const float* __restrict__ wpe32, int pos0, const int* __restrict__ pos_arr,
                             float* __restrict__ x) {
    pdl_wait();
    const int t = blockIdx.y;
    const int c = blockIdx.x * blockDim.x + threadIdx.x;
    if (t >= T || c >= C) return;
    const int row = tokens[t] - row_base;
    if (row < 0 || row >= nrows) return;
    float v = dequant_one(fmt, table + int64_t(row) * rb, C, c);
    const int pos = pos_arr ? pos_arr[t] : pos0 + t;
    if (wpe16) v += half_bits_to_float(wpe16[int64_t(pos) * C + c]);
    if (wpe32) v += wpe32[int64_t(pos) * C + c];
    x[int64_t(t) * C + c] = v;
}

// kv_store.comp: K, V rows of qkv (f32) -> f16 caches [ctx][W] at pos0 + t (cpu::storeKv, cpu_ops.cpp:535-542).
__global__ void kv_store_kernel(const float* __restrict__ qkv, int T, int W, int pos0, int stride, int k_off,
                                int v_off, uint16_t* __restrict__ kc, uint16_t* __restrict__ vc) {
    const int t = blockIdx.y;
    const int c = blockIdx.x * blockDim.x + threadIdx.x;
    if (t >= T || c >= W) return;
    const float* src = qkv + int64_t(t) * stride;
    const int64_t dst = int64_t(pos0 + t) * W + c;
    kc[dst] = __half_as_ushort(__float2half_rn(src[k_off + c]));
    vc[dst] = __half_as_ushort(__float2half_rn(src[v_off + c]));
}

// Per-head QK RMSNorm (cpu::rmsNorm over hd, qwen3_model.cpp:249-252), NeoX rotation from the host table
// (cpu::rope, cpu_ops.cpp:513-524) and the f16 KV store (cpu::storeKv), one warp per head. Heads
// [0, H) are queries (rotated in place), [H, H + KV) keys and [H + KV, H + 2 KV) values (both stored).
constexpr int kPostWarps = 4;
__global__ void __launch_bounds__(kPostWarps * 32) qkv_post_kernel(const QkvPostArgs a) {
    __shared__ float buf[kPostWarps][256];
    pdl_wait();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int head = blockIdx.x * kPostWarps + warp;
    const int r = blockIdx.y;
    const int heads_total = a.n_head + (a.store_kv ? 2 : 1) * a.n_kv;
    if (head >= heads_total || r >= a.rows) return;
    const int hd = a.hd;
    const bool is_q = head < a.n_head, is_k = !is_q && head < a.n_head + a.n_kv;
    float* row = a.qkv + int64_t(r) * a.qkv_stride;
    const int col = is_q ? head * hd : is_k ? a.k_off + (head - a.n_head) * hd
                                             : a.v_off + (head - a.n_head - a.n_kv) * hd;
    const int pos = a.row_pos ? a.row_pos[r] : a.pos0 + r;
    if (pos < 0 || pos >= a.pos_limit) {  // a cache row outside the context: report, never write it
        if (lane == 0) set_device_error(kErrBadIndex);
        return;
    }
    float* v = buf[warp];
    double ss = 0.0;
    for (int d = lane; d < hd; d += 32) {
        const float t = row[col + d];
        v[d] = t;
        ss += double(t) * t;
    }
    __syncwarp();
    if (!is_q && !is_k) {  // value head: store only
        const int slot = a.row_slot ? a.row_slot[r] : a.slot0;
        uint16_t* dst = a.vc + slot * a.slot_stride + int64_t(pos) * a.pos_stride +
                        int64_t(head - a.n_head - a.n_kv) * a.head_stride;
        for (int d = lane; d < hd; d += 32) dst[d] = __half_as_ushort(__float2half_rn(v[d]));
        return;
    }
    if (a.do_norm) {
        ss = warp_sum_d(ss);
        const float s = float(1.0 / sqrt(ss / hd + double(a.eps)));
        const float* w = a.wn + (is_q ? 0 : hd);
        for (int d = lane; d < hd; d += 32) v[d] = __fmul_rn(__fmul_rn(v[d], s), w[d]);
        __syncwarp();
    }
    const int half = hd / 2;
    if (a.do_rope && (is_q || a.rope_kv_heads)) {
        const float* cs = a.cs + int64_t(pos) * hd;
        // Lane l owns the pairs (i, i + half) with i = l (mod 32): no element is shared between lanes.
        for (int i = lane; i < half; i += 32) {
            const float c = cs[2 * i], sn = cs[2 * i + 1];
            const float x0 = v[i], x1 = v[i + half];
            v[i] = __fsub_rn(__fmul_rn(x0, c), __fmul_rn(x1, sn));
            v[i + half] = __fadd_rn(__fmul_rn(x0, sn), __fmul_rn(x1, c));
        }
        __syncwarp();
    }
    if (is_q || !a.store_kv || a.write_back_k) {
        for (int d = lane; d < hd; d += 32) row[col + d] = v[d];
    }
    if (is_k && a.store_kv) {
        const int slot = a.row_slot ? a.row_slot[r] : a.slot0;
        uint16_t* dst = a.kc + slot * a.slot_stride + int64_t(pos) * a.pos_stride +
                        int64_t(head - a.n_head) * a.head_stride;
        for (int d = lane; d < hd; d += 32) dst[d] = __half_as_ushort(__float2half_rn(v[d]));
    }
}

}  // namespace

// The row-cache shared-memory limit of a norm / softmax kernel on the current device (function attributes are
// per device), set once per (kernel, device).
template <typename K>
cudaError_t row_cache_attr(K kernel) {
    static unsigned done[2] = {0u, 0u};  // bit d: device d (< 32) done; [0] norm, [1] softmax
    const int which = reinterpret_cast<const void*>(kernel) == reinterpret_cast<const void*>(norm_kernel) ? 0 : 1;
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 32 && ((done[which] >> dev) & 1u)) return cudaSuccess;
    const cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kRowCacheFloats * 4);
    if (e == cudaSuccess && dev < 32) done[which] |= 1u << dev;
    return e;
}

cudaError_t launch_rows_cluster(const float* x, int64_t xs, float* y, int64_t ys, const float* g, const float* b,
                                int rows, int C, float eps, int kind, cudaStream_t st, bool pdl);

cudaError_t launch_norm(const float* x, int64_t x_stride, float* y, int64_t y_stride, const float* gamma,
                        const float* beta, int rows, int C, float eps, bool rms, cudaStream_t st, bool pdl) {
    if (rows <= 0) return cudaSuccess;
    // many narrow rows: a warp per row (measured at 4096 rows: C = 1024 / 2048 / 2560 25.6 / 39.9 / 46.1 -> 16.4 /
    // 26.6 / 30.8 us); few rows keep a CTA per row (one row of 2560: 15 vs 25 us)
    if (C <= kWarpRowMaxC && rows >= 2 * num_sms())
        return launch_ex(rows_warp_kernel, dim3((rows + kNormThreads / 32 - 1) / (kNormThreads / 32)),
                         dim3(kNormThreads), 0, st, pdl, x, x_stride, y, y_stride, gamma, beta, rows, C, eps,
                         rms ? 0 : 1);
    if (cudaError_t e = launch_rows_cluster(x, x_stride, y, y_stride, gamma, beta, rows, C, eps, rms ? 0 : 1, st, pdl);
        e != cudaErrorNotSupported)
        return e;
    const size_t smem = C <= kRowCacheFloats ? size_t(C) * 4 : 0;
    if (cudaError_t e = row_cache_attr(norm_kernel); e != cudaSuccess) return e;
    return launch_ex(norm_kernel, dim3(rows), dim3(kNormThreads), smem, st, pdl, x, x_stride, y, y_stride, gamma, beta,
                     C, eps, rms ? 1 : 0);
}

int wide_row_chunks(int rows, int C) {
    if (rows <= 0 || C < kWideRowMinC || rows >= num_sms()) return 0;
    // about two CTAs per SM over the rows' chunks, each chunk at least 512 columns
    return std::max(1, std::min((2 * num_sms() + rows - 1) / rows, C / 512));
}

cudaError_t launch_wide_rows(const float* x, int64_t x_stride, float* y, int64_t y_stride, const float* gamma,
                             int rows, int C, float eps, bool softmax, double* part, int S, cudaStream_t st) {
    if (rows <= 0) return cudaSuccess;
    if (S <= 0 || !part) return cudaErrorInvalidValue;
    const int chunk = (C + S - 1) / S;
    if (cudaError_t e = launch_ex(wide_partial_kernel, dim3(S, rows), dim3(kNormThreads), 0, st, false, x, x_stride,
                                  C, chunk, softmax ? 1 : 0, part);
        e != cudaSuccess)
        return e;
    return launch_ex(wide_apply_kernel, dim3(S, rows), dim3(kNormThreads), 0, st, true, x, x_stride, y, y_stride,
                     gamma, C, chunk, softmax ? 1 : 0, eps, static_cast<const double*>(part));
}

// Cluster per row for rows wider than the row cache (up to 8 x kRowCacheFloats); cudaErrorNotSupported otherwise.
cudaError_t launch_rows_cluster(const float* x, int64_t xs, float* y, int64_t ys, const float* g, const float* b,
                                int rows, int C, float eps, int kind, cudaStream_t st, bool pdl) {
    const int CL = (C + kRowCacheFloats - 1) / kRowCacheFloats;
    if (C <= kRowCacheFloats || CL > 8 || rows > 65535) return cudaErrorNotSupported;
    const int chunk = ((C + CL - 1) / CL + 3) / 4 * 4;  // a multiple of 4, at most kRowCacheFloats
    const auto al16 = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; };
    const int bulk = C % 4 == 0 && xs % 4 == 0 && ys % 4 == 0 && al16(x) && al16(y) ? 1 : 0;
    static unsigned done = 0u;  // bit d: device d (< 32); function attributes are per device
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 32 || !((done >> dev) & 1u)) {
        if (cudaError_t e = cudaFuncSetAttribute(rows_cluster_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                 kRowCacheFloats * 4);
            e != cudaSuccess)
            return e;
        if (dev < 32) done |= 1u << dev;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(CL, rows);
    cfg.blockDim = dim3(kNormThreads);
    cfg.dynamicSmemBytes = size_t(chunk) * 4;
    cfg.stream = st;
    cudaLaunchAttribute attr[2];
    int na = 0;
    attr[na].id = cudaLaunchAttributeClusterDimension;
    attr[na].val.clusterDim.x = CL;
    attr[na].val.clusterDim.y = 1;
    attr[na].val.clusterDim.z = 1;
    na++;
    if (pdl) {
        attr[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[na].val.programmaticStreamSerializationAllowed = 1;
        na++;
    }
    cfg.attrs = attr;
    cfg.numAttrs = na;
    return cudaLaunchKernelEx(&cfg, rows_cluster_kernel, x, xs, y, ys, g, b, C, chunk, eps, kind, bulk);
}

cudaError_t launch_softmax(const float* x, float* y, int rows, int C, cudaStream_t st) {
    if (rows <= 0) return cudaSuccess;
    // a warp per row only for many rows of at most 1024 (wider rows: the CTA kernel's float4 loads and row cache
    // measured faster, 2048 wide x 4096 rows 25.6 vs 28.7 us)
    if (C <= 1024 && rows >= 2 * num_sms())
        return launch_ex(rows_warp_kernel, dim3((rows + kNormThreads / 32 - 1) / (kNormThreads / 32)),
                         dim3(kNormThreads), 0, st, false, x, int64_t(C), y, int64_t(C), static_cast<const float*>(nullptr),
                         static_cast<const float*>(nullptr), rows, C, 0.0f, 2);
    if (cudaError_t e = launch_rows_cluster(x, C, y, C, nullptr, nullptr, rows, C, 0.0f, 2, st, false);
        e != cudaErrorNotSupported)
        return e;
    const size_t smem = C <= kRowCacheFloats ? size_t(C) * 4 : 0;
    if (cudaError_t e = row_cache_attr(softmax_kernel); e != cudaSuccess) return e;
    softmax_kernel<<<rows, kNormThreads, smem, st>>>(x, y, C);
    return cudaGetLastError();
}

cudaError_t launch_argmax(const float* x, int64_t stride, int rows, int C, int* out, cudaStream_t st, bool pdl) {
    if (rows <= 0) return cudaSuccess;
    return launch_ex(argmax_kernel, dim3(rows), dim3(kNormThreads), 0, st, pdl, x, stride, C, out);
}

cudaError_t launch_silu_mul(const float* h, float* g, int T, int I, cudaStream_t st) {
    const int64_t n = int64_t(T) * I;
    if (n <= 0) return cudaSuccess;
    silu_mul_kernel<<<unsigned((n + 255) / 256), 256, 0, st>>>(h, g, T, I);
    return cudaGetLastError();
}

cudaError_t launch_embed(const int* tokens, int T, int C, int fmt, const uint8_t* table, int64_t rb, int row_base,
                         int nrows, const uint16_t* wpe16, const float* wpe32, int pos0, const int* pos_arr, float* x,
                         cudaStream_t st, bool pdl) {
    if (T <= 0 || C <= 0) return cudaSuccess;
    return launch_ex(embed_kernel, dim3((C + 255) / 256, T), dim3(256), 0, st, pdl, tokens, T, C, fmt, table, rb,
                     row_base, nrows, wpe16, wpe32, pos0, pos_arr, x);
}

cudaError_t launch_kv_store(const float* qkv, int T, int W, int pos0, int stride, int k_off, int v_off, uint16_t* kc,
                            uint16_t* vc, cudaStream_t st) {
    if (T <= 0 || W <= 0) return cudaSuccess;
    kv_store_kernel<<<dim3((W + 127) / 128, T), 128, 0, st>>>(qkv, T, W, pos0, stride, k_off, v_off, kc, vc);
    return cudaGetLastError();
}

cudaError_t launch_qkv_post(const QkvPostArgs& a, cudaStream_t st, bool pdl) {
    if (a.rows <= 0) return cudaSuccess;
    if (a.hd > 256 || (a.hd & 1)) return cudaErrorInvalidValue;
    const int heads = a.n_head + (a.store_kv ? 2 : 1) * a.n_kv;
    return launch_ex(qkv_post_kernel, dim3((heads + kPostWarps - 1) / kPostWarps, a.rows), dim3(kPostWarps * 32), 0,
                     st, pdl, a);
}

}  // namespace neko
