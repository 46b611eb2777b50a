// FP8 (E4M3) checkpoint weights to f32 on the device, as TensorStore::rows reads them (tensor_store.cpp:543-571):
// each byte is an OCP E4M3 ("e4m3fn") code, exponent bias 7, no infinities and no NaN code (0x7F / 0xFF decode
// to +-480, as the reference's table has them), times the f32 scale of its block; the scale tensor
// ("<name>_scale_inv" or "<name>_scale") is [sR][sC] and a block spans bR x bC elements, 128 x 128 for
// DeepSeek / Qwen FP8 checkpoints, else the shape split evenly (fp8_block_of below). The product is one f32
// multiply, as on the CPU, so the result is bit-identical to the reference's rows.
// One launch per weight at load time: 1 byte read + 4 bytes written per element (HBM-bound); four codes per
// thread when the rows are 4-byte aligned.
#include <cstdint>

#include "neko_common.cuh"
#include "neko_internal.h"

namespace neko {

namespace {

// (1 + m/8) * 2^(e-7) = (8 + m) * 2^(e-10) for e >= 1, m/8 * 2^-6 = m * 2^-9 for e == 0: both products are exact
// in f32, so this equals the reference's std::ldexp table entry for every code.
__device__ __forceinline__ float e4m3fn_value(uint32_t c) {
    const uint32_t e = (c >> 3) & 15u, mt = c & 7u;
    const float mag = e == 0 ? float(mt) * 0x1p-9f : float(8u + mt) * __uint_as_float((e + 117u) << 23);
    return (c & 0x80u) ? -mag : mag;
}

template <bool V4>
__global__ void fp8_block_dequant_kernel(const uint8_t* __restrict__ codes, int64_t rows, int64_t cols,
                                         const float* __restrict__ scales, int64_t sR, int64_t sC, int64_t bR,
                                         int64_t bC, float* __restrict__ out) {
    const int64_t per_row = V4 ? cols / 4 : cols;
    const int64_t n = rows * per_row;
    for (int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += int64_t(gridDim.x) * blockDim.x) {
        const int64_t r = i / per_row, c0 = (i - r * per_row) * (V4 ? 4 : 1);
        const float* srow = scales + min(r / bR, sR - 1) * sC;
        if constexpr (V4) {
            const uint32_t q = reinterpret_cast<const uint32_t*>(codes + r * cols)[c0 / 4];
            float4 v;
            v.x = __fmul_rn(e4m3fn_value(q & 255u), srow[min(c0 / bC, sC - 1)]);
            v.y = __fmul_rn(e4m3fn_value((q >> 8) & 255u), srow[min((c0 + 1) / bC, sC - 1)]);
            v.z = __fmul_rn(e4m3fn_value((q >> 16) & 255u), srow[min((c0 + 2) / bC, sC - 1)]);
            v.w = __fmul_rn(e4m3fn_value(q >> 24), srow[min((c0 + 3) / bC, sC - 1)]);
            reinterpret_cast<float4*>(out + r * cols)[c0 / 4] = v;
        } else {
            out[r * cols + c0] = __fmul_rn(e4m3fn_value(codes[r * cols + c0]), srow[min(c0 / bC, sC - 1)]);
        }
    }
}

}  // namespace

// The block length along an axis of n elements split into `parts` scale entries (tensor_store.cpp:550-554).
int64_t fp8_block_of(int64_t n, int64_t parts) {
    if (parts <= 1) return n;
    if ((n + 127) / 128 == parts) return 128;
    return (n + parts - 1) / parts;
}

cudaError_t launch_fp8_block_dequant(const uint8_t* codes, int64_t rows, int64_t cols, const float* scales,
                                     int64_t sR, int64_t sC, float* out, cudaStream_t st) {
    if (rows <= 0 || cols <= 0) return cudaSuccess;
    const int64_t bR = fp8_block_of(rows, sR), bC = fp8_block_of(cols, sC);
    const bool v4 = cols % 4 == 0 && (reinterpret_cast<uintptr_t>(codes) & 3u) == 0 &&
                    (reinterpret_cast<uintptr_t>(out) & 15u) == 0;
    const int64_t work = rows * (v4 ? cols / 4 : cols);
    const int threads = 256;
    const int blocks = int(std::min<int64_t>((work + threads - 1) / threads, int64_t(num_sms()) * 8));
    if (v4)
        fp8_block_dequant_kernel<true><<<blocks, threads, 0, st>>>(codes, rows, cols, scales, sR, sC, bR, bC, out);
    else
        fp8_block_dequant_kernel<false><<<blocks, threads, 0, st>>>(codes, rows, cols, scales, sR, sC, bR, bC, out);
    return cudaGetLastError();
}

}  // namespace neko
