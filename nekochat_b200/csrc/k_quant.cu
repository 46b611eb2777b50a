// Weight codec on the GPU: quantizeMatrix (app/architecture/shared/cpp/quant.cpp:255-279) and
// QMatrix::dequantizeRow (quant.cpp:230-253), byte-identical to the engine's CPU code.
//
// One thread owns one 32-weight block. Every float operation uses an explicit _rn intrinsic so the compiler
// cannot fuse or reorder it: the results must match the CPU reference bit for bit (the reference is built
// without FMA contraction). Loads are strided (each thread walks its own 128-byte block); this runs once at
// model load and is far from the decode path.
#include "neko_common.cuh"
#include "neko_internal.h"

namespace neko {

namespace {

__device__ __forceinline__ uint16_t f2h_bits(float f) { return __half_as_ushort(__float2half_rn(f)); }
__device__ __forceinline__ float h2f(uint16_t b) { return __half2float(__ushort_as_half(b)); }

// E4M3 encode (quant.cpp:43-49): round y/256 to f16, then round the f16 pattern's 7 low mantissa bits away
// (ties to even) and clamp to 0x7E.
__device__ __forceinline__ uint8_t enc_fp8(float y) {
    uint32_t h = f2h_bits(__fmul_rn(y, 1.0f / 256.0f));
    uint32_t mag = h & 0x7fffu;
    uint32_t c = (mag + 0x3fu + ((mag >> 7) & 1u)) >> 7;
    c = c > 0x7eu ? 0x7eu : c;
    return uint8_t(c | ((h >> 8) & 0x80u));
}

// E2M1 encode by midpoint thresholds (quant.cpp:57-61).
__device__ __forceinline__ uint32_t enc_fp4(float y) {
    float a = fabsf(y);
    int c = (a > 0.25f) + (a > 0.75f) + (a > 1.25f) + (a > 1.75f) + (a > 2.5f) + (a > 3.5f) + (a > 5.0f);
    return c == 0 ? 0u : uint32_t(c | (y < 0.0f ? 8 : 0));
}

__device__ __forceinline__ float fp4_round(float a) {  // quant.cpp:93-97 (nearbyint = round half even)
    if (a < 1.75f) return __fmul_rn(rintf(__fmul_rn(a, 2.0f)), 0.5f);
    if (a < 3.5f) return rintf(a);
    return a < 5.0f ? 4.0f : 6.0f;
}

struct Fit {
    float err, xr, rr;
};

__device__ __forceinline__ Fit fit_fp4(const float* ax, float s) {  // scalar fitFp4, quant.cpp:126-136
    Fit f{0.0f, 0.0f, 0.0f};
    const float inv = __fdiv_rn(1.0f, s);
#pragma unroll 4
    for (int i = 0; i < kQuantBlock; i++) {
        float r = fp4_round(__fmul_rn(ax[i], inv));
        float d = __fsub_rn(ax[i], __fmul_rn(r, s));
        f.err = __fadd_rn(f.err, __fmul_rn(d, d));
        f.xr = __fadd_rn(f.xr, __fmul_rn(ax[i], r));
        f.rr = __fadd_rn(f.rr, __fmul_rn(r, r));
    }
    return f;
}

// Reads the 32 inputs of block b of output row r. transpose: w is [cols][rows] (Conv1D), each value rounded to
// f16 first (Gpt2Model::conv1d, gpt2_model.cpp:78-82, goes through TensorStore::toF16).
__device__ __forceinline__ void load_block(const float* w, int64_t ld, int r, int b, bool transpose, float* x) {
#pragma unroll 8
    for (int i = 0; i < kQuantBlock; i++) {
        const int c = b * kQuantBlock + i;
        x[i] = transpose ? h2f(f2h_bits(w[int64_t(c) * ld + r])) : w[int64_t(r) * ld + c];
    }
}

__global__ void quantize_kernel(int fmt, const float* __restrict__ w, int rows, int cols, int64_t ld, int transpose,
                                uint8_t* __restrict__ out) {
    const int nb = cols / kQuantBlock;
    const int64_t idx = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
    if (idx >= int64_t(rows) * nb) return;
    const int r = int(idx / nb), b = int(idx % nb);
    const int64_t rb = row_bytes(fmt, cols);
    uint8_t* row = out + int64_t(r) * rb;
    float x[kQuantBlock];
    load_block(w, ld, r, b, transpose != 0, x);
    float amax = 0.0f;
#pragma unroll
    for (int i = 0; i < kQuantBlock; i++) amax = fmaxf(amax, fabsf(x[i]));
    uint16_t s;
    if (fmt == kFP8) {
        // blockScale (quant.cpp:72-79) + quantizeRowFp8 (:81-91)
        s = f2h_bits(__fdiv_rn(amax, 448.0f));
        const float sv = h2f(s);
        const float inv = sv > 0.0f ? __fdiv_rn(1.0f, sv) : 0.0f;
        s = sv > 0.0f ? s : uint16_t(0);
        uint32_t packed[8];
#pragma unroll
        for (int q = 0; q < 8; q++) {
            packed[q] = 0;
#pragma unroll
            for (int k = 0; k < 4; k++) packed[q] |= uint32_t(enc_fp8(__fmul_rn(x[4 * q + k], inv))) << (8 * k);
        }
        uint4* dst = reinterpret_cast<uint4*>(row + b * kQuantBlock);
        dst[0] = make_uint4(packed[0], packed[1], packed[2], packed[3]);
        dst[1] = make_uint4(packed[4], packed[5], packed[6], packed[7]);
    } else {
        // fp4BlockScale (quant.cpp:142-165) + quantizeRowFp4 (:167-178)
        uint16_t best = f2h_bits(__fdiv_rn(amax, 6.0f));
        if (!(h2f(best) > 0.0f)) {
            best = 0;
        } else {
            float ax[kQuantBlock];
#pragma unroll
            for (int i = 0; i < kQuantBlock; i++) ax[i] = fabsf(x[i]);
            Fit fit = fit_fp4(ax, h2f(best));
            float bestErr = fit.err;
            for (int it = 0; it < 2 && fit.rr > 0.0f; it++) {
                const uint16_t cand = f2h_bits(__fdiv_rn(fit.xr, fit.rr));
                if (!(h2f(cand) > 0.0f) || cand == best) break;
                fit = fit_fp4(ax, h2f(cand));
                if (fit.err >= bestErr) break;
                bestErr = fit.err;
                best = cand;
            }
        }
        s = best;
        const float inv = s ? __fdiv_rn(1.0f, h2f(s)) : 0.0f;
        uint32_t packed[4];
#pragma unroll
        for (int q = 0; q < 4; q++) {
            packed[q] = 0;
#pragma unroll
            for (int k = 0; k < 4; k++) {
                const int j = 4 * q + k;
                const uint32_t byte = enc_fp4(__fmul_rn(x[j], inv)) | (enc_fp4(__fmul_rn(x[16 + j], inv)) << 4);
                packed[q] |= byte << (8 * k);
            }
        }
        *reinterpret_cast<uint4*>(row + b * 16) = make_uint4(packed[0], packed[1], packed[2], packed[3]);
    }
    uint16_t* scales = reinterpret_cast<uint16_t*>(row + scale_offset(fmt, cols));
    scales[b] = s;
    if (b == 0) {  // zero the scale padding (quantizeMatrix zero-fills the whole buffer)
        const int pad_end = int((rb - scale_offset(fmt, cols)) / 2);
        for (int p = nb; p < pad_end; p++) scales[p] = 0;
    }
}

// rowToHalf (quant.cpp:180-186): the F16 "format" of matrices whose width is not a multiple of 32.
__global__ void to_half_kernel(const float* __restrict__ w, int rows, int cols, int64_t ld, int transpose,
                               uint16_t* __restrict__ out) {
    const int64_t idx = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
    if (idx >= int64_t(rows) * cols) return;
    const int r = int(idx / cols), c = int(idx % cols);
    const float v = transpose ? w[int64_t(c) * ld + r] : w[int64_t(r) * ld + c];
    out[idx] = f2h_bits(v);
}

__global__ void dequantize_kernel(int fmt, const uint8_t* __restrict__ q, int rows, int cols, float* __restrict__ out) {
    const int64_t idx = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
    if (idx >= int64_t(rows) * cols) return;
    const int r = int(idx / cols), c = int(idx % cols);
    out[idx] = dequant_one(fmt, q + int64_t(r) * row_bytes(fmt, cols), cols, c);
}

}  // namespace

cudaError_t launch_quantize(int fmt, const float* w, int rows, int cols, int64_t ld, int transpose, uint8_t* out,
                            cudaStream_t st) {
    if (rows <= 0 || cols <= 0) return cudaSuccess;
    if (fmt == kF16) {
        const int64_t n = int64_t(rows) * cols;
        to_half_kernel<<<unsigned((n + 255) / 256), 256, 0, st>>>(w, rows, cols, ld, transpose,
                                                                   reinterpret_cast<uint16_t*>(out));
    } else {
        const int64_t n = int64_t(rows) * (cols / kQuantBlock);
        quantize_kernel<<<unsigned((n + 127) / 128), 128, 0, st>>>(fmt, w, rows, cols, ld, transpose, out);
    }
    return cudaGetLastError();
}

cudaError_t launch_dequantize(int fmt, const uint8_t* q, int rows, int cols, float* out, cudaStream_t st) {
    const int64_t n = int64_t(rows) * cols;
    if (n <= 0) return cudaSuccess;
    dequantize_kernel<<<unsigned((n + 255) / 256), 256, 0, st>>>(fmt, q, rows, cols, out);
    return cudaGetLastError();
}

}  // namespace neko
