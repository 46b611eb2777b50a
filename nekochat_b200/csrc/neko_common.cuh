// Shared device helpers for the B200 (sm_100a) kernels: the engine's weight-format decoders, warp/block
// reductions, mbarrier + bulk-copy (TMA engine) primitives, programmatic dependent launch (PDL) controls and
// the device-side error word.
#pragma once

#include <cstdint>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

namespace neko {

// Weight formats (quant.h:19 WeightFormat) and matmul flags (gpu/shaders/matmul.comp:5).
enum Fmt : int { kF16 = 0, kFP8 = 1, kFP4 = 2 };
enum MatmulFlag : int { kGelu = 1, kAccumulate = 2, kBias = 4 };
constexpr int kQuantBlock = 32;   // quant.h:23
constexpr float kFp8Factor = 256.0f;    // quant.h:27: code bits read as f16 give value / 256
constexpr float kFp4Factor = 16384.0f;  // quant.h:28: value / 16384

// Row bytes of the engine's packed layout (quant.cpp:199-208): FP8 = K code bytes, FP4 = K/2, then K/32 f16
// scales padded to 16 bytes; F16 = 2K.
__host__ __device__ inline int64_t row_bytes(int fmt, int64_t K) {
    int64_t scales = (K / kQuantBlock * 2 + 15) / 16 * 16;
    return fmt == kF16 ? 2 * K : fmt == kFP8 ? K + scales : K / 2 + scales;
}
__host__ __device__ inline int64_t scale_offset(int fmt, int64_t K) { return fmt == kFP8 ? K : K / 2; }

// ----------------------------------------------------------------------------------------------- errors
// Device-side error word: bounded waits that give up record a code here instead of trapping, and the host
// reads it after every synchronisation (neko_device_error in backend.cu).
enum DeviceError : unsigned {
    kErrNone = 0,
    kErrMbarTimeout = 1,
    kErrBadIndex = 2,
    kErrMisalignedSmem = 3,  // a tensor-copy destination or mbarrier off its required alignment (copies skipped)
    kErrMisalignedMap = 4,   // a tensor map whose address is not 64-byte aligned (copies skipped)
};
extern __device__ unsigned g_device_error;
__device__ inline void set_device_error(unsigned code) { atomicCAS(&g_device_error, 0u, code); }

// ----------------------------------------------------------------------------------------------- decoders
// Engine FP8 (E4M3) codes to f16 the way the format defines them (quant.cpp:51-53): code c becomes the f16
// bit pattern (c & 0x80) << 8 | (c & 0x7F) << 7, i.e. value / 256, exact for every byte (0x7F reads as 480
// like the reference decoder; the encoder never writes it). Bytes 0,2 and 1,3 of q come out as two f16x2.
__device__ __forceinline__ void fp8x4_to_half2(uint32_t q, __half2& even, __half2& odd) {
    uint32_t e = q & 0x00FF00FFu;
    uint32_t o = (q >> 8) & 0x00FF00FFu;
    uint32_t a = (e + (e & 0x00800080u)) << 7;
    uint32_t b = (o + (o & 0x00800080u)) << 7;
    even = *reinterpret_cast<__half2*>(&a);
    odd = *reinterpret_cast<__half2*>(&b);
}

// Engine FP4 (E2M1) nibbles to f16 (quant.cpp:63-65): code c becomes (c & 8) << 12 | (c & 7) << 9, i.e.
// value / 16384. n holds one nibble in bits 0-3 of each 16-bit half.
__device__ __forceinline__ __half2 fp4x2_to_half2(uint32_t n) {
    uint32_t h = ((n & 0x00070007u) << 9) | ((n & 0x00080008u) << 12);
    return *reinterpret_cast<__half2*>(&h);
}

__device__ __forceinline__ float half_bits_to_float(uint16_t b) { return __half2float(__ushort_as_half(b)); }

// Exact dequantised weight (QMatrix::dequantizeRow, quant.cpp:230-253): decode(code) * scale in f32. Both
// factors are exact and their product has at most 15 significant bits, so the f32 result is exact.
__device__ __forceinline__ float dequant_one(int fmt, const uint8_t* row, int K, int c) {
    if (fmt == kF16) return half_bits_to_float(reinterpret_cast<const uint16_t*>(row)[c]);
    const uint16_t* sc = reinterpret_cast<const uint16_t*>(row + scale_offset(fmt, K));
    const int b = c / kQuantBlock, j = c % kQuantBlock;
    const float s = half_bits_to_float(sc[b]);
    uint16_t h;
    float f;
    if (fmt == kFP8) {
        const uint32_t code = row[c];
        h = uint16_t(((code & 0x80u) << 8) | ((code & 0x7Fu) << 7));
        f = half_bits_to_float(h) * kFp8Factor;
    } else {
        const uint32_t byte = row[b * 16 + (j & 15)];
        const uint32_t code = j < 16 ? (byte & 15u) : (byte >> 4);
        h = uint16_t(((code & 8u) << 12) | ((code & 7u) << 9));
        f = half_bits_to_float(h) * kFp4Factor;
    }
    return f * s;
}

// ----------------------------------------------------------------------------------------------- reductions
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// Sum over the block; red must hold one float per warp. Every thread gets the total.
template <int kThreads>
__device__ __forceinline__ float block_sum(float v, float* red) {
    constexpr int kWarps = kThreads / 32;
    v = warp_sum(v);
    const int w = threadIdx.x / 32, l = threadIdx.x % 32;
    __syncthreads();
    if (l == 0) red[w] = v;
    __syncthreads();
    float t = l < kWarps ? red[l] : 0.0f;
    return warp_sum(t);
}

// GPT-2 "gelu_new" (cpu_ops.cpp:20-23). tanhf is CUDA's; the argument is clamped like the shaders
// (matmul.comp:16-19) so it stays finite, which does not change the result beyond |u| = 15.
__device__ __forceinline__ float gelu(float x) {
    float u = 0.7978845608f * (x + 0.044715f * x * x * x);
    u = fminf(fmaxf(u, -15.0f), 15.0f);
    return 0.5f * x * (1.0f + tanhf(u));
}

// ----------------------------------------------------------------------------------------------- PDL
// Programmatic dependent launch: a kernel launched with cudaLaunchAttributeProgrammaticStreamSerialization may
// start while its predecessor is still running. Everything before pdl_wait() must only read data no earlier
// kernel writes (the weights); pdl_wait() returns once the predecessor grid has completed and its writes are
// visible. Without the attribute both are no-ops.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// ----------------------------------------------------------------------------------------------- mbarrier + bulk copy
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
// Makes barrier initialisation visible to the async (bulk-copy) proxy.
__device__ __forceinline__ void fence_barrier_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}
// Bounded wait: each try_wait already suspends for a hardware-chosen time; after kMaxTries the wait gives up,
// records kErrMbarTimeout and returns false so the kernel can leave instead of hanging the GPU.
constexpr uint32_t kMbarMaxTries = 1u << 22;
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity) {
    for (uint32_t i = 0; i < kMbarMaxTries; i++)
        if (mbar_try_wait(bar, parity)) return true;
    set_device_error(kErrMbarTimeout);
    return false;
}

// Global -> shared bulk copy on the TMA engine, completing on bar. dst, src and bytes must be multiples of 16.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}

// Streaming 128-bit load that bypasses L1 allocation (weights are read once per step).
__device__ __forceinline__ uint4 ldg_stream(const void* p) {
    uint4 v;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p));
    return v;
}

}  // namespace neko
