// Attention that never allocates device memory (neko_op_attention_noalloc in include/neko_cuda.h).
//
// neko_op_attention takes its split-KV scratch (per-split partial softmax state and the tickets that elect
// the CTA which merges them) from the stream-ordered allocator on every call. Some callers cannot allow that:
// an engine that budgets and reports every byte it holds on the device (the way NekoChat's MemoryStats counts
// weight, KV and workspace buffers) would see memory it never asked for, a caller under memory pressure could
// hit an out-of-memory failure in the middle of generating a reply, and a host that forbids allocator calls
// after start-up to keep each decode step's latency predictable cannot call it at all. This variant runs the
// same kernel with its scratch in a fixed array that is part of the library image instead.
//
// Limits and sharing:
//  * the scratch holds kNoAllocPartFloats floats of partial state and kNoAllocTickets tickets (4 MiB + 32 KiB,
//    resident on every GPU that loads the library until the process exits); a call that would need more is
//    rejected with NEKO_ERR_UNSUPPORTED and launches nothing;
//  * every call uses the same array and leaves its contents behind; the tickets are cleared on the caller's
//    stream before each launch, so a call never depends on what a previous one left there;
//  * calls whose kernels can overlap on the GPU (two streams, or two threads on one device) race on the array
//    and give wrong results: order them on one stream or serialise them;
//  * the first call on each device looks up the array's device address (cudaGetSymbolAddress) with that device
//    current; make that first call before any stream capture begins.
#include <mutex>

#include "../../include/neko_cuda.h"
#include "neko_common.cuh"
#include "neko_internal.h"

namespace neko {
namespace {

constexpr int64_t kNoAllocPartFloats = int64_t(1) << 20;  // 4 MiB of partial (max, sum, acc[hd]) records
constexpr int64_t kNoAllocTickets = 8192;                   // one per (row, KV head) of a split call

static __device__ __align__(256) float g_noalloc_part[kNoAllocPartFloats];
static __device__ __align__(256) unsigned g_noalloc_tickets[kNoAllocTickets];

struct DeviceScratch {
    float* part = nullptr;
    unsigned* tickets = nullptr;
};

constexpr int kMaxDevices = 64;
DeviceScratch g_scratch[kMaxDevices];
std::mutex g_scratch_mu;

int noalloc_fail(int code, const std::string& msg) {
    set_last_error(msg);  // readable through neko_last_error()
    return code;
}

// Device addresses of the two arrays on the current device, looked up once per device. In host code the
// arrays' names only stand for host-side shadows, so the kernel must get these addresses, never the names.
cudaError_t scratch_for_current_device(DeviceScratch* out) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
    std::lock_guard<std::mutex> lock(g_scratch_mu);
    DeviceScratch& s = g_scratch[dev];
    if (!s.part) {
        void* part = nullptr;
        void* tickets = nullptr;
        if ((e = cudaGetSymbolAddress(&part, g_noalloc_part)) != cudaSuccess) return e;
        if ((e = cudaGetSymbolAddress(&tickets, g_noalloc_tickets)) != cudaSuccess) return e;
        s.part = static_cast<float*>(part);
        s.tickets = static_cast<unsigned*>(tickets);
    }
    *out = s;
    return cudaSuccess;
}

}  // namespace
}  // namespace neko

using namespace neko;

extern "C" int neko_op_attention_noalloc(const float* q, int q_stride, const uint16_t* k_cache,
                                         const uint16_t* v_cache, float* out, int T, int n_head, int n_kv, int hd,
                                         int pos0, void* stream) {
    if (!q || !k_cache || !v_cache || !out || T <= 0 || pos0 < 0 || !attention_shape_ok(n_head, n_kv, hd))
        return noalloc_fail(NEKO_ERR_ARG, "attention_noalloc: bad arguments (at most 8 query heads per KV head, "
                                          "head_dim a multiple of 8 up to 256)");
    int64_t need_part = 0, need_tickets = 0;
    attention_scratch(T, n_head, n_kv, hd, pos0 + T - 1, &need_part, &need_tickets);
    // A single-split plan uses no scratch at all (no partials, no tickets), whatever its size.
    if (need_part == 0) need_tickets = 0;
    if (need_part > kNoAllocPartFloats || need_tickets > kNoAllocTickets)
        return noalloc_fail(NEKO_ERR_UNSUPPORTED,
                            "attention_noalloc: this shape needs " + std::to_string(need_part) +
                                " scratch floats and " + std::to_string(need_tickets) + " tickets; the fixed scratch holds " +
                                std::to_string(kNoAllocPartFloats) + " and " + std::to_string(kNoAllocTickets));
    DeviceScratch s;
    if (cudaError_t e = scratch_for_current_device(&s); e != cudaSuccess)
        return noalloc_fail(NEKO_ERR_CUDA, cuda_msg(e, "attention_noalloc scratch address"));
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    if (need_tickets) {
        if (cudaError_t e = cudaMemsetAsync(s.tickets, 0, size_t(need_tickets) * sizeof(unsigned), st); e != cudaSuccess)
            return noalloc_fail(NEKO_ERR_CUDA, cuda_msg(e, "attention_noalloc ticket clear"));
    }
    AttnArgs a;
    a.q = q;
    a.q_stride = q_stride;
    a.kc = k_cache;
    a.vc = v_cache;
    a.pos_stride = int64_t(n_kv) * hd;
    a.head_stride = hd;
    a.pos0 = pos0;
    a.rows = T;
    a.n_head = n_head;
    a.n_kv = n_kv;
    a.hd = hd;
    a.scale = 1.0f / sqrtf(float(hd));
    a.out = out;
    a.out_stride = int64_t(n_head) * hd;
    a.max_pos = pos0 + T - 1;
    a.part = s.part;
    a.tickets = s.tickets;
    a.part_capacity = kNoAllocPartFloats;
    a.ticket_capacity = kNoAllocTickets;
    if (cudaError_t e = launch_attention(a, st, false); e != cudaSuccess)
        return noalloc_fail(NEKO_ERR_CUDA, cuda_msg(e, "attention_noalloc"));
    return NEKO_OK;
}
