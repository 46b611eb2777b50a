// The engine's gpu::ComputeBackend contract (app/architecture/shared/cpp/gpu/compute.h:24-48) on CUDA, and the
// single-operator C ABI. See include/neko_cuda.h.
//
// A context is one device plus one non-blocking stream. Buffers are plain device allocations owned by the
// context. dispatch() translates the GLSL kernels' parameter blocks (gpu/shaders/*.comp) into launches of the
// sm_100a kernels; consecutive dispatches are ordered by the stream (compute.h:38), flush() is a no-op and
// submitAndWait() polls the stream with a deadline, reporting kernel-side errors from the device error word.
#include <algorithm>
#include <chrono>
#include <cstdio>
#include <cstring>
#include <new>
#include <mutex>
#include <string>
#include <thread>
#include <vector>

#include "../../include/neko_cuda.h"
#include "neko_common.cuh"
#include "neko_internal.h"

namespace neko {

__device__ unsigned g_device_error = 0;

cudaError_t launch_kv_store(const float* qkv, int T, int W, int pos0, int stride, int k_off, int v_off, uint16_t* kc,
                            uint16_t* vc, cudaStream_t st);

std::string cuda_msg(cudaError_t e, const char* what) {
    return std::string(what) + ": " + cudaGetErrorName(e) + " (" + cudaGetErrorString(e) + ")";
}

cudaError_t enqueue_device_error_read(unsigned* host, cudaStream_t st) {
    return cudaMemcpyFromSymbolAsync(host, g_device_error, sizeof(unsigned), 0, cudaMemcpyDeviceToHost, st);
}

unsigned read_device_error(bool clear) {
    unsigned v = 0;
    if (cudaMemcpyFromSymbol(&v, g_device_error, sizeof v) != cudaSuccess) return 0;
    if (v && clear) {
        unsigned z = 0;
        cudaMemcpyToSymbol(g_device_error, &z, sizeof z);
    }
    return v;
}

int num_sms() {
    static int cache[64] = {0};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64) dev = 0;
    if (!cache[dev]) {
        int n = 0;
        cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
        cache[dev] = n > 0 ? n : 1;
    }
    return cache[dev];
}

namespace {
struct DynSmem {
    int limit = -1;  // opt-in per-block limit less the kernel's static shared memory
    int set = 0;     // the kernel's dynamic shared memory attribute as last raised here
};
std::mutex g_dyn_mu;
std::vector<std::pair<std::pair<const void*, int>, DynSmem>> g_dyn;  // (function, device) -> state

DynSmem& dyn_state(const void* fn, int dev) {  // with g_dyn_mu held
    for (auto& e : g_dyn)
        if (e.first.first == fn && e.first.second == dev) return e.second;
    g_dyn.push_back({{fn, dev}, DynSmem{}});
    DynSmem& d = g_dyn.back().second;
    int optin = 0;
    cudaFuncAttributes fa{};
    if (cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev) == cudaSuccess &&
        cudaFuncGetAttributes(&fa, fn) == cudaSuccess)
        d.limit = std::max(0, optin - int(fa.sharedSizeBytes));
    else
        d.limit = 0;
    cudaGetLastError();
    return d;
}
}  // namespace

int max_dyn_smem(const void* fn) {
    int dev = 0;
    cudaGetDevice(&dev);
    std::lock_guard<std::mutex> lk(g_dyn_mu);
    return dyn_state(fn, dev).limit;
}

cudaError_t ensure_dyn_smem(const void* fn, size_t bytes) {
    int dev = 0;
    cudaGetDevice(&dev);
    std::lock_guard<std::mutex> lk(g_dyn_mu);
    DynSmem& d = dyn_state(fn, dev);
    if (bytes > size_t(d.limit)) return cudaErrorNotSupported;
    if (bytes <= size_t(d.set)) return cudaSuccess;
    const cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, int(bytes));
    if (e != cudaSuccess) {
        cudaGetLastError();  // leave no pending error for a later launch check to pick up
        return e;
    }
    d.set = int(bytes);
    return cudaSuccess;
}

}  // namespace neko

using namespace neko;

namespace {

thread_local std::string t_err;

}  // namespace

void neko::set_last_error(const std::string& msg) { t_err = msg; }

namespace {

int set_err(std::string* dst, int code, const std::string& msg) {
    if (dst) *dst = msg;
    t_err = msg;
    return code;
}

// Polls until all work on `st` is done or the deadline passes (the engine polls its fences the same way,
// vk_compute.cpp:185-215). Device-side error codes become NEKO_ERR_DEVICE.
int wait_stream(cudaStream_t st, std::string* err, double seconds = 120.0) {
    const auto t0 = std::chrono::steady_clock::now();
    for (int spin = 0;; spin++) {
        cudaError_t e = cudaStreamQuery(st);
        if (e == cudaSuccess) break;
        if (e != cudaErrorNotReady) return set_err(err, NEKO_ERR_CUDA, cuda_msg(e, "stream"));
        if (std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count() > seconds)
            return set_err(err, NEKO_ERR_TIMEOUT, "GPU work did not finish within the deadline");
        if (spin > 64) std::this_thread::sleep_for(std::chrono::microseconds(20));
    }
    if (unsigned d = read_device_error(true))
        return set_err(err, NEKO_ERR_DEVICE, "kernel reported device error " + std::to_string(d) +
                                                 (d == kErrMbarTimeout ? " (bounded wait timed out)" : ""));
    return NEKO_OK;
}

struct DeviceGuard {
    int prev = -1;
    explicit DeviceGuard(int dev) {
        cudaGetDevice(&prev);
        if (prev != dev) cudaSetDevice(dev);
    }
    ~DeviceGuard() {
        int cur = -1;
        cudaGetDevice(&cur);
        if (prev >= 0 && cur != prev) cudaSetDevice(prev);
    }
};

// Stream-ordered scratch for operators called outside a model comes from the library's own memory pool on the
// current device: it keeps what it has grown to (release threshold at its maximum), so after the first calls an
// allocation maps no memory, and the default pool's settings stay the caller's.
cudaError_t scratch_alloc(void** p, size_t bytes, cudaStream_t st) {
    static std::mutex mu;
    static cudaMemPool_t pools[64] = {};
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= 64) return cudaMallocAsync(p, bytes, st);
    cudaMemPool_t pool;
    {
        std::lock_guard<std::mutex> lock(mu);
        if (!pools[dev]) {
            cudaMemPoolProps props = {};
            props.allocType = cudaMemAllocationTypePinned;
            props.handleTypes = cudaMemHandleTypeNone;
            props.location.type = cudaMemLocationTypeDevice;
            props.location.id = dev;
            if ((e = cudaMemPoolCreate(&pools[dev], &props)) != cudaSuccess) return e;
            uint64_t keep = UINT64_MAX;
            cudaMemPoolSetAttribute(pools[dev], cudaMemPoolAttrReleaseThreshold, &keep);
        }
        pool = pools[dev];
    }
    return cudaMallocFromPoolAsync(p, bytes, pool, st);
}

// A matmul outside a model: a stream-ordered workspace for the tensor-core path's K splits and activation split,
// allocated and freed around the call (both stream-ordered, so the call can be captured in a graph). Without the
// memory the call still runs, on fewer CTAs.
cudaError_t launch_gemv_op(GemvArgs a, cudaStream_t st, bool pdl) {
    int64_t wf = 0, wt = 0;
    if (a.M >= 5) gemm_tc_scratch(a.fmt, a.rows, a.K, a.M, a.pair_off != 0, a.norm != kNormNone, &wf, &wt);
    if (wf == 0) return launch_gemv(a, st, pdl);
    const size_t fb = (size_t(wf) * 4 + 255) / 256 * 256, tb = size_t(wt) * 4;
    void* mem = nullptr;
    if (scratch_alloc(&mem, fb + tb, st) != cudaSuccess) {
        cudaGetLastError();
        return launch_gemv(a, st, pdl);
    }
    if (tb) cudaMemsetAsync(static_cast<char*>(mem) + fb, 0, tb, st);
    a.ws = static_cast<float*>(mem);
    a.ws_floats = wf;
    a.ws_tickets = tb ? reinterpret_cast<unsigned*>(static_cast<char*>(mem) + fb) : nullptr;
    a.ws_ntickets = int(wt);
    const cudaError_t e = launch_gemv(a, st, pdl);
    cudaFreeAsync(mem, st);
    return e;
}

}  // namespace

struct neko_buf {
    size_t size = 0;
    void* dev = nullptr;
    bool readback = false;
};

struct neko_ctx {
    int device = 0;
    cudaStream_t stream = nullptr;
    std::string err;
    std::string devname;
    std::vector<neko_buf*> bufs;
    // split-KV attention scratch for the Attention dispatch, grown on demand
    float* part = nullptr;
    unsigned* tickets = nullptr;
    int64_t part_cap = 0, tick_cap = 0;
};

extern "C" {

const char* neko_last_error(void) { return t_err.c_str(); }
int neko_abi_version(void) { return NEKO_ABI_VERSION; }

neko_ctx* neko_cuda_create(int device, char* err, size_t err_len) {
    auto fail = [&](const std::string& m) -> neko_ctx* {
        t_err = m;
        if (err && err_len) std::snprintf(err, err_len, "%s", m.c_str());
        return nullptr;
    };
    int n = 0;
    cudaError_t e = cudaGetDeviceCount(&n);
    if (e != cudaSuccess || n == 0) return fail("no CUDA device: " + std::string(cudaGetErrorString(e)));
    if (device < 0 || device >= n) return fail("CUDA device index out of range");
    DeviceGuard g(device);
    cudaDeviceProp p{};
    if ((e = cudaGetDeviceProperties(&p, device)) != cudaSuccess) return fail(cuda_msg(e, "properties"));
    if (p.major < 10) return fail(std::string("kernels are built for sm_100a; device is ") + p.name);
    auto* c = new (std::nothrow) neko_ctx;
    if (!c) return fail("out of host memory");
    c->device = device;
    if ((e = cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking)) != cudaSuccess) {
        delete c;
        return fail(cuda_msg(e, "stream"));
    }
    c->devname = std::string(p.name) + " (sm_" + std::to_string(p.major * 10 + p.minor) + ", " +
                 std::to_string(p.multiProcessorCount) + " SMs)";
    return c;
}

void neko_cuda_destroy(neko_ctx* c) {
    if (!c) return;
    DeviceGuard g(c->device);
    cudaStreamSynchronize(c->stream);
    for (auto* b : c->bufs) {
        cudaFree(b->dev);
        delete b;
    }
    cudaFree(c->part);
    cudaFree(c->tickets);
    cudaStreamDestroy(c->stream);
    delete c;
}

const char* neko_cuda_last_error(neko_ctx* c) { return c ? c->err.c_str() : t_err.c_str(); }
const char* neko_cuda_name(neko_ctx*) { return "CUDA"; }

int neko_cuda_device_name(neko_ctx* c, char* buf, size_t len) {
    if (!c) return NEKO_ERR_ARG;
    if (buf && len) std::snprintf(buf, len, "%s", c->devname.c_str());
    return int(c->devname.size());
}

size_t neko_cuda_max_buffer_bytes(neko_ctx* c) {
    if (!c) return 0;
    DeviceGuard g(c->device);
    size_t free_b = 0, total = 0;
    cudaMemGetInfo(&free_b, &total);
    return total;  // a single allocation may use all of HBM
}

neko_buf* neko_cuda_create_buffer(neko_ctx* c, size_t bytes, const void* init, int readback) {
    if (!c) return nullptr;
    DeviceGuard g(c->device);
    auto* b = new (std::nothrow) neko_buf;
    if (!b) return nullptr;
    b->size = bytes;
    b->readback = readback != 0;
    const size_t alloc = std::max<size_t>(256, (bytes + 255) / 256 * 256);
    cudaError_t e = cudaMalloc(&b->dev, alloc);
    if (e != cudaSuccess) {
        set_err(&c->err, NEKO_ERR_NOMEM, cuda_msg(e, "cudaMalloc"));
        delete b;
        return nullptr;
    }
    e = init ? cudaMemcpyAsync(b->dev, init, bytes, cudaMemcpyHostToDevice, c->stream)
             : cudaMemsetAsync(b->dev, 0, alloc, c->stream);
    if (e == cudaSuccess && init) e = cudaStreamSynchronize(c->stream);
    if (e != cudaSuccess) {
        set_err(&c->err, NEKO_ERR_CUDA, cuda_msg(e, "buffer init"));
        cudaFree(b->dev);
        delete b;
        return nullptr;
    }
    c->bufs.push_back(b);
    return b;
}

int neko_cuda_upload(neko_ctx* c, neko_buf* b, size_t off, const void* src, size_t n) {
    if (!c || !b || !src || off + n > b->size) return set_err(c ? &c->err : nullptr, NEKO_ERR_ARG, "upload out of range");
    DeviceGuard g(c->device);
    cudaError_t e = cudaMemcpyAsync(static_cast<char*>(b->dev) + off, src, n, cudaMemcpyHostToDevice, c->stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(c->stream);  // src may be reused by the caller right away
    return e == cudaSuccess ? NEKO_OK : set_err(&c->err, NEKO_ERR_CUDA, cuda_msg(e, "upload"));
}

int neko_cuda_download(neko_ctx* c, neko_buf* b, size_t off, void* dst, size_t n) {
    if (!c || !b || !dst || off + n > b->size)
        return set_err(c ? &c->err : nullptr, NEKO_ERR_ARG, "download out of range");
    DeviceGuard g(c->device);
    if (int rc = wait_stream(c->stream, &c->err); rc != NEKO_OK) return rc;
    cudaError_t e = cudaMemcpyAsync(dst, static_cast<char*>(b->dev) + off, n, cudaMemcpyDeviceToHost, c->stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(c->stream);
    return e == cudaSuccess ? NEKO_OK : set_err(&c->err, NEKO_ERR_CUDA, cuda_msg(e, "download"));
}

int neko_cuda_begin(neko_ctx* c) { return c ? NEKO_OK : NEKO_ERR_ARG; }
int neko_cuda_flush(neko_ctx* c) { return c ? NEKO_OK : NEKO_ERR_ARG; }

int neko_cuda_submit_and_wait(neko_ctx* c) {
    if (!c) return NEKO_ERR_ARG;
    DeviceGuard g(c->device);
    return wait_stream(c->stream, &c->err);
}

size_t neko_cuda_buffer_size(const neko_buf* b) { return b ? b->size : 0; }
void* neko_cuda_buffer_device_ptr(const neko_buf* b) { return b ? b->dev : nullptr; }

int neko_cuda_dispatch(neko_ctx* c, int kernel, neko_buf* const bind[4], const int32_t p[8], uint32_t gx,
                       uint32_t gy) {
    if (!c || !bind || !p) return NEKO_ERR_ARG;
    DeviceGuard guard(c->device);
    auto ptr = [&](int i) -> void* { return bind[i] ? bind[i]->dev : nullptr; };
    auto size = [&](int i) -> size_t { return bind[i] ? bind[i]->size : 0; };
    auto fbits = [](int32_t v) {
        float f;
        std::memcpy(&f, &v, 4);
        return f;
    };
    auto bad = [&](const std::string& m) { return set_err(&c->err, NEKO_ERR_ARG, "dispatch: " + m); };
    cudaError_t e = cudaSuccess;
    switch (kernel) {
        case NEKO_K_EMBED: {  // embed.comp
            const int T = p[0], C = p[1], pos0 = p[2], flags = p[3], base = p[4], rows = p[5];
            const int fmt = (flags & 2) ? kFP8 : (flags & 4) ? kFP4 : kF16;
            const int64_t rb = fmt == kF16 ? int64_t(C) * 2 : int64_t(p[6]) * 4;
            if (T <= 0 || C <= 0 || size(0) < size_t(T) * 4 || size(3) < size_t(T) * C * 4 ||
                size(1) < size_t(rows) * rb || ((flags & 1) && size(2) < size_t(pos0 + T) * C * 2) ||
                (fmt != kF16 && rb != row_bytes(fmt, C)))
                return bad("embed sizes");
            e = launch_embed(static_cast<const int*>(ptr(0)), T, C, fmt, static_cast<const uint8_t*>(ptr(1)), rb, base,
                             rows, (flags & 1) ? static_cast<const uint16_t*>(ptr(2)) : nullptr, nullptr, pos0, nullptr,
                             static_cast<float*>(ptr(3)), c->stream, true);
            break;
        }
        case NEKO_K_LAYERNORM: {  // layernorm.comp
            const int C = p[0], off = p[2], rms = p[3] & 1, rows = int(gx);
            if (C <= 0 || size(0) < size_t(rows + off) * C * 4 || size(1) < size_t(rows) * C * 4 ||
                size(2) < size_t(C) * 4 || (!rms && size(3) < size_t(C) * 4))
                return bad("layernorm sizes");
            e = launch_norm(static_cast<const float*>(ptr(0)) + int64_t(off) * C, C, static_cast<float*>(ptr(1)), C,
                            static_cast<const float*>(ptr(2)), static_cast<const float*>(ptr(3)), rows, C, fbits(p[1]),
                            rms != 0, c->stream, true);
            break;
        }
        case NEKO_K_MATMUL:
        case NEKO_K_MATMUL_Q8:
        case NEKO_K_MATMUL_Q4: {  // matmul.comp, matmul_q8.comp, matmul_q4.comp
            const int fmt = kernel == NEKO_K_MATMUL ? kF16 : kernel == NEKO_K_MATMUL_Q8 ? kFP8 : kFP4;
            const int K = p[0], N = p[1], T = p[2], flags = p[3], x0 = p[4], noff = p[5], rows = int(gx);
            const int64_t rb = row_bytes(fmt, K);
            if (K <= 0 || T <= 0 || rows <= 0 || (fmt == kF16 ? K % 8 : K % 32) != 0)
                return bad("matmul K must be a multiple of 8 (F16) or 32 (FP8/FP4)");
            if (size(1) < size_t(rows) * rb || size(0) < size_t(x0 + T) * K * 4 ||
                size(3) < (size_t(T - 1) * N + noff + rows) * 4 || ((flags & 4) && size(2) < size_t(rows) * 4))
                return bad("matmul sizes");
            GemvArgs a;
            a.W = static_cast<const uint8_t*>(ptr(1));
            a.row_bytes = rb;
            a.rows = rows;
            a.K = K;
            a.fmt = fmt;
            a.x = static_cast<const float*>(ptr(0)) + int64_t(x0) * K;
            a.x_stride = K;
            a.M = T;
            a.bias = static_cast<const float*>(ptr(2));
            a.flags = flags & (kGelu | kAccumulate | kBias);
            a.y = static_cast<float*>(ptr(3));
            a.y_stride = N;
            a.n_off = noff;
            e = launch_gemv_op(a, c->stream, true);
            break;
        }
        case NEKO_K_KVSTORE: {  // kv_store.comp
            const int T = p[0], W = p[1], pos0 = p[2], stride = p[4], ko = p[5], vo = p[6];
            if (T <= 0 || W <= 0 || size(0) < (size_t(T - 1) * stride + std::max(ko, vo) + W) * 4 ||
                size(1) < size_t(pos0 + T) * W * 2 || size(2) < size_t(pos0 + T) * W * 2)
                return bad("kv_store sizes");
            e = launch_kv_store(static_cast<const float*>(ptr(0)), T, W, pos0, stride, ko, vo,
                                static_cast<uint16_t*>(ptr(1)), static_cast<uint16_t*>(ptr(2)), c->stream);
            break;
        }
        case NEKO_K_ATTENTION: {  // attention.comp
            const int T = p[0], qs = p[1], H = p[2], pos0 = p[3], hd = p[4], kvW = p[6];
            if (T <= 0 || H <= 0 || hd <= 0 || kvW <= 0 || kvW % hd != 0) return bad("attention params");
            const int KV = kvW / hd;
            if (H % KV != 0 || size(1) < size_t(pos0 + T) * kvW * 2 || size(2) < size_t(pos0 + T) * kvW * 2 ||
                size(0) < (size_t(T - 1) * qs + size_t(H) * hd) * 4 || size(3) < size_t(T) * H * hd * 4)
                return bad("attention sizes");
            AttnArgs a;
            a.q = static_cast<const float*>(ptr(0));
            a.q_stride = qs;
            a.kc = static_cast<const uint16_t*>(ptr(1));
            a.vc = static_cast<const uint16_t*>(ptr(2));
            a.slot_stride = 0;
            a.pos_stride = kvW;
            a.head_stride = hd;
            a.pos0 = pos0;
            a.rows = T;
            a.n_head = H;
            a.n_kv = KV;
            a.hd = hd;
            a.scale = fbits(p[5]);
            a.out = static_cast<float*>(ptr(3));
            a.out_stride = int64_t(H) * hd;
            a.max_pos = pos0 + T - 1;
            int64_t need_p = 0, need_t = 0;
            attention_scratch(T, H, KV, hd, a.max_pos, &need_p, &need_t);
            if (need_p > c->part_cap) {
                cudaStreamSynchronize(c->stream);
                cudaFree(c->part);
                c->part = nullptr;
                if ((e = cudaMalloc(&c->part, size_t(need_p) * 4)) != cudaSuccess) break;
                c->part_cap = need_p;
            }
            if (need_t > c->tick_cap) {
                cudaStreamSynchronize(c->stream);
                cudaFree(c->tickets);
                c->tickets = nullptr;
                if ((e = cudaMalloc(&c->tickets, size_t(need_t) * 4)) != cudaSuccess) break;
                if ((e = cudaMemset(c->tickets, 0, size_t(need_t) * 4)) != cudaSuccess) break;
                c->tick_cap = need_t;
            }
            a.part = c->part;
            a.tickets = c->tickets;
            a.part_capacity = c->part_cap;
            a.ticket_capacity = c->tick_cap;
            e = launch_attention(a, c->stream, true);
            break;
        }
        case NEKO_K_ROPE: {  // rope.comp
            const int stride = p[0], H = p[1], hd = p[2], pos0 = p[3], flags = p[5], T = int(gy);
            const int KV = int(gx) - H;
            if (T <= 0 || H <= 0 || KV < 0 || hd <= 0 || hd > 256 || (hd & 1) ||
                size(0) < (size_t(T - 1) * stride + size_t(H + KV) * hd) * 4 || size(2) < size_t(pos0 + T) * hd * 4 ||
                ((flags & 1) && size(1) < size_t(2) * hd * 4))
                return bad("rope sizes");
            QkvPostArgs a;
            a.qkv = static_cast<float*>(ptr(0));
            a.qkv_stride = stride;
            a.rows = T;
            a.n_head = H;
            a.n_kv = KV;
            a.hd = hd;
            a.do_norm = flags & 1;
            a.wn = static_cast<const float*>(ptr(1));
            a.eps = fbits(p[4]);
            a.do_rope = 1;
            a.cs = static_cast<const float*>(ptr(2));
            a.pos0 = pos0;
            a.k_off = H * hd;
            e = launch_qkv_post(a, c->stream, true);
            break;
        }
        case NEKO_K_SILUMUL: {  // silu_mul.comp
            const int T = p[0], I = p[1];
            if (T <= 0 || I <= 0 || size(0) < size_t(T) * 2 * I * 4 || size(1) < size_t(T) * I * 4)
                return bad("silu_mul sizes");
            e = launch_silu_mul(static_cast<const float*>(ptr(0)), static_cast<float*>(ptr(1)), T, I, c->stream);
            break;
        }
        default:
            return bad("unknown kernel id " + std::to_string(kernel));
    }
    if (e != cudaSuccess) {
        cudaGetLastError();  // reported here; none stays pending for the next call's launch check
        return set_err(&c->err, NEKO_ERR_CUDA, cuda_msg(e, "dispatch"));
    }
    return NEKO_OK;
}

// ------------------------------------------------------------------ operators on device pointers

int64_t neko_row_bytes(int format, int cols) { return row_bytes(format, cols); }

#define NEKO_OP_RETURN(expr)                                                        \
    do {                                                                            \
        cudaError_t e_ = (expr);                                                    \
        if (e_ == cudaSuccess) return NEKO_OK;                                      \
        cudaGetLastError(); /* the error is reported here; none stays pending */   \
        return set_err(nullptr, NEKO_ERR_CUDA, cuda_msg(e_, __func__));             \
    } while (0)

int neko_op_quantize(int format, const float* w, int rows, int cols, int64_t ld, int transpose_f16, uint8_t* out,
                     void* stream) {
    if (!w || !out || rows < 0 || cols <= 0 || format < 0 || format > 2) return set_err(nullptr, NEKO_ERR_ARG, "quantize args");
    if (format != kF16 && cols % kQuantBlock) return set_err(nullptr, NEKO_ERR_ARG, "FP8/FP4 need cols % 32 == 0");
    NEKO_OP_RETURN(launch_quantize(format, w, rows, cols, ld, transpose_f16, out, static_cast<cudaStream_t>(stream)));
}

int neko_op_dequantize(int format, const uint8_t* q, int rows, int cols, float* out, void* stream) {
    if (!q || !out || rows < 0 || cols <= 0 || format < 0 || format > 2) return set_err(nullptr, NEKO_ERR_ARG, "dequantize args");
    if (format != kF16 && cols % kQuantBlock) return set_err(nullptr, NEKO_ERR_ARG, "FP8/FP4 need cols % 32 == 0");
    NEKO_OP_RETURN(launch_dequantize(format, q, rows, cols, out, static_cast<cudaStream_t>(stream)));
}

int neko_op_matmul(int format, const float* x, int T, int K, const uint8_t* W, int rows, const float* bias, float* y,
                   int y_stride, int n_off, int flags, void* stream) {
    if (!x || !W || !y || T <= 0 || K <= 0 || rows <= 0 || format < 0 || format > 2)
        return set_err(nullptr, NEKO_ERR_ARG, "matmul args");
    if ((format == kF16 ? K % 8 : K % 32) != 0) return set_err(nullptr, NEKO_ERR_ARG, "matmul K alignment");
    if ((flags & kBias) && !bias) return set_err(nullptr, NEKO_ERR_ARG, "matmul bias flag without bias");
    GemvArgs a;
    a.W = W;
    a.row_bytes = row_bytes(format, K);
    a.rows = rows;
    a.K = K;
    a.fmt = format;
    a.x = x;
    a.x_stride = K;
    a.M = T;
    a.bias = bias;
    a.flags = flags & (kGelu | kAccumulate | kBias);
    a.y = y;
    a.y_stride = y_stride;
    a.n_off = n_off;
    NEKO_OP_RETURN(launch_gemv_op(a, static_cast<cudaStream_t>(stream), (flags & NEKO_PDL) != 0));
}

int neko_op_matmul_fused(int format, const float* x, int T, int K, const uint8_t* W, int rows, int norm,
                         const float* gamma, const float* beta, float eps, int swiglu, const float* bias, float* y,
                         int y_stride, int n_off, int flags, void* stream) {
    if (!x || !W || !y || T <= 0 || K <= 0 || rows <= 0 || format < 0 || format > 2 || norm < 0 || norm > 2)
        return set_err(nullptr, NEKO_ERR_ARG, "matmul_fused args");
    if ((format == kF16 ? K % 8 : K % 32) != 0) return set_err(nullptr, NEKO_ERR_ARG, "matmul K alignment");
    if (norm && (!gamma || (norm == kNormLayer && !beta))) return set_err(nullptr, NEKO_ERR_ARG, "norm weights");
    if (norm && !gemv_norm_fusable(format, T, K))
        return set_err(nullptr, NEKO_ERR_ARG,
                       "norm prologue needs T * K <= 4096, K % 128 == 0 and T * K padded to 512-byte code "
                       "segments within 40 KB of activations");
    if ((flags & kBias) && !bias) return set_err(nullptr, NEKO_ERR_ARG, "matmul bias flag without bias");
    GemvArgs a;
    a.W = W;
    a.row_bytes = row_bytes(format, K);
    a.rows = rows;
    a.K = K;
    a.fmt = format;
    a.x = x;
    a.x_stride = K;
    a.M = T;
    a.norm = norm;
    a.gamma = gamma;
    a.beta = beta;
    a.eps = eps;
    a.bias = bias;
    a.flags = swiglu ? 0 : flags & (kGelu | kAccumulate | kBias);
    a.y = y;
    a.y_stride = y_stride;
    a.n_off = n_off;
    a.pair_off = swiglu ? rows : 0;
    NEKO_OP_RETURN(launch_gemv_op(a, static_cast<cudaStream_t>(stream), (flags & NEKO_PDL) != 0));
}

namespace {
// RMSNorm / softmax over wide rows, fewer than the SMs: the split-row kernels with their partials in pool scratch.
cudaError_t wide_rows_op(const float* x, float* y, const float* gamma, int rows, int C, float eps, bool softmax,
                         int S, cudaStream_t st) {
    void* part = nullptr;
    if (cudaError_t e = scratch_alloc(&part, size_t(rows) * S * 2 * sizeof(double), st); e != cudaSuccess) return e;
    const cudaError_t e = launch_wide_rows(x, C, y, C, gamma, rows, C, eps, softmax, static_cast<double*>(part), S, st);
    cudaFreeAsync(part, st);
    return e;
}
}  // namespace

int neko_op_norm(const float* x, float* y, const float* gamma, const float* beta, int rows, int C, float eps,
                 void* stream) {
    if (!x || !y || !gamma || rows < 0 || C <= 0) return set_err(nullptr, NEKO_ERR_ARG, "norm args");
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    if (const int S = beta == nullptr ? wide_row_chunks(rows, C) : 0; S > 0)
        NEKO_OP_RETURN(wide_rows_op(x, y, gamma, rows, C, eps, false, S, st));
    NEKO_OP_RETURN(launch_norm(x, C, y, C, gamma, beta, rows, C, eps, beta == nullptr, st, false));
}

int neko_op_softmax(const float* x, float* y, int rows, int C, void* stream) {
    if (!x || !y || rows < 0 || C <= 0) return set_err(nullptr, NEKO_ERR_ARG, "softmax args");
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    if (const int S = wide_row_chunks(rows, C); S > 0) NEKO_OP_RETURN(wide_rows_op(x, y, nullptr, rows, C, 0.0f, true, S, st));
    NEKO_OP_RETURN(launch_softmax(x, y, rows, C, st));
}

int neko_op_argmax(const float* x, int rows, int C, int* out, void* stream) {
    if (!x || !out || rows < 0 || C <= 0) return set_err(nullptr, NEKO_ERR_ARG, "argmax args");
    NEKO_OP_RETURN(launch_argmax(x, C, rows, C, out, static_cast<cudaStream_t>(stream), false));
}

int neko_op_sample(float* logits, int rows, int V, const int* history, const int* hist_len, int hist_stride,
                   const double* u, const neko_sampling* params, int* out, void* stream) {
    if (!logits || !out || !params || rows < 0 || V <= 0 || hist_stride < 0)
        return set_err(nullptr, NEKO_ERR_ARG, "sample args");
    const neko_sampling sp = *params;
    if (sp.temperature > 0.0f && !u) return set_err(nullptr, NEKO_ERR_ARG, "sample: u is needed when temperature > 0");
    if (sp.repeat_penalty != 1.0f && sp.repeat_last_n > 0 && (!history || !hist_len))
        return set_err(nullptr, NEKO_ERR_ARG, "sample: the repetition penalty needs the history");
    if (sp.temperature > 0.0f && (sp.top_k <= 0 ? V : std::min(sp.top_k, V)) > kMaxTopK)
        return set_err(nullptr, NEKO_ERR_UNSUPPORTED, "sample: top_k above NEKO_MAX_TOP_K");
    NEKO_OP_RETURN(launch_sample(logits, rows, V, history, hist_len, hist_stride, u, sp, out,
                                 static_cast<cudaStream_t>(stream)));
}

int neko_op_fp8_block_dequant(const uint8_t* codes, int64_t rows, int64_t cols, const float* scales,
                              int64_t scale_rows, int64_t scale_cols, float* out, void* stream) {
    if (!codes || !scales || !out || rows < 0 || cols < 0 || scale_rows < 1 || scale_cols < 1)
        return set_err(nullptr, NEKO_ERR_ARG, "fp8_block_dequant args");
    NEKO_OP_RETURN(launch_fp8_block_dequant(codes, rows, cols, scales, scale_rows, scale_cols, out,
                                            static_cast<cudaStream_t>(stream)));
}

int neko_op_attention(const float* q, int q_stride, const uint16_t* k_cache, const uint16_t* v_cache, float* out,
                      int T, int n_head, int n_kv, int hd, int pos0, void* stream) {
    if (!q || !k_cache || !v_cache || !out || T <= 0 || !attention_shape_ok(n_head, n_kv, hd))
        return set_err(nullptr, NEKO_ERR_ARG, "attention args");
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
    int64_t need_p = 0, need_t = 0;
    attention_scratch(T, n_head, n_kv, hd, a.max_pos, &need_p, &need_t);
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    // Scratch for the split-KV merge, allocated per call (stream-ordered, from the library's pool).
    cudaError_t e = cudaSuccess;
    if (need_p) {
        if ((e = scratch_alloc(reinterpret_cast<void**>(&a.part), size_t(need_p) * 4, st)) != cudaSuccess)
            return set_err(nullptr, NEKO_ERR_NOMEM, cuda_msg(e, "attention scratch"));
        if ((e = scratch_alloc(reinterpret_cast<void**>(&a.tickets), size_t(need_t) * 4, st)) != cudaSuccess) {
            cudaFreeAsync(a.part, st);
            return set_err(nullptr, NEKO_ERR_NOMEM, cuda_msg(e, "attention scratch"));
        }
        cudaMemsetAsync(a.tickets, 0, size_t(need_t) * 4, st);
        a.part_capacity = need_p;
        a.ticket_capacity = need_t;
    }
    e = launch_attention(a, st, false);
    if (need_p) {
        cudaFreeAsync(a.part, st);
        cudaFreeAsync(a.tickets, st);
    }
    NEKO_OP_RETURN(e);
}

}  // extern "C"
