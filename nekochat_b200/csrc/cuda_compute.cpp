// CUDA implementation of the engine's gpu::ComputeBackend (app/architecture/shared/cpp/gpu/compute.h:24-45).
//
// This file is written to be added to the engine's own source tree next to vk_compute.cpp / gl_compute.cpp,
// with a createCuda() slot in Model::startGpu (model.cpp:137-148): it includes the engine's "gpu/compute.h" and "common.h" and calls the B200 kernels
// only through the C ABI of libneko_cuda.so (include/neko_cuda.h). Semantics follow the Vulkan backend:
// buffers are owned by the backend until it is destroyed, every dispatch is ordered after the previous one,
// flush() submits nothing extra (CUDA streams already run ahead of the host), submitAndWait() blocks until
// the GPU is done, and every failure is reported with fail() (a NekoError), which makes Model::startGpu fall
// back to the next backend (model.cpp:164-171).
#include <cstdlib>
#include <memory>
#include <string>
#include <vector>

#include "common.h"
#include "gpu/compute.h"
#include "neko_cuda.h"

namespace neko::gpu {

namespace {

struct CudaBuffer : Buffer {
    neko_buf* handle = nullptr;
};

class CudaBackend : public ComputeBackend {
public:
    explicit CudaBackend(neko_ctx* ctx) : ctx_(ctx) {}
    ~CudaBackend() override { neko_cuda_destroy(ctx_); }

    const char* name() const override { return "CUDA"; }

    std::string deviceName() const override {
        char buf[256];
        neko_cuda_device_name(ctx_, buf, sizeof buf);
        return buf;
    }

    size_t maxBufferBytes() const override { return neko_cuda_max_buffer_bytes(ctx_); }

    Buffer* create(size_t bytes, const void* init, bool readback) override {
        neko_buf* h = neko_cuda_create_buffer(ctx_, bytes, init, readback ? 1 : 0);
        if (!h) fail(std::string("CUDA buffer of ") + std::to_string(bytes) + " bytes: " + neko_cuda_last_error(ctx_));
        auto b = std::make_unique<CudaBuffer>();
        b->size = bytes;
        b->handle = h;
        buffers_.push_back(std::move(b));
        return buffers_.back().get();
    }

    void upload(Buffer* b, size_t offset, const void* src, size_t bytes) override {
        check(neko_cuda_upload(ctx_, handle(b), offset, src, bytes), "upload");
    }

    void download(Buffer* b, size_t offset, void* dst, size_t bytes) override {
        check(neko_cuda_download(ctx_, handle(b), offset, dst, bytes), "download");
    }

    void begin() override { check(neko_cuda_begin(ctx_), "begin"); }

    void dispatch(Kernel k, Buffer* const bindings[4], const int32_t params[8], uint32_t gx, uint32_t gy) override {
        neko_buf* h[4];
        for (int i = 0; i < 4; i++) h[i] = bindings[i] ? handle(bindings[i]) : nullptr;
        check(neko_cuda_dispatch(ctx_, int(k), h, params, gx, gy), "dispatch");
    }

    void flush() override { check(neko_cuda_flush(ctx_), "flush"); }

    void submitAndWait() override { check(neko_cuda_submit_and_wait(ctx_), "submitAndWait"); }

private:
    static neko_buf* handle(Buffer* b) { return static_cast<CudaBuffer*>(b)->handle; }

    void check(int rc, const char* what) {
        if (rc != NEKO_OK) fail(std::string("CUDA ") + what + ": " + neko_cuda_last_error(ctx_));
    }

    neko_ctx* ctx_;
    std::vector<std::unique_ptr<CudaBuffer>> buffers_;
};

}  // namespace

// Factory next to createVulkan / createGles (compute.h:47-48). NEKO_CUDA_DEVICE selects the device (default 0).
std::unique_ptr<ComputeBackend> createCuda(std::string& error) {
    const char* env = std::getenv("NEKO_CUDA_DEVICE");
    const int device = env ? std::atoi(env) : 0;
    char err[512] = {0};
    neko_ctx* ctx = neko_cuda_create(device, err, sizeof err);
    if (!ctx) {
        error = err;
        return nullptr;
    }
    return std::make_unique<CudaBackend>(ctx);
}

}  // namespace neko::gpu
