// extern "C" view of the NekoChat reference CPU engine, for ctypes.
//
// TEST INFRASTRUCTURE ONLY. Linked into oracle/_ref/libneko_ref*.so together with the reference's own
// sources; tests and the bench's CPU-baseline leg load it as the checker and the timed CPU baseline.
// Every function forwards to the reference API named in its comment (paths relative to
// app/architecture/shared/cpp unless stated otherwise) and converts C++ exceptions into an error string.

#include <cstdint>
#include <cstring>
#include <memory>
#include <random>
#include <stdexcept>
#include <string>
#include <thread>
#include <vector>

#include "common.h"
#include "cpu_ops.h"
#include "gpu/compute.h"
#include "model.h"
#include "quant.h"
#include "sampler.h"
#include "tensor_store.h"
#include "thread_pool.h"

using namespace neko;

namespace {

thread_local std::string g_err;

QMatrix wrap(int fmt, int rows, int cols, const uint8_t* data) {
    QMatrix m;
    m.format = WeightFormat(fmt);
    m.rows = rows;
    m.cols = cols;
    m.rowBytes = quantRowBytes(m.format, cols);
    m.data.assign(data, data + m.rowBytes * size_t(rows));
    return m;
}

ThreadPool& pool(int threads) {
    static std::unique_ptr<ThreadPool> p;
    static int n = -1;
    if (!p || n != threads) {
        p.reset();
        p = std::make_unique<ThreadPool>(threads);
        n = threads;
    }
    return *p;
}

template <class F>
int guarded(F&& f) {
    try {
        f();
        return 0;
    } catch (const std::exception& e) {
        g_err = e.what();
        return -1;
    }
}

}  // namespace

extern "C" {

const char* ref_last_error() { return g_err.c_str(); }

// quant.cpp:199-208
long ref_quant_row_bytes(int fmt, int cols) { return long(quantRowBytes(WeightFormat(fmt), cols)); }

// quant.cpp:255-279. w is [rows][cols] f32; out receives rows * quantRowBytes bytes.
int ref_quantize_matrix(int fmt, int rows, int cols, const float* w, uint8_t* out, int threads) {
    return guarded([&] {
        ThreadPool* p = threads > 0 ? &pool(threads) : nullptr;
        QMatrix m = quantizeMatrix(WeightFormat(fmt), rows, cols, [&](int r, float* o) {
            std::memcpy(o, w + size_t(r) * size_t(cols), size_t(cols) * 4);
        }, p);
        if (int(m.format) != fmt) fail("quantizeMatrix stored the matrix as F16 (cols % 32 != 0)");
        std::memcpy(out, m.data.data(), m.data.size());
    });
}

// quant.cpp:230-253
int ref_dequantize_rows(int fmt, int rows, int cols, const uint8_t* data, float* out) {
    return guarded([&] {
        QMatrix m = wrap(fmt, rows, cols, data);
        for (int r = 0; r < rows; r++) m.dequantizeRow(r, out + size_t(r) * size_t(cols));
    });
}

// cpu_ops.cpp:462-481 (x86: matmulGeneric :442-458; F16: matmulF16 :108-128)
int ref_matmul(int fmt, const float* x, int T, int K, const uint8_t* W, int rows, const float* bias, float* y,
               int yStride, int flags, int threads) {
    return guarded([&] {
        QMatrix m = wrap(fmt, rows, K, W);
        cpu::matmul(pool(threads), x, T, K, m, bias, y, yStride, flags);
    });
}

// cpu_ops.cpp:483-500
void ref_layer_norm(const float* x, float* y, const float* g, const float* b, int T, int C, float eps) {
    cpu::layerNorm(x, y, g, b, T, C, eps);
}

// cpu_ops.cpp:502-511
void ref_rms_norm(const float* x, float* y, const float* w, int rows, int C, float eps) {
    cpu::rmsNorm(x, y, w, rows, C, eps);
}

// cpu_ops.cpp:513-524
void ref_rope(float* x, int nHeads, int hd, const float* cs) { cpu::rope(x, nHeads, hd, cs); }

// cpu_ops.cpp:526-533
void ref_silu_mul(const float* h, float* out, int T, int I) { cpu::siluMul(h, out, T, I); }

// cpu_ops.cpp:20-23
float ref_gelu(float x) { return cpu::gelu(x); }

// cpu_ops.cpp:535-542
void ref_store_kv(const float* k, const float* v, int srcStride, uint16_t* kc, uint16_t* vc, int width, int T,
                  int pos0) {
    cpu::storeKv(k, v, srcStride, kc, vc, width, T, pos0);
}

// cpu_ops.cpp:544-575
void ref_attention(const float* q, int qStride, const uint16_t* kc, const uint16_t* vc, float* out, int T, int nHead,
                   int nKv, int hd, int pos0, int threads) {
    cpu::attention(pool(threads), q, qStride, kc, vc, out, T, nHead, nKv, hd, pos0);
}

// common.h:33-80
uint16_t ref_f32_to_f16(float f) { return f32_to_f16(f); }
float ref_f16_to_f32(uint16_t h) { return f16_to_f32(h); }

// model.cpp:175-193 + LoadOptions (model.h:29-33). backend: 0 Auto, 3 CPU. fmt: 0 F16, 1 FP8, 2 FP4.
void* ref_model_load(const char* dir, int backend, int fmt, int threads) {
    try {
        LoadOptions opt;
        opt.backend = BackendPref(backend);
        opt.weights = WeightFormat(fmt);
        opt.threads = threads;
        std::string d(dir);
        auto m = loadModel(readModelType(d), d, opt, [](float, const std::string&) {});
        return m.release();
    } catch (const std::exception& e) {
        g_err = e.what();
        return nullptr;
    }
}

void ref_model_free(void* m) { delete static_cast<Model*>(m); }

// Model::forward (model.h:72)
int ref_model_forward(void* m, const int* tokens, int T, int pos0, float* logits) {
    return guarded([&] { static_cast<Model*>(m)->forward(tokens, T, pos0, logits); });
}

// Model::setDebugLayers (model.h:101-104)
void ref_model_set_debug(void* m, int layers, int stage) { static_cast<Model*>(m)->setDebugLayers(layers, stage); }

int ref_model_vocab(void* m) { return static_cast<Model*>(m)->shape().vocab; }
int ref_model_context(void* m) { return static_cast<Model*>(m)->contextLength(); }

// Model::backendName / backendNote (model.h:83-85)
int ref_model_backend(void* m, char* buf, int len) {
    std::string s = static_cast<Model*>(m)->backendName() + "\n" + static_cast<Model*>(m)->backendNote();
    std::snprintf(buf, size_t(len), "%s", s.c_str());
    return int(s.size());
}

// Model::memory (model.h:91): weights, kvCapacity, workspace
void ref_model_memory(void* m, long long* weights, long long* kvCapacity, long long* workspace) {
    MemoryStats s = static_cast<Model*>(m)->memory(0);
    *weights = (long long)s.weights;
    *kvCapacity = (long long)s.kvCapacity;
    *workspace = (long long)s.workspace;
}

int ref_hardware_threads() { return int(std::thread::hardware_concurrency()); }

// Sampler::sample (sampler.cpp:14-55) with a fixed seed, on host logits (modified in place, as the engine's).
int ref_sample(float* logits, int n, const int* history, int hlen, float temperature, int top_k, float top_p,
               float repeat_penalty, int repeat_last_n, unsigned long long seed) {
    SamplingParams sp;
    sp.temperature = temperature;
    sp.topK = top_k;
    sp.topP = top_p;
    sp.repeatPenalty = repeat_penalty;
    sp.repeatLastN = repeat_last_n;
    sp.seed = seed;
    Sampler s(sp);
    const std::vector<int> h(history, history + hlen);
    return s.sample(logits, n, h);
}

// The uniform value in [0, 1) behind the first draw of a Sampler seeded with `seed`: its
// uniform_real_distribution<double>(0, total) on the same std::mt19937_64 returns total times this value.
double ref_sampler_draw(unsigned long long seed) {
    std::mt19937_64 rng(seed);
    std::uniform_real_distribution<double> u(0.0, 1.0);
    return u(rng);
}

// TensorStore::toF32 (tensor_store.cpp:578-590) of one tensor of a safetensors file: an FP8 (E4M3) weight comes
// out dequantized with its "_scale_inv" / "_scale" block scales (tensor_store.cpp:543-571). Returns the element
// count, or -1 (error text in ref_last_error).
long ref_tensor_f32(const char* path, const char* name, float* out, long cap) {
    long n = -1;
    const int rc = guarded([&] {
        TensorStore ts;
        ts.addFile(path);
        const std::vector<float> v = ts.toF32(name);
        if (long(v.size()) > cap) throw std::runtime_error("ref_tensor_f32: output buffer too small");
        std::memcpy(out, v.data(), v.size() * 4);
        n = long(v.size());
    });
    return rc ? -1 : n;
}

#if defined(NEKO_REF_WITH_CUDA)
}  // extern "C"
namespace neko::gpu {
std::unique_ptr<ComputeBackend> createCuda(std::string& error);
}
extern "C" {

// gpu/compute.cpp:32-290, run unmodified on the CUDA backend.
int ref_selftest_cuda(char* err, int len) {
    std::string e;
    auto be = gpu::createCuda(e);
    if (!be) {
        std::snprintf(err, size_t(len), "createCuda failed: %s", e.c_str());
        return -1;
    }
    bool ok = gpu::selfTest(*be, e);
    std::snprintf(err, size_t(len), "%s", e.c_str());
    return ok ? 0 : 1;
}
#endif

}  // extern "C"
