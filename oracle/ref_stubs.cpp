// Link stubs for compiling the NekoChat reference CPU engine on x86 as a test oracle.
//
// TEST INFRASTRUCTURE ONLY: this file is linked into oracle/_ref/*.so together with the reference's own
// sources (compiled where they lie, never copied). Nothing in the product links it.
//
// * The Vulkan and OpenGL ES factories (app/architecture/shared/cpp/gpu/vk_compute.cpp,
//   gl_compute.cpp) need a graphics stack that neither the build box nor the GPU box has, so they are
//   replaced by factories that report the API as unavailable. When NEKO_REF_WITH_CUDA is defined the
//   first backend slot that Model::startGpu tries (app/architecture/shared/cpp/model.cpp:137-148)
//   returns the CUDA backend instead, which is how the integration tests run the reference's own
//   gpu::selfTest and forwardGpu code on the B200 backend without editing a reference file.
// * GraniteModel (app/architecture/granite/cpp/granite_model.cpp) includes <arm_neon.h>
//   unconditionally and cannot be compiled on x86; model.cpp:191 still references its constructor.
//   Granite is outside the accelerated path, so loading it fails with a NekoError.

#include <memory>
#include <string>

#include "common.h"
#include "gpu/compute.h"
#include "granite_model.h"

namespace neko {
namespace gpu {

#if defined(NEKO_REF_WITH_CUDA)
std::unique_ptr<ComputeBackend> createCuda(std::string& error);  // nekochat_b200/csrc/cuda_compute.cpp

std::unique_ptr<ComputeBackend> createVulkan(std::string& error) { return createCuda(error); }
#else
std::unique_ptr<ComputeBackend> createVulkan(std::string& error) {
    error = "Vulkan is unavailable on this box (no graphics stack)";
    return nullptr;
}
#endif

std::unique_ptr<ComputeBackend> createGles(std::string& error) {
    error = "OpenGL ES is unavailable on this box (no graphics stack)";
    return nullptr;
}

}  // namespace gpu

GraniteModel::GraniteModel(const std::string&, const LoadOptions& opt, const ProgressFn&) : Model(opt) {
    fail("Granite 4.0-H is not part of the oracle build (its source requires arm_neon.h)");
}
GraniteModel::~GraniteModel() = default;
void GraniteModel::forward(const int*, int, int, float*) { fail("Granite is not built"); }
std::vector<Model::DebugStage> GraniteModel::debugStages() const { return {}; }
int GraniteModel::resumeFrom(int pos) { return pos; }
void GraniteModel::saveRestorePoint(int) {}

}  // namespace neko
