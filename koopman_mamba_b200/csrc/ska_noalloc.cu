// ska_noalloc.cu -- ska_fwd_noalloc: the forward with a compiled-in workspace.
//
// For callers that cannot allocate device memory (FFI hosts without a CUDA
// allocator, inference loops that must not call cudaMalloc).  The workspace is
// a fixed file-scope device array; its device address is looked up once per
// device and then handed to the ordinary forward.
#include "../../include/ska_b200.h"

#include <cuda_runtime.h>

#include <mutex>

namespace {

// Shared by every call on a device; holds the last call's contents.
static __device__ __align__(256) unsigned char g_noalloc_scratch[SKA_NOALLOC_SCRATCH_BYTES];

constexpr int kMaxDevices = 64;
std::mutex g_mu;
void* g_ptr[kMaxDevices] = {};

// Device address of g_noalloc_scratch on the current device (looked up once per
// device, with that device current).  nullptr on failure.
void* scratch_on_current_device() {
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return nullptr;
  std::lock_guard<std::mutex> lock(g_mu);
  if (!g_ptr[dev]) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_noalloc_scratch) != cudaSuccess || !p) return nullptr;
    g_ptr[dev] = p;
  }
  return g_ptr[dev];
}

}  // namespace

extern "C" int ska_fwd_noalloc(const SkaShape* shape, int io_dtype, const SkaTensor* z, const SkaTensor* zq,
                               const SkaTensor* v, const float* gamma, const SkaTensor* y, void* stream) {
  // the forward-only size: no backward reads this array, so the chunk operators
  // that a backward would need are not written
  size_t need = 0;
  int rc = ska_forward_workspace_size(shape, &need);
  if (rc != SKA_OK) return rc;
  if (need > SKA_NOALLOC_SCRATCH_BYTES) return SKA_ERR_WORKSPACE;
  if (shape->B == 0) return ska_fwd(shape, io_dtype, z, zq, v, gamma, y, nullptr, 0, stream);
  void* ws = scratch_on_current_device();
  if (!ws) return SKA_ERR_LAUNCH;
  return ska_fwd(shape, io_dtype, z, zq, v, gamma, y, ws, need, stream);
}
