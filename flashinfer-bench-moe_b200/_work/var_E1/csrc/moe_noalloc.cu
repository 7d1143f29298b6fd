// moe_noalloc.cu -- fbmoe_forward_noalloc: the fused MoE forward for callers
// that cannot allocate device memory.
//
// Some callers have no way to obtain device scratch: code that runs while a
// framework's allocator is unavailable or forbidden (inside a custom runtime,
// a plugin host that hands over only input/output pointers, or a serving loop
// that must not touch the allocator on the hot path).  fbmoe_forward needs a
// workspace from its caller; this entry point instead keeps its workspace in a
// file-scope device array of a fixed size, so the caller passes only inputs,
// the output and a stream.
//
// Limits: T <= kNoAllocMaxTokens (16) and E_local <= kNoAllocMaxExperts (32),
// i.e. decode batches of one 32-expert shard.  The array is 12 MiB; every GPU
// on which the library's device code is loaded holds it until the process
// exits.  All calls share it and it keeps the last call's contents; the
// forward initialises everything it reads, so nothing needs clearing between
// calls, but two calls that overlap on the GPU (different streams, or
// different host threads without ordering) race on it.
//
// Set-up: the first call on each device looks up the array's device address
// with cudaGetSymbolAddress while that device is current.  With lazy module
// loading (the CUDA default), that lookup is also what makes the driver load
// this library's device code on the device, and with it commit the 12 MiB
// array.  So make the first call at set-up time, before any stream capture
// begins and before any memory budget on the hot path applies; after it, no
// call allocates or frees device memory.
//
// Errors: device-side status bits (a bounded wait that expired, an f16 value
// clamped) land in the array's status word; fbmoe_noalloc_read_status reads the
// word of the last call on the current device.
#include <mutex>

#include "fbmoe.h"
#include "fbmoe_common.cuh"
#include "fbmoe_launch.h"

namespace fbmoe {
namespace {

constexpr int kNoAllocMaxTokens = 16;
constexpr int kNoAllocMaxExperts = 32;
constexpr size_t kNoAllocScratchBytes = 12u << 20;  // >= make_layout(16, 32).total (checked at set-up)
constexpr int kMaxDevices = 64;

static __device__ __align__(256) uint8_t g_noalloc_scratch[kNoAllocScratchBytes];

std::mutex g_setup_mu;
void* g_scratch_ptr[kMaxDevices] = {nullptr};

// Device address of g_noalloc_scratch on the current device (looked up once).
int scratch_for_current_device(void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return (int)e;
  if (dev < 0 || dev >= kMaxDevices) return FBMOE_ERR_INVALID_ARG;
  std::lock_guard<std::mutex> lk(g_setup_mu);
  if (g_scratch_ptr[dev] == nullptr) {
    if (make_layout(kNoAllocMaxTokens, kNoAllocMaxExperts, false).total > kNoAllocScratchBytes)
      return FBMOE_ERR_NOALLOC_LIMIT;
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess) return (int)e;
    g_scratch_ptr[dev] = p;
  }
  *out = g_scratch_ptr[dev];
  return FBMOE_OK;
}

}  // namespace
}  // namespace fbmoe

extern "C" int fbmoe_noalloc_read_status(uint32_t* status, void* stream) {
  using namespace fbmoe;
  if (!status) return FBMOE_ERR_NULL_POINTER;
  *status = 0;
  void* scratch = nullptr;
  const int rc = scratch_for_current_device(&scratch);
  if (rc != FBMOE_OK) return rc;
  // the status word sits at offset 0 of the forward's layout (make_layout)
  return fbmoe_read_status(scratch, status, stream);
}

extern "C" int fbmoe_forward_noalloc(const float* routing_logits, const void* routing_bias, const void* hidden_states,
                                     const float* hidden_states_scale, const void* gemm1_weights,
                                     const float* gemm1_weights_scale, const void* gemm2_weights,
                                     const float* gemm2_weights_scale, int T, int E_local, int local_expert_offset,
                                     float routed_scaling_factor, void* out, void* stream) {
  using namespace fbmoe;
  if (T < 0 || E_local < 1 || E_local > kExperts) return FBMOE_ERR_INVALID_ARG;
  if (T > kNoAllocMaxTokens || E_local > kNoAllocMaxExperts) return FBMOE_ERR_NOALLOC_LIMIT;
  if (T == 0) return FBMOE_OK;
  void* scratch = nullptr;
  const int rc = scratch_for_current_device(&scratch);
  if (rc != FBMOE_OK) return rc;
  return forward_core(routing_logits, routing_bias, hidden_states, hidden_states_scale, gemm1_weights,
                      gemm1_weights_scale, gemm2_weights, gemm2_weights_scale, T, E_local, local_expert_offset,
                      routed_scaling_factor, out, false, scratch, kNoAllocScratchBytes, stream,
                      /*allow_split=*/false);
}
