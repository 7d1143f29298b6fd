// moe_prepack.cu -- offline W1 pre-pack: the linear and gate halves of each
// expert's W1 interleaved in 64-row slices, so that GEMM1 loads each operand
// tile with one TMA box.
//
// The reference passes raw weights on every call (solution/triton/main.py:
// 2720-2730) and has no pre-pack.  Raw W1 [E, 4096, 7168]: rows 0..2047 are the
// linear half (X1), rows 2048..4095 the half that goes through silu (X2).  GEMM1's
// operand tiles stack matching slices of the two halves: the decode kernel's
// 128-row tile is X1 rows [64g, 64g+64) over X2 rows [2048+64g, ..+64), the
// prefill kernel's 256-row tile X1 block j over X2 block j.  Packed, slice s of
// 64 rows of each half sit next to each other:
//     packed[e, 128s + w]      = W1[e, 64s + w]          (w < 64)
//     packed[e, 128s + 64 + w] = W1[e, 2048 + 64s + w]
// so the decode tile is packed rows [128g, 128g+128) and the prefill tile packed
// rows [256j, 256j+256), one box each.  The prefill tile then holds X1 and X2
// columns in 64-column runs (X1 2j, X2 2j, X1 2j+1, X2 2j+1), which its epilogue
// maps back.  The block scales keep the raw layout.  A pure copy: HBM-bound, 2 x 29 MB
// per expert.
#include "fbmoe.h"
#include "fbmoe_common.cuh"
#include "fbmoe_launch.h"

namespace fbmoe {
namespace {

constexpr int kPackWarps = 8;

__global__ void __launch_bounds__(kPackWarps * 32) prepack_w1_kernel(const uint8_t* __restrict__ w1,
                                                                    uint8_t* __restrict__ packed, long rows) {
  const int lane = threadIdx.x & 31;
  for (long p = (long)blockIdx.x * kPackWarps + (threadIdx.x >> 5); p < rows; p += (long)gridDim.x * kPackWarps) {
    const long e = p / kGemm1N;
    const int q = (int)(p % kGemm1N), s = q / 128, w = q % 128;
    const int src_row = w < 64 ? 64 * s + w : kInter + 64 * s + (w - 64);
    const uint4* src = reinterpret_cast<const uint4*>(w1 + ((size_t)e * kGemm1N + src_row) * kHidden);
    uint4* dst = reinterpret_cast<uint4*>(packed + (size_t)p * kHidden);
    uint4 v[kHidden / 16 / 32];
#pragma unroll
    for (int c = 0; c < kHidden / 16 / 32; ++c) v[c] = __ldcs(src + lane + 32 * c);
#pragma unroll
    for (int c = 0; c < kHidden / 16 / 32; ++c) __stcs(dst + lane + 32 * c, v[c]);
  }
}

}  // namespace
}  // namespace fbmoe

using namespace fbmoe;

extern "C" {

int fbmoe_prepack_w1(const void* gemm1_weights, int E_local, void* packed, void* stream) {
  if (E_local < 1 || E_local > kExperts) return FBMOE_ERR_INVALID_ARG;
  if (!gemm1_weights || !packed) return FBMOE_ERR_NULL_POINTER;
  if ((reinterpret_cast<uintptr_t>(gemm1_weights) | reinterpret_cast<uintptr_t>(packed)) & 15u)
    return FBMOE_ERR_MISALIGNED;
  if (gemm1_weights == packed) return FBMOE_ERR_INVALID_ARG;  // not in place
  const long rows = (long)E_local * kGemm1N;
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  prepack_w1_kernel<<<sms * 8, kPackWarps * 32, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint8_t*>(gemm1_weights), static_cast<uint8_t*>(packed), rows);
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? FBMOE_OK : (int)e;
}

int fbmoe_forward_prepacked(const float* routing_logits, const void* routing_bias, const void* hidden_states,
                            const float* hidden_states_scale, const void* gemm1_weights_packed,
                            const float* gemm1_weights_scale, const void* gemm2_weights,
                            const float* gemm2_weights_scale, int T, int E_local, int local_expert_offset,
                            float routed_scaling_factor, void* out, void* workspace, size_t workspace_bytes,
                            void* stream) {
  return forward_core(routing_logits, routing_bias, hidden_states, hidden_states_scale, gemm1_weights_packed,
                      gemm1_weights_scale, gemm2_weights, gemm2_weights_scale, T, E_local, local_expert_offset,
                      routed_scaling_factor, out, false, workspace, workspace_bytes, stream, true, nullptr, nullptr,
                      nullptr, /*w1_packed=*/true);
}

}  // extern "C"
