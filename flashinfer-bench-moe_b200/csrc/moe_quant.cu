// moe_quant.cu -- activation quantiser: bf16 [T, 7168] -> e4m3 [T, 7168] plus the
// operator's transposed 1x128 scales fp32 [56, T] (the producer of fused_moe's
// hidden_states / hidden_states_scale).
//
// The rule is the reference's own 1x128 quantisation (solution/triton/main.py:
// 1476-1488, there applied to the SwiGLU output): per row and 128-column block,
// scale = amax / 448 (1 when the block is all zeros), q = e4m3(clamp(x / scale,
// -448, 448)) with round-to-nearest-even.  x / scale is an IEEE fp32 division, so
// results are bit-identical to the same formula evaluated in fp32 on the host.
//
// One warp per (row, 8 consecutive blocks): 128 bf16 = 8 bytes per lane per
// block, warp max by shuffles, one 4-byte store per lane per block.  HBM-bound:
// 14,336 B read + 7,168 B + 224 B written per row.
#include "fbmoe.h"
#include "fbmoe_common.cuh"
#include "fbmoe_launch.h"

namespace fbmoe {
namespace {

constexpr int kWarps = 8;

// Blocks per warp task: their loads are issued together, so each warp keeps
// 8 x 256 B in flight (streaming needs ~100 KB in flight per SM).
constexpr int kGroup = 8;
static_assert(kHBlocks % kGroup == 0, "blocks per row must split into groups");

__global__ void __launch_bounds__(kWarps * 32) quant_act_kernel(const __nv_bfloat16* __restrict__ x, int T,
                                                                uint8_t* __restrict__ q, float* __restrict__ scale) {
  const int lane = threadIdx.x & 31;
  constexpr int kGroupsPerRow = kHBlocks / kGroup;
  const long n_tasks = (long)T * kGroupsPerRow;
  pdl_wait();
  pdl_trigger();
  for (long task = (long)blockIdx.x * kWarps + (threadIdx.x >> 5); task < n_tasks; task += (long)gridDim.x * kWarps) {
    const int t = (int)(task / kGroupsPerRow), kb0 = (int)(task % kGroupsPerRow) * kGroup;
    const size_t base = (size_t)t * kHidden + (size_t)kb0 * kBlk + lane * 4;
    uint2 raw[kGroup];
#pragma unroll
    for (int j = 0; j < kGroup; ++j) raw[j] = __ldg(reinterpret_cast<const uint2*>(x + base + j * kBlk));
    float m[kGroup];
#pragma unroll
    for (int j = 0; j < kGroup; ++j) {
      const float v0 = __uint_as_float(raw[j].x << 16), v1 = __uint_as_float(raw[j].x & 0xFFFF0000u);
      const float v2 = __uint_as_float(raw[j].y << 16), v3 = __uint_as_float(raw[j].y & 0xFFFF0000u);
      m[j] = fmaxf(fmaxf(fabsf(v0), fabsf(v1)), fmaxf(fabsf(v2), fabsf(v3)));
    }
#pragma unroll
    for (int d = 16; d >= 1; d >>= 1)
#pragma unroll
      for (int j = 0; j < kGroup; ++j) m[j] = fmaxf(m[j], __shfl_xor_sync(0xffffffffu, m[j], d));
#pragma unroll
    for (int j = 0; j < kGroup; ++j) {
      const float s = m[j] > 0.0f ? __fdiv_rn(m[j], 448.0f) : 1.0f;
      const float v[4] = {__uint_as_float(raw[j].x << 16), __uint_as_float(raw[j].x & 0xFFFF0000u),
                          __uint_as_float(raw[j].y << 16), __uint_as_float(raw[j].y & 0xFFFF0000u)};
      uint32_t packed = 0;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float y = fminf(fmaxf(__fdiv_rn(v[i], s), -448.0f), 448.0f);
        packed |= (uint32_t)__nv_cvt_float_to_fp8(y, __NV_SATFINITE, __NV_E4M3) << (8 * i);
      }
      *reinterpret_cast<uint32_t*>(q + base + j * kBlk) = packed;
      if (lane == j) scale[(size_t)(kb0 + j) * T + t] = s;
    }
  }
}

}  // namespace
}  // namespace fbmoe

extern "C" FBMOE_API int fbmoe_quantize_act(const void* x_bf16, int T, void* q_e4m3, float* scale, void* stream) {
  if (T < 0) return FBMOE_ERR_INVALID_ARG;
  if (T == 0) return FBMOE_OK;
  if (!x_bf16 || !q_e4m3 || !scale) return FBMOE_ERR_NULL_POINTER;
  if (((uintptr_t)x_bf16 & 7) || ((uintptr_t)q_e4m3 & 3)) return FBMOE_ERR_MISALIGNED;
  const long tasks = (long)T * (fbmoe::kHBlocks / fbmoe::kGroup);
  long blocks = (tasks + fbmoe::kWarps - 1) / fbmoe::kWarps;
  if (blocks > 148L * 16) blocks = 148L * 16;
  const cudaError_t e = fbmoe::launch_pdl(fbmoe::quant_act_kernel, dim3((unsigned)blocks), dim3(fbmoe::kWarps * 32),
                                          0, reinterpret_cast<cudaStream_t>(stream),
                                          reinterpret_cast<const __nv_bfloat16*>(x_bf16), T,
                                          reinterpret_cast<uint8_t*>(q_e4m3), scale);
  return e == cudaSuccess ? FBMOE_OK : (int)e;
}
