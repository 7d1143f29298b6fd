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
// One warp per task = (row, 8 consecutive blocks): each half-warp owns one block
// per load (16 lanes x 16 B = 128 bf16), so a task is 4 loads of 16 B per lane,
// half-warp max by 4 shuffles, one 8-byte store per lane per block pair.  The
// next task's loads are issued before the current one is converted.  HBM-bound:
// 14,336 B read + 7,168 B + 224 B written per row.
//
// Division: q needs e4m3(RN(x / s)) only, which e4m3x2_quotient (fbmoe_common.cuh)
// gets from a multiplication by RN(1/s) and a bracketing conversion, dividing
// exactly only near an e4m3 rounding midpoint; results stay bit-identical to
// x / s in fp32.
#include "fbmoe.h"
#include "fbmoe_common.cuh"
#include "fbmoe_launch.h"

namespace fbmoe {
namespace {

constexpr int kWarps = 8;

// Blocks per warp task (4 loads of 16 B per lane, 2 blocks per load).
constexpr int kGroup = 8;
static_assert(kHBlocks % kGroup == 0, "blocks per row must split into groups");
constexpr int kLoads = kGroup / 2;

__device__ __forceinline__ void load_task(const __nv_bfloat16* __restrict__ x, long task, long n_tasks, int lane,
                                          uint4 (&v)[kLoads]) {
  if (task >= n_tasks) return;
  constexpr int kGroupsPerRow = kHBlocks / kGroup;
  const int t = (int)(task / kGroupsPerRow), kb0 = (int)(task % kGroupsPerRow) * kGroup;
  const __nv_bfloat16* p = x + (size_t)t * kHidden + (size_t)kb0 * kBlk + (lane >> 4) * kBlk + (lane & 15) * 8;
#pragma unroll
  for (int j = 0; j < kLoads; ++j) v[j] = __ldg(reinterpret_cast<const uint4*>(p + 2 * j * kBlk));
}

__global__ void __launch_bounds__(kWarps * 32) quant_act_kernel(const __nv_bfloat16* __restrict__ x, int T,
                                                                uint8_t* __restrict__ q, float* __restrict__ scale) {
  const int lane = threadIdx.x & 31;
  constexpr int kGroupsPerRow = kHBlocks / kGroup;
  const long n_tasks = (long)T * kGroupsPerRow;
  const long stride = (long)gridDim.x * kWarps;
  pdl_wait();
  pdl_trigger();
  long task = (long)blockIdx.x * kWarps + (threadIdx.x >> 5);
  uint4 cur[kLoads], nxt[kLoads];
  load_task(x, task, n_tasks, lane, cur);
  for (; task < n_tasks; task += stride) {
    load_task(x, task + stride, n_tasks, lane, nxt);
    const int t = (int)(task / kGroupsPerRow), kb0 = (int)(task % kGroupsPerRow) * kGroup;
#pragma unroll
    for (int j = 0; j < kLoads; ++j) {
      const uint32_t w[4] = {cur[j].x, cur[j].y, cur[j].z, cur[j].w};
      float v[8];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        v[2 * i] = __uint_as_float(w[i] << 16);
        v[2 * i + 1] = __uint_as_float(w[i] & 0xFFFF0000u);
      }
      float m = 0.0f;
#pragma unroll
      for (int i = 0; i < 8; ++i) m = fmaxf(m, fabsf(v[i]));
#pragma unroll
      for (int d = 8; d >= 1; d >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, d));
      const E4m3Scale qs = e4m3_block_scale(m);
      const float s = qs.s;
      uint32_t lo = 0, hi = 0;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const uint32_t pair = e4m3x2_quotient(v[2 * i], v[2 * i + 1], qs);
        if (i < 2) lo |= pair << (16 * i);
        else hi |= pair << (16 * (i - 2));
      }
      const int kb = kb0 + 2 * j + (lane >> 4);
      *reinterpret_cast<uint2*>(q + (size_t)t * kHidden + (size_t)kb * kBlk + (lane & 15) * 8) = make_uint2(lo, hi);
      if ((lane & 15) == 0) scale[(size_t)kb * T + t] = s;
    }
#pragma unroll
    for (int j = 0; j < kLoads; ++j) cur[j] = nxt[j];
  }
}

}  // namespace
}  // namespace fbmoe

extern "C" FBMOE_API int fbmoe_quantize_act(const void* x_bf16, int T, void* q_e4m3, float* scale, void* stream) {
  if (T < 0) return FBMOE_ERR_INVALID_ARG;
  if (T == 0) return FBMOE_OK;
  if (!x_bf16 || !q_e4m3 || !scale) return FBMOE_ERR_NULL_POINTER;
  if (((uintptr_t)x_bf16 & 15) || ((uintptr_t)q_e4m3 & 7)) return FBMOE_ERR_MISALIGNED;
  const long tasks = (long)T * (fbmoe::kHBlocks / fbmoe::kGroup);
  long blocks = (tasks + fbmoe::kWarps - 1) / fbmoe::kWarps;
  if (blocks > 148L * 8) blocks = 148L * 8;
  const cudaError_t e = fbmoe::launch_pdl(fbmoe::quant_act_kernel, dim3((unsigned)blocks), dim3(fbmoe::kWarps * 32),
                                          0, reinterpret_cast<cudaStream_t>(stream),
                                          reinterpret_cast<const __nv_bfloat16*>(x_bf16), T,
                                          reinterpret_cast<uint8_t*>(q_e4m3), scale);
  return e == cudaSuccess ? FBMOE_OK : (int)e;
}
