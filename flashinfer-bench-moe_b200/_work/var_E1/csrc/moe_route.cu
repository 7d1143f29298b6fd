// moe_route.cu -- DeepSeek-V3 no-aux router, one warp per token.
//
// Computes what the reference operator's routing computes (reference
// solution/triton/main.py:2522-2553; its CUDA counterpart is fusedGatingKernel,
// main.py:851-1038):
//   s = 1/(1+exp(-x)), s_with_bias = s + bias, group score = sum of the group's
//   two largest s_with_bias, keep the 4 best of 8 groups, keep the 8 best experts
//   of the kept groups, weight = s / (sum of the kept s + 1e-20) * scale.
//
// Exactness.  exp is evaluated in double and rounded once (the correctly rounded
// fp32 exp); add/div/mul are IEEE round-to-nearest intrinsics, so s and
// s_with_bias are bit-identical to the CPU restatement.  Selection sets are
// unique unless the k-th and (k+1)-th largest values are equal; in that case the
// warp replays torch.topk's CPU selection (std::nth_element introselect over
// (value, index) pairs) in shared memory, so tie-breaking matches torch.topk.
// Outputs are in canonical order: descending s_with_bias, ascending id among equals.
//
// Layout: lane l owns experts 8l..8l+7, so lanes 4g..4g+3 hold group g.
#include <float.h>
#include <math.h>

#include "fbmoe_common.cuh"
#include "fbmoe_launch.h"
#include "moe_route.cuh"

namespace fbmoe {
namespace {

constexpr int kWarpsPerBlock = 8;

__global__ void __launch_bounds__(kWarpsPerBlock * 32) route_kernel(const float* __restrict__ logits,
                                                                    const __nv_bfloat16* __restrict__ bias,
                                                                    int T, float scale, int32_t* __restrict__ topk_idx,
                                                                    float* __restrict__ topk_w,
                                                                    uint32_t* __restrict__ status) {
  __shared__ float sh_v[kWarpsPerBlock][kExperts];
  __shared__ int sh_i[kWarpsPerBlock][kExperts];
  __shared__ float sh_s[kWarpsPerBlock][kExperts];
  __shared__ int sh_sel[kWarpsPerBlock][kTopK];

  pdl_wait();
  pdl_trigger();
  if (blockIdx.x == 0 && threadIdx.x == 0 && status != nullptr) status[0] = 0u;

  const int warp = threadIdx.x >> 5;
  int t = blockIdx.x * kWarpsPerBlock + warp;
  float x[8];
  if (t < T) route_dev::load_logits8(logits, t, x);  // issued before the bias load: both in flight together
  float bs[8];
  route_dev::load_bias8(bias, bs);
  for (; t < T; t += gridDim.x * kWarpsPerBlock) {
    route_dev::route_token(x, t, bs, scale, topk_idx, topk_w, sh_v[warp], sh_i[warp], sh_s[warp], sh_sel[warp]);
    const int tn = t + gridDim.x * kWarpsPerBlock;
    if (tn < T) route_dev::load_logits8(logits, tn, x);
  }
}

}  // namespace

cudaError_t launch_route(const float* logits, const void* bias_bf16, int T, float scale, int32_t* topk_idx,
                         float* topk_w, uint32_t* status, cudaStream_t stream) {
  if (T <= 0) return cudaSuccess;
  int blocks = (T + kWarpsPerBlock - 1) / kWarpsPerBlock;
  if (blocks > 148 * 8) blocks = 148 * 8;
  return launch_pdl(route_kernel, dim3(blocks), dim3(kWarpsPerBlock * 32), 0, stream, logits,
                    reinterpret_cast<const __nv_bfloat16*>(bias_bf16), T, scale, topk_idx, topk_w, status);
}

}  // namespace fbmoe
