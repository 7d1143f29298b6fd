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
// next task's loads are issued before the current one is converted.  14,336 B
// read + 7,168 B + 224 B written per row.
//
// Arithmetic.  The kernel is bound by instruction issue, not by HBM, unless the
// per-element work stays small, so no IEEE division runs on the common path:
// * scale: s = RN(amax / 448) as q0 = RN(amax * c), c = RN(1/448), then
//   s = RN(q0 + RN(amax - q0 * 448) * c) (two FMAs);
// * reciprocal: r = RN(1 / s) as one Newton step from rcp.approx,
//   r = RN(r0 + RN(1 - s * r0) * r0);
// * quotient: Markstein's correction (P. Markstein, "Computation of elementary
//   functions on the IBM RISC System/6000 processor", IBM J. Res. Dev. 34(1),
//   1990): y0 = RN(x * r), e = RN(x - y0 * s), z = RN(y0 + e * r), two elements
//   per packed f32x2 instruction.  y0 can be 1.5 ulps from x / s, so z is not
//   always RN(x / s); what holds is e4m3(z) == e4m3(RN(x / s)).
// All three were checked exhaustively on a B200 against IEEE division: every finite
// positive bf16 amax (scale and reciprocal bit for bit), and the e4m3 byte of every
// bf16 x with |x| <= amax for each of those amax whose scale takes this path
// (981,047,200 pairs, 0 differences); the GPU tests sweep the same domain through
// this kernel.
// The path needs amax finite and s >= 2^-64 (so that the residual and the
// reciprocal stay normal); other blocks (9,183 of the 32,639 finite amax values,
// all below 2.42e-17, and blocks holding an infinity) divide exactly per element.
// z = +0 for x = -0 (an exact-zero residual drops the sign), so each element's
// sign bit is carried into its e4m3 byte.  A NaN element converts to an e4m3 NaN
// that keeps its sign; NaNs do not enter amax (fmaxf).
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

// RN(amax / 448) for every finite positive bf16 amax.
__device__ __forceinline__ float scale_of_amax(float amax) {
  const float c = 1.0f / 448.0f;
  const float q0 = amax * c;
  return fmaf(fmaf(-q0, 448.0f, amax), c, q0);
}

// RN(1 / s) for every scale the fast path takes.
__device__ __forceinline__ float rcp_rn_newton(float s) {
  float r0;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r0) : "f"(s));
  return fmaf(fmaf(-s, r0, 1.0f), r0, r0);
}

constexpr float kBf16Max = 3.3895313892515355e38f;
constexpr float kFastMinScale = 5.421010862427522e-20f;  // 2^-64

// e4m3 of RN(a / s), RN(b / s): rr = (r, r), nss = (-s, -s).
__device__ __forceinline__ uint32_t e4m3x2_markstein(float a, float b, uint64_t rr, uint64_t nss) {
  const uint64_t x = f32x2_pack(a, b);
  const uint64_t y = f32x2_mul(x, rr);
  uint64_t e = x;
  f32x2_fma(e, y, nss);  // x - y * s
  uint64_t z = y;
  f32x2_fma(z, e, rr);   // y + e * r
  float za, zb;
  f32x2_unpack(z, za, zb);
  return e4m3x2_of(za, zb);
}

__device__ __forceinline__ void load_task(const __nv_bfloat16* __restrict__ x, long task, long n_tasks, int lane,
                                          uint4 (&v)[kLoads]) {
  if (task >= n_tasks) return;
  constexpr int kGroupsPerRow = kHBlocks / kGroup;
  const int t = (int)(task / kGroupsPerRow), kb0 = (int)(task % kGroupsPerRow) * kGroup;
  const __nv_bfloat16* p = x + (size_t)t * kHidden + (size_t)kb0 * kBlk + (lane >> 4) * kBlk + (lane & 15) * 8;
#pragma unroll
  for (int j = 0; j < kLoads; ++j) v[j] = __ldg(reinterpret_cast<const uint4*>(p + 2 * j * kBlk));
}

// 64 registers: four CTAs of 256 threads per SM.
__global__ void __launch_bounds__(kWarps * 32, 4) quant_act_kernel(const __nv_bfloat16* __restrict__ x, int T,
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
      float s = m > 0.0f ? scale_of_amax(m) : 1.0f;
      uint32_t lo, hi;
      if (m <= kBf16Max && s >= kFastMinScale) {
        const float r = rcp_rn_newton(s);
        const uint64_t rr = f32x2_pack(r, r), nss = f32x2_pack(-s, -s);
        lo = e4m3x2_markstein(v[0], v[1], rr, nss) | (e4m3x2_markstein(v[2], v[3], rr, nss) << 16);
        hi = e4m3x2_markstein(v[4], v[5], rr, nss) | (e4m3x2_markstein(v[6], v[7], rr, nss) << 16);
        // byte k of lo/hi takes the sign bit of element k (bits 15 / 31 of the bf16 pairs)
        lo |= __byte_perm(w[0], w[1], 0x7531) & 0x80808080u;
        hi |= __byte_perm(w[2], w[3], 0x7531) & 0x80808080u;
      } else {
        s = m > 0.0f ? __fdiv_rn(m, 448.0f) : 1.0f;
        uint32_t p[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) p[i] = e4m3x2_of(__fdiv_rn(v[2 * i], s), __fdiv_rn(v[2 * i + 1], s));
        lo = p[0] | (p[1] << 16);
        hi = p[2] | (p[3] << 16);
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
  if (blocks > 148L * 4) blocks = 148L * 4;  // one wave of four CTAs per SM
  const cudaError_t e = fbmoe::launch_pdl(fbmoe::quant_act_kernel, dim3((unsigned)blocks), dim3(fbmoe::kWarps * 32),
                                          0, reinterpret_cast<cudaStream_t>(stream),
                                          reinterpret_cast<const __nv_bfloat16*>(x_bf16), T,
                                          reinterpret_cast<uint8_t*>(q_e4m3), scale);
  return e == cudaSuccess ? FBMOE_OK : (int)e;
}
