// moe_gather.cu -- copies each routed token's activation row to its permuted
// position (and its 56 1x128 scales), for GEMM1 on 128-row blocks.
//
// Reference counterpart: moe_permute_copy_fp8_with_scale_kernel
// (solution/triton/main.py:1241-1271), which also keeps the scales in the
// transposed [56, rows] layout: GEMM1 loads, per K-block, the 128 scales of a
// row block as one 512-byte TMA box.
// A materialised copy costs 2 x 7 KB of HBM traffic per routed row; it lets
// GEMM1 load each 128-row x 128-K tile with one TMA box instead of 32 row
// gathers, which on B200 halved GEMM1's throughput (measured: 2.68 ms with
// row gathers vs 1.32 ms with a plain 2-D box for the same bytes).
// Padding rows (row_token < 0) are skipped: the GEMM never stores their results.
#include "fbmoe_common.cuh"
#include "fbmoe_launch.h"

namespace fbmoe {
namespace {

constexpr int kWarps = 8;

__global__ void __launch_bounds__(kWarps * 32) gather_rows_kernel(const uint8_t* __restrict__ hidden,
                                                                  const float* __restrict__ hidden_scale, int T,
                                                                  const int32_t* __restrict__ expert_poff_end,
                                                                  const int32_t* __restrict__ row_token,
                                                                  uint8_t* __restrict__ a_perm,
                                                                  float* __restrict__ a_scale_perm, int pcap,
                                                                  uint32_t* __restrict__ status) {
  const int lane = threadIdx.x & 31;
  pdl_wait();
  pdl_trigger();
  const int rows = *expert_poff_end;  // padded row count of all local experts
  // a warp per group of 32 rows: the scales with lane = row (coalesced stores),
  // then the 32 activation rows one after another
  for (int r0 = (blockIdx.x * kWarps + (threadIdx.x >> 5)) * 32; r0 < rows; r0 += gridDim.x * kWarps * 32) {
    const int my_tok = r0 + lane < rows ? dbg_row(row_token[r0 + lane], T, status) : -1;
    for (int kb = 0; kb < kHBlocks; ++kb)
      if (r0 + lane < rows)
        a_scale_perm[(size_t)kb * pcap + r0 + lane] = my_tok >= 0 ? __ldg(hidden_scale + (size_t)kb * T + my_tok) : 0.0f;
    for (int i = 0; i < 32 && r0 + i < rows; ++i) {
      const int tok = __shfl_sync(0xffffffffu, my_tok, i);
      if (tok < 0) continue;
      const uint4* src = reinterpret_cast<const uint4*>(hidden + (size_t)tok * kHidden);
      uint4* dst = reinterpret_cast<uint4*>(a_perm + (size_t)(r0 + i) * kHidden);
#pragma unroll
      for (int c = 0; c < kHidden / 16 / 32; ++c) dst[lane + 32 * c] = __ldg(src + lane + 32 * c);
    }
  }
}

}  // namespace

cudaError_t launch_gather_rows(const uint8_t* hidden, const float* hidden_scale, int T, const Layout& L,
                               uint8_t* ws, cudaStream_t stream) {
  const int groups = (L.pcap + 31) / 32;
  int blocks = (groups + kWarps - 1) / kWarps;
  if (blocks > 148 * 8) blocks = 148 * 8;
  return launch_pdl(gather_rows_kernel, dim3(blocks), dim3(kWarps * 32), 0, stream, hidden, hidden_scale, T,
                    reinterpret_cast<const int32_t*>(ws + L.expert_poff) + L.e_local,
                    reinterpret_cast<const int32_t*>(ws + L.row_token), ws + L.a_perm,
                    reinterpret_cast<float*>(ws + L.a_scale_perm), L.pcap,
                    reinterpret_cast<uint32_t*>(ws + L.status));
}

}  // namespace fbmoe
