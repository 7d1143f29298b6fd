// moe_gather.cu -- copies each routed token's activation row to its permuted
// position (and its 56 1x128 scales, transposed to row-major), for GEMM1 on
// 128-row blocks.
//
// Reference counterpart: moe_permute_copy_fp8_with_scale_kernel
// (solution/triton/main.py:1241-1271), which keeps the scales in the transposed
// [56, 8T] layout.  Here the scales become row-major [row, 56] so that a GEMM
// epilogue thread, which owns one row, reads its row's scales contiguously.
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
                                                                  float* __restrict__ a_scale_perm) {
  const int lane = threadIdx.x & 31;
  pdl_wait();
  pdl_trigger();
  const int rows = *expert_poff_end;  // padded row count of all local experts
  for (int r = blockIdx.x * kWarps + (threadIdx.x >> 5); r < rows; r += gridDim.x * kWarps) {
    const int tok = row_token[r];
    if (tok < 0) continue;
    const uint4* src = reinterpret_cast<const uint4*>(hidden + (size_t)tok * kHidden);
    uint4* dst = reinterpret_cast<uint4*>(a_perm + (size_t)r * kHidden);
#pragma unroll
    for (int i = 0; i < kHidden / 16 / 32; ++i) dst[lane + 32 * i] = __ldg(src + lane + 32 * i);
    for (int kb = lane; kb < kHBlocks; kb += 32) a_scale_perm[(size_t)r * kHBlocks + kb] = __ldg(hidden_scale + (size_t)kb * T + tok);
  }
}

}  // namespace

cudaError_t launch_gather_rows(const uint8_t* hidden, const float* hidden_scale, int T, const Layout& L,
                               uint8_t* ws, cudaStream_t stream) {
  const int max_rows = L.pcap;
  int blocks = (max_rows + kWarps - 1) / kWarps;
  if (blocks > 148 * 16) blocks = 148 * 16;
  return launch_pdl(gather_rows_kernel, dim3(blocks), dim3(kWarps * 32), 0, stream, hidden, hidden_scale, T,
                    reinterpret_cast<const int32_t*>(ws + L.expert_poff) + L.e_local,
                    reinterpret_cast<const int32_t*>(ws + L.row_token), ws + L.a_perm,
                    reinterpret_cast<float*>(ws + L.a_scale_perm));
}

}  // namespace fbmoe
