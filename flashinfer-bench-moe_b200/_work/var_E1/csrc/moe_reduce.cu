// moe_reduce.cu -- per-token combine of the weighted (token, expert) rows.
//
// Reference counterpart: reduce_add_kernel_small/large (solution/triton/main.py:
// 1604-1714), which adds bf16 pair rows with bf16 __hadd2.  Here the f16 pair
// rows are summed in fp32 over the token's slots in fixed slot order
// (deterministic) and rounded to bf16 once; when GEMM2 split its K (decode) the
// planes of pair rows are added too, plane by plane.  Tokens with no local expert get a zero row, as in the reference.
#include "fbmoe_common.cuh"
#include "fbmoe_launch.h"

namespace fbmoe {
namespace {

constexpr int kReduceThreads = 128;               // 128 threads x 8 bf16 = 1024 columns
constexpr int kReduceChunks = kHidden / (kReduceThreads * 8);  // 7

template <bool kF32Out>
__global__ void __launch_bounds__(kReduceThreads) reduce_kernel(const __half* __restrict__ pair_out,
                                                                const int32_t* __restrict__ token_rows,
                                                                void* __restrict__ out_,
                                                                const int32_t* __restrict__ splits,
                                                                size_t plane_elems, uint32_t* status,
                                                                uint32_t* sink, int pcap) {
  pdl_wait();
  // the last kernel of the call: every earlier kernel's status bits are visible now
  if (blockIdx.x == 0 && blockIdx.y == 0 && threadIdx.x == 0) forward_status_to_sink(status, sink);
  const int t = blockIdx.y;
  const int col = (blockIdx.x * kReduceThreads + threadIdx.x) * 8;
  float acc[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) acc[i] = 0.0f;
  const int4* rows4 = reinterpret_cast<const int4*>(token_rows + (size_t)t * kTopK);
  const int4 ra = __ldg(rows4), rb = __ldg(rows4 + 1);
  int rows[kTopK] = {ra.x, ra.y, ra.z, ra.w, rb.x, rb.y, rb.z, rb.w};
#pragma unroll
  for (int k = 0; k < kTopK; ++k) rows[k] = dbg_row(rows[k], pcap, status);
  const int planes = splits[1];  // GEMM2 K splits: one plane of pair rows each
  for (int s = 0; s < planes; ++s)
#pragma unroll
  for (int k = 0; k < kTopK; ++k) {
    if (rows[k] >= 0) {
      const uint4 v = __ldg(reinterpret_cast<const uint4*>(pair_out + (size_t)s * plane_elems +
                                                           (size_t)rows[k] * kHidden + col));
      const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&w[i]));
        acc[2 * i] += f.x;
        acc[2 * i + 1] += f.y;
      }
    }
  }
  if constexpr (kF32Out) {
    float4* o = reinterpret_cast<float4*>(reinterpret_cast<float*>(out_) + (size_t)t * kHidden + col);
    o[0] = make_float4(acc[0], acc[1], acc[2], acc[3]);
    o[1] = make_float4(acc[4], acc[5], acc[6], acc[7]);
  } else {
    uint4 o;
    uint32_t* ow = reinterpret_cast<uint32_t*>(&o);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const __nv_bfloat162 b = __floats2bfloat162_rn(acc[2 * i], acc[2 * i + 1]);
      ow[i] = *reinterpret_cast<const uint32_t*>(&b);
    }
    *reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(out_) + (size_t)t * kHidden + col) = o;
  }
}

}  // namespace

cudaError_t launch_reduce(int T, const Layout& L, uint8_t* ws, void* out, bool f32_out, uint32_t* sink,
                          cudaStream_t stream) {
  if (T <= 0) return cudaSuccess;
  dim3 grid(kReduceChunks, T);
  const __half* pairs = reinterpret_cast<const __half*>(ws + L.pair_out);
  const int32_t* rows = reinterpret_cast<const int32_t*>(ws + L.token_rows);
  const int32_t* splits = reinterpret_cast<const int32_t*>(ws + L.splits);
  const size_t plane = (size_t)L.pcap * kHidden;
  uint32_t* status = reinterpret_cast<uint32_t*>(ws + L.status);
  if (f32_out)
    return launch_pdl(reduce_kernel<true>, grid, dim3(kReduceThreads), 0, stream, pairs, rows, out, splits, plane,
                      status, sink, L.pcap);
  return launch_pdl(reduce_kernel<false>, grid, dim3(kReduceThreads), 0, stream, pairs, rows, out, splits, plane,
                    status, sink, L.pcap);
}

}  // namespace fbmoe
