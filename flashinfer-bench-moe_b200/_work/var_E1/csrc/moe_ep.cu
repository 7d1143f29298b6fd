// moe_ep.cu -- expert parallelism with the combine fused into GEMM2 (sm_100a).
//
// Rank r of N owns experts [r * 256/N, (r+1) * 256/N) (its local_expert_offset,
// the reference operator's expert-parallel knob, solution/triton/main.py:
// 2558-2564) and tokens [r * T/N, (r+1) * T/N) of the output.  Routing is
// replicated.  Each rank runs route -> permute -> gather -> GEMM1 -> GEMM2 on
// its experts, and GEMM2's epilogue stores every pair row (token t, slot k)
// straight into the receive buffer of t's owner (NVLink peer memory through
// CUDA IPC), so the exchange overlaps the GEMM; there is no fp32 partial and no
// reduce-scatter.  A one-thread kernel then releases this rank's flag on every
// peer.  The owner waits for all N flags and sums each token's 8 slots in slot
// order, fp32, one bf16 rounding: the same values in the same order as the
// single-GPU reduce, so the result equals the single-GPU operator bit for bit.
//
// Receive buffer of a rank (fbmoe_ep_recv_bytes): a 256-byte header of flags
// (uint32 per source rank, the epoch of that rank's last completed send), then
// two pair regions [T/N][8][7168] f16 used by alternate epochs.  Two regions
// suffice: a rank writes region e % 2 for epoch e only after its own combine of
// epoch e - 1, which waited for every peer's send of e - 1, which each peer
// issued after its combine of e - 2 (the last reader of that region).
//
// Token dispatch (fbmoe_forward_ep_dispatch*): rank r holds only its own T/N
// tokens (logits, fp8 rows, scales).  It routes them, then writes every token's
// top-8 (ids and weights, 64 bytes) into every rank's dispatch buffer and the
// token's fp8 row and 56 scales only into the ranks that own one of its experts,
// at the token's global index; then releases its dispatch flag on every peer.
// Each rank waits for all dispatch flags and runs permute -> gather -> GEMM1 ->
// GEMM2 over the global token space with that routing (rows of tokens without a
// local expert are never read), GEMM2 scattering pair rows back to the tokens'
// home ranks as above.  Dispatch regions alternate by epoch parity for the same
// reason as the pair regions (a rank dispatches epoch e only after its combine
// of e - 1, which follows every peer's GEMM2 of e - 1, which follows that
// peer's gather of e - 2).  Layout of a rank's dispatch buffer
// (fbmoe_ep_dispatch_bytes): 256-byte flag header, then two regions of
// rows e4m3 [T][7168] | scales fp32 [56][T] | ids int32 [T][8] | weights fp32 [T][8].
#include <string.h>

#include "fbmoe.h"
#include "fbmoe_common.cuh"
#include "fbmoe_launch.h"

namespace fbmoe {
namespace {

constexpr size_t kEpHeader = 256;
constexpr uint64_t kPeerWaitNs = 4000000000ull;
constexpr int kCombineThreads = 256;

size_t ep_pair_bytes(int rows_per_rank) { return (size_t)rows_per_rank * kTopK * kHidden * 2; }
__host__ __device__ inline size_t ep_dispatch_region_bytes(int T) { return (size_t)T * (kHidden + kHBlocks * 4 + kTopK * 8); }

// One rank's dispatch region of the current epoch, and its four arrays.
struct DispatchRegion {
  uint8_t* rows;
  float* scales;
  int32_t* idx;
  float* w;
};
__host__ __device__ inline DispatchRegion dispatch_region(void* buf, int T, uint32_t epoch) {
  uint8_t* base = static_cast<uint8_t*>(buf) + kEpHeader + (size_t)(epoch & 1u) * ep_dispatch_region_bytes(T);
  DispatchRegion d;
  d.rows = base;
  d.scales = reinterpret_cast<float*>(base + (size_t)T * kHidden);
  d.idx = reinterpret_cast<int32_t*>(base + (size_t)T * (kHidden + kHBlocks * 4));
  d.w = reinterpret_cast<float*>(base + (size_t)T * (kHidden + kHBlocks * 4 + kTopK * 4));
  return d;
}
struct DispatchTable {
  DispatchRegion dst[kMaxPeers];
};

struct FlagTable {
  uint32_t* f[kMaxPeers];
};

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Launched without programmatic serialization: GEMM2 has completed, and its
// epilogue threads fenced their peer stores at system scope.
__global__ void ep_signal_kernel(const FlagTable ft, int world, uint32_t epoch) {
  if (threadIdx.x != 0) return;
  __threadfence_system();
  for (int p = 0; p < world; ++p) st_release_sys(ft.f[p], epoch);
}

// out[t, 8c .. 8c+7] for this rank's tokens, after every source rank's flag
// reached `epoch`.  Grid-stride over (token, 8-column group) tasks.
__global__ void __launch_bounds__(kCombineThreads) ep_combine_kernel(const uint32_t* flags, int world, uint32_t epoch,
                                                                   const __half* pairs, int rows,
                                                                   __nv_bfloat16* __restrict__ out,
                                                                   uint32_t* status, uint32_t* sink) {
  __shared__ int ok;
  if (threadIdx.x == 0) {
    int good = 1;
    const uint64_t t0 = globaltimer_ns();
    for (int s = 0; s < world && good; ++s) {
      while ((int)(ld_acquire_sys(flags + s) - epoch) < 0) {
        if (globaltimer_ns() - t0 > kPeerWaitNs) {
          good = 0;
          break;
        }
        __nanosleep(256);
      }
    }
    if (!good) atomicOr(status, kStatusTimeoutPeer);
    ok = good;
    // the last kernel of the call on this rank (its own send kernels have completed)
    if (blockIdx.x == 0 || !good) forward_status_to_sink(status, sink);
  }
  __syncthreads();
  if (!ok) return;
  constexpr int kGroups = kHidden / 8;
  const long tasks = (long)rows * kGroups;
  for (long task = (long)blockIdx.x * kCombineThreads + threadIdx.x; task < tasks;
       task += (long)gridDim.x * kCombineThreads) {
    const long t = task / kGroups;
    const int col = (int)(task % kGroups) * 8;
    const __half* src = pairs + (size_t)t * kTopK * kHidden + col;
    uint4 v[kTopK];
#pragma unroll
    for (int k = 0; k < kTopK; ++k) v[k] = __ldcg(reinterpret_cast<const uint4*>(src + (size_t)k * kHidden));
    float acc[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) acc[i] = 0.0f;
#pragma unroll
    for (int k = 0; k < kTopK; ++k) {  // slot order, as the single-GPU reduce
      const uint32_t w[4] = {v[k].x, v[k].y, v[k].z, v[k].w};
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&w[i]));
        acc[2 * i] += f.x;
        acc[2 * i + 1] += f.y;
      }
    }
    uint4 o;
    uint32_t* ow = reinterpret_cast<uint32_t*>(&o);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const __nv_bfloat162 b = __floats2bfloat162_rn(acc[2 * i], acc[2 * i + 1]);
      ow[i] = *reinterpret_cast<const uint32_t*>(&b);
    }
    *reinterpret_cast<uint4*>(out + (size_t)t * kHidden + col) = o;
  }
}

// A warp per local token t (global index rank * T_r + t): its top-8 to every
// rank, its fp8 row and 56 scales to the ranks that own one of its experts.
constexpr int kDispatchWarps = 8;
__global__ void __launch_bounds__(kDispatchWarps * 32) ep_dispatch_kernel(
    const int32_t* __restrict__ idx, const float* __restrict__ w, const uint8_t* __restrict__ hidden,
    const float* __restrict__ hidden_scale, int T_r, int T, int rank, int world, int E_local, const DispatchTable dt) {
  pdl_wait();
  const int lane = threadIdx.x & 31;
  const int t = blockIdx.x * kDispatchWarps + (threadIdx.x >> 5);
  if (t < T_r) {
    const int g = rank * T_r + t;
    const int e = lane < kTopK ? __ldg(idx + (size_t)t * kTopK + lane) : -1;
    const float wt = lane < kTopK ? __ldg(w + (size_t)t * kTopK + lane) : 0.0f;
    const int d = (e >= 0 && e < kExperts) ? e / E_local : -1;
    uint32_t mask = 0;
#pragma unroll
    for (int k = 0; k < kTopK; ++k) {
      const int dk = __shfl_sync(0xffffffffu, d, k);
      if (dk >= 0 && dk < world) mask |= 1u << dk;
    }
    const uint4* src = reinterpret_cast<const uint4*>(hidden + (size_t)t * kHidden);
    uint4 row[kHidden / 16 / 32];
#pragma unroll
    for (int c = 0; c < kHidden / 16 / 32; ++c) row[c] = __ldg(src + lane + 32 * c);
    const float sc0 = __ldg(hidden_scale + (size_t)lane * T_r + t);
    const float sc1 = lane + 32 < kHBlocks ? __ldg(hidden_scale + (size_t)(lane + 32) * T_r + t) : 0.0f;
    for (int o = 0; o < world; ++o) {
      const DispatchRegion& r = dt.dst[o];
      if (lane < kTopK) {
        r.idx[(size_t)g * kTopK + lane] = e;
        r.w[(size_t)g * kTopK + lane] = wt;
      }
      if ((mask >> o) & 1u) {
        uint4* dst = reinterpret_cast<uint4*>(r.rows + (size_t)g * kHidden);
#pragma unroll
        for (int c = 0; c < kHidden / 16 / 32; ++c) dst[lane + 32 * c] = row[c];
        r.scales[(size_t)lane * T + g] = sc0;
        if (lane + 32 < kHBlocks) r.scales[(size_t)(lane + 32) * T + g] = sc1;
      }
    }
  }
  __threadfence_system();  // ordered before the flag release that follows this kernel
}

// Waits until every source rank's flag reached `epoch` (bounded; status bit 7 on expiry).
__global__ void ep_wait_kernel(const uint32_t* flags, int world, uint32_t epoch, uint32_t* status) {
  if (threadIdx.x != 0) return;
  const uint64_t t0 = globaltimer_ns();
  for (int s = 0; s < world; ++s) {
    while ((int)(ld_acquire_sys(flags + s) - epoch) < 0) {
      if (globaltimer_ns() - t0 > kPeerWaitNs) {
        atomicOr(status, kStatusTimeoutPeer);
        return;
      }
      __nanosleep(256);
    }
  }
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

int check_shape(int T, int E_local, int local_expert_offset, int rank, int world) {
  if (world < 1 || world > kMaxPeers || rank < 0 || rank >= world) return FBMOE_ERR_INVALID_ARG;
  if (T < 0 || T % world != 0) return FBMOE_ERR_INVALID_ARG;
  if (E_local * world != kExperts || local_expert_offset != rank * E_local) return FBMOE_ERR_INVALID_ARG;
  return FBMOE_OK;
}

int from_cuda_ep(cudaError_t e) { return e == cudaSuccess ? FBMOE_OK : (int)e; }

}  // namespace
}  // namespace fbmoe

using namespace fbmoe;

extern "C" {

size_t fbmoe_ep_recv_bytes(int T, int world) {
  if (world < 1 || world > kMaxPeers || T < 0 || T % world != 0) return 0;
  return kEpHeader + 2 * ep_pair_bytes(T / world);
}

size_t fbmoe_ep_workspace_size(int T, int E_local) {
  if (T < 0 || E_local < 1 || E_local > kExperts) return 0;
  return make_layout(T, E_local, false, 128).total;
}

int fbmoe_forward_ep_send(const float* routing_logits, const void* routing_bias, const void* hidden_states,
                          const float* hidden_states_scale, const void* gemm1_weights,
                          const float* gemm1_weights_scale, const void* gemm2_weights,
                          const float* gemm2_weights_scale, int T, int E_local, int local_expert_offset,
                          float routed_scaling_factor, int rank, int world, void* const* peer_recv, uint32_t epoch,
                          void* workspace, size_t workspace_bytes, void* stream) {
  int rc = check_shape(T, E_local, local_expert_offset, rank, world);
  if (rc) return rc;
  if (epoch == 0) return FBMOE_ERR_INVALID_ARG;
  if (peer_recv == nullptr) return FBMOE_ERR_NULL_POINTER;
  for (int o = 0; o < world; ++o) {
    if (peer_recv[o] == nullptr) return FBMOE_ERR_NULL_POINTER;
    if (!aligned16(peer_recv[o])) return FBMOE_ERR_MISALIGNED;
  }
  if (T == 0) return FBMOE_OK;
  const int rows = T / world;
  const size_t region = kEpHeader + (size_t)(epoch & 1u) * ep_pair_bytes(rows);
  PeerScatter ps{};
  FlagTable ft{};
  for (int o = 0; o < world; ++o) {
    uint8_t* base = static_cast<uint8_t*>(peer_recv[o]);
    ps.base[o] = reinterpret_cast<__half*>(base + region);
    ft.f[o] = reinterpret_cast<uint32_t*>(base) + rank;
  }
  ps.rows_per_rank = rows;
  ps.world = world;
  rc = forward_core(routing_logits, routing_bias, hidden_states, hidden_states_scale, gemm1_weights,
                    gemm1_weights_scale, gemm2_weights, gemm2_weights_scale, T, E_local, local_expert_offset,
                    routed_scaling_factor, nullptr, false, workspace, workspace_bytes, stream, false, &ps);
  if (rc) return rc;
  ep_signal_kernel<<<1, 32, 0, reinterpret_cast<cudaStream_t>(stream)>>>(ft, world, epoch);
  return from_cuda_ep(cudaGetLastError());
}

int fbmoe_forward_ep_recv(const void* my_recv, int T, int rank, int world, uint32_t epoch, void* out_rows_bf16,
                          void* workspace, void* stream) {
  if (world < 1 || world > kMaxPeers || rank < 0 || rank >= world || T < 0 || T % world != 0 || epoch == 0)
    return FBMOE_ERR_INVALID_ARG;
  if (T == 0) return FBMOE_OK;
  if (!my_recv || !out_rows_bf16 || !workspace) return FBMOE_ERR_NULL_POINTER;
  if (!aligned16(my_recv) || !aligned16(out_rows_bf16)) return FBMOE_ERR_MISALIGNED;
  const int rows = T / world;
  const uint8_t* base = static_cast<const uint8_t*>(my_recv);
  const __half* pairs = reinterpret_cast<const __half*>(base + kEpHeader + (size_t)(epoch & 1u) * ep_pair_bytes(rows));
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const long tasks = (long)rows * (kHidden / 8);
  long grid = (tasks + kCombineThreads - 1) / kCombineThreads;
  if (grid > (long)sms * 8) grid = (long)sms * 8;
  ep_combine_kernel<<<(unsigned)grid, kCombineThreads, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      reinterpret_cast<const uint32_t*>(base), world, epoch, pairs, rows,
      static_cast<__nv_bfloat16*>(out_rows_bf16), static_cast<uint32_t*>(workspace), status_sink_for(workspace));
  return from_cuda_ep(cudaGetLastError());
}

int fbmoe_forward_ep(const float* routing_logits, const void* routing_bias, const void* hidden_states,
                     const float* hidden_states_scale, const void* gemm1_weights, const float* gemm1_weights_scale,
                     const void* gemm2_weights, const float* gemm2_weights_scale, int T, int E_local,
                     int local_expert_offset, float routed_scaling_factor, int rank, int world,
                     void* const* peer_recv, uint32_t epoch, void* out_rows_bf16, void* workspace,
                     size_t workspace_bytes, void* stream) {
  int rc = fbmoe_forward_ep_send(routing_logits, routing_bias, hidden_states, hidden_states_scale, gemm1_weights,
                                 gemm1_weights_scale, gemm2_weights, gemm2_weights_scale, T, E_local,
                                 local_expert_offset, routed_scaling_factor, rank, world, peer_recv, epoch, workspace,
                                 workspace_bytes, stream);
  if (rc) return rc;
  return fbmoe_forward_ep_recv(peer_recv[rank], T, rank, world, epoch, out_rows_bf16, workspace, stream);
}

size_t fbmoe_ep_dispatch_bytes(int T, int world) {
  if (world < 1 || world > kMaxPeers || T < 0 || T % world != 0) return 0;
  return kEpHeader + 2 * ep_dispatch_region_bytes(T);
}

int fbmoe_forward_ep_dispatch_send(const float* routing_logits, const void* routing_bias, const void* hidden_states,
                                   const float* hidden_states_scale, int T, int E_local, float routed_scaling_factor,
                                   int rank, int world, void* const* peer_dispatch, uint32_t epoch, void* workspace,
                                   size_t workspace_bytes, void* stream_) {
  int rc = check_shape(T, E_local, rank * E_local, rank, world);
  if (rc) return rc;
  if (epoch == 0) return FBMOE_ERR_INVALID_ARG;
  if (!peer_dispatch || !workspace) return FBMOE_ERR_NULL_POINTER;
  for (int o = 0; o < world; ++o) {
    if (peer_dispatch[o] == nullptr) return FBMOE_ERR_NULL_POINTER;
    if (!aligned16(peer_dispatch[o])) return FBMOE_ERR_MISALIGNED;
  }
  if (T == 0) return FBMOE_OK;
  if (!routing_logits || !routing_bias || !hidden_states || !hidden_states_scale) return FBMOE_ERR_NULL_POINTER;
  if (!aligned16(routing_logits) || !aligned16(routing_bias) || !aligned16(hidden_states) ||
      (reinterpret_cast<uintptr_t>(workspace) & 255u))
    return FBMOE_ERR_MISALIGNED;
  const Layout L = make_layout(T, E_local, false, 128);
  if (workspace_bytes < L.total) return FBMOE_ERR_WORKSPACE_TOO_SMALL;
  cudaStream_t stream = reinterpret_cast<cudaStream_t>(stream_);
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  const int T_r = T / world;
  // this rank's tokens' routing, in the workspace's routing arrays (the router also clears the status word)
  int32_t* idx = reinterpret_cast<int32_t*>(ws + L.topk_idx);
  float* w = reinterpret_cast<float*>(ws + L.topk_w);
  cudaError_t e = launch_route(routing_logits, routing_bias, T_r, routed_scaling_factor, idx, w,
                               reinterpret_cast<uint32_t*>(ws + L.status), stream);
  if (e != cudaSuccess) return from_cuda_ep(e);
  DispatchTable dt{};
  FlagTable ft{};
  for (int o = 0; o < world; ++o) {
    dt.dst[o] = dispatch_region(peer_dispatch[o], T, epoch);
    ft.f[o] = static_cast<uint32_t*>(peer_dispatch[o]) + rank;
  }
  e = launch_pdl(ep_dispatch_kernel, dim3((T_r + kDispatchWarps - 1) / kDispatchWarps), dim3(kDispatchWarps * 32), 0,
                 stream, static_cast<const int32_t*>(idx), static_cast<const float*>(w),
                 static_cast<const uint8_t*>(hidden_states), hidden_states_scale, T_r, T, rank, world, E_local, dt);
  if (e != cudaSuccess) return from_cuda_ep(e);
  ep_signal_kernel<<<1, 32, 0, stream>>>(ft, world, epoch);
  return from_cuda_ep(cudaGetLastError());
}

int fbmoe_forward_ep_dispatch_compute(const void* gemm1_weights, const float* gemm1_weights_scale,
                                      const void* gemm2_weights, const float* gemm2_weights_scale, int T, int E_local,
                                      int rank, int world, void* my_dispatch, void* const* peer_recv, uint32_t epoch,
                                      void* workspace, size_t workspace_bytes, void* stream_) {
  int rc = check_shape(T, E_local, rank * E_local, rank, world);
  if (rc) return rc;
  if (epoch == 0) return FBMOE_ERR_INVALID_ARG;
  if (!my_dispatch || !peer_recv || !workspace) return FBMOE_ERR_NULL_POINTER;
  for (int o = 0; o < world; ++o) {
    if (peer_recv[o] == nullptr) return FBMOE_ERR_NULL_POINTER;
    if (!aligned16(peer_recv[o])) return FBMOE_ERR_MISALIGNED;
  }
  if (!aligned16(my_dispatch)) return FBMOE_ERR_MISALIGNED;
  if (T == 0) return FBMOE_OK;
  cudaStream_t stream = reinterpret_cast<cudaStream_t>(stream_);
  const Layout L = make_layout(T, E_local, false, 128);
  if (workspace_bytes < L.total) return FBMOE_ERR_WORKSPACE_TOO_SMALL;
  ep_wait_kernel<<<1, 32, 0, stream>>>(static_cast<const uint32_t*>(my_dispatch), world, epoch,
                                       reinterpret_cast<uint32_t*>(static_cast<uint8_t*>(workspace) + L.status));
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return from_cuda_ep(e);
  const DispatchRegion d = dispatch_region(my_dispatch, T, epoch);
  const int rows = T / world;
  const size_t region = kEpHeader + (size_t)(epoch & 1u) * ep_pair_bytes(rows);
  PeerScatter ps{};
  FlagTable ft{};
  for (int o = 0; o < world; ++o) {
    uint8_t* base = static_cast<uint8_t*>(peer_recv[o]);
    ps.base[o] = reinterpret_cast<__half*>(base + region);
    ft.f[o] = reinterpret_cast<uint32_t*>(base) + rank;
  }
  ps.rows_per_rank = rows;
  ps.world = world;
  rc = forward_core(nullptr, nullptr, d.rows, d.scales, gemm1_weights, gemm1_weights_scale, gemm2_weights,
                    gemm2_weights_scale, T, E_local, rank * E_local, 1.0f, nullptr, false, workspace,
                    workspace_bytes, stream, false, &ps, d.idx, d.w);
  if (rc) return rc;
  ep_signal_kernel<<<1, 32, 0, stream>>>(ft, world, epoch);
  return from_cuda_ep(cudaGetLastError());
}

int fbmoe_forward_ep_dispatch(const float* routing_logits, const void* routing_bias, const void* hidden_states,
                              const float* hidden_states_scale, const void* gemm1_weights,
                              const float* gemm1_weights_scale, const void* gemm2_weights,
                              const float* gemm2_weights_scale, int T, int E_local, float routed_scaling_factor,
                              int rank, int world, void* const* peer_dispatch, void* const* peer_recv, uint32_t epoch,
                              void* out_rows_bf16, void* workspace, size_t workspace_bytes, void* stream) {
  int rc = fbmoe_forward_ep_dispatch_send(routing_logits, routing_bias, hidden_states, hidden_states_scale, T, E_local,
                                          routed_scaling_factor, rank, world, peer_dispatch, epoch, workspace,
                                          workspace_bytes, stream);
  if (rc) return rc;
  rc = fbmoe_forward_ep_dispatch_compute(gemm1_weights, gemm1_weights_scale, gemm2_weights, gemm2_weights_scale, T,
                                         E_local, rank, world, peer_dispatch[rank], peer_recv, epoch, workspace,
                                         workspace_bytes, stream);
  if (rc) return rc;
  return fbmoe_forward_ep_recv(peer_recv[rank], T, rank, world, epoch, out_rows_bf16, workspace, stream);
}

int fbmoe_ipc_alloc(size_t bytes, void** ptr) {
  if (!ptr) return FBMOE_ERR_NULL_POINTER;
  *ptr = nullptr;
  if (bytes == 0) return FBMOE_ERR_INVALID_ARG;
  cudaError_t e = cudaMalloc(ptr, bytes);
  if (e == cudaSuccess) e = cudaMemset(*ptr, 0, bytes);
  return from_cuda_ep(e);
}

int fbmoe_ipc_free(void* ptr) { return ptr ? from_cuda_ep(cudaFree(ptr)) : FBMOE_OK; }

int fbmoe_ipc_handle(const void* ptr, void* handle_out) {
  if (!ptr || !handle_out) return FBMOE_ERR_NULL_POINTER;
  cudaIpcMemHandle_t h;
  cudaError_t e = cudaIpcGetMemHandle(&h, const_cast<void*>(ptr));
  if (e != cudaSuccess) return from_cuda_ep(e);
  memcpy(handle_out, &h, sizeof h);
  return FBMOE_OK;
}

int fbmoe_ipc_open(const void* handle, void** ptr) {
  if (!handle || !ptr) return FBMOE_ERR_NULL_POINTER;
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof h);
  *ptr = nullptr;
  return from_cuda_ep(cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess));
}

int fbmoe_ipc_close(void* ptr) { return ptr ? from_cuda_ep(cudaIpcCloseMemHandle(ptr)) : FBMOE_OK; }

}  // extern "C"
