// moe_capi.cu -- the C ABI (include/fbmoe.h): argument checks, workspace
// layout, TMA descriptors and the launch chain of the fused MoE forward.
//
// Launch chain of fbmoe_forward (reference fused_moe, solution/triton/main.py:
// 2668-2774, five stages):
//   route -> permute (histogram / padded scan / deterministic scatter)
//         -> GEMM1 + SwiGLU (tcgen05) -> GEMM2 x weight (tcgen05) -> combine.
// Nothing synchronises the host and nothing allocates device memory; the caller
// owns the workspace (the reference keeps a module-global 15000-token one).
#include <cudaTypedefs.h>
#include <stdio.h>
#include <string.h>

#include <atomic>
#include <mutex>

#include "fbmoe.h"
#include "fbmoe_common.cuh"
#include "fbmoe_launch.h"

namespace fbmoe {

static size_t align_up(size_t x, size_t a) { return (x + a - 1) / a * a; }

// Rows per GEMM block.  16 selects the swap-AB decode kernels (weights as the
// 128-row MMA operand, up to 16 tokens as N, device-chosen split-K); 128 selects
// the row-major kernels (128 permuted rows as M, 256 weight rows as N).  A
// swap-AB block re-streams its expert's weights for every 16 rows, so it only
// pays while experts see few rows: on B200 the row-major kernels were already
// faster at T = 80 under every routing tried (uniform, one hot group, 4 hot
// experts), and 3-8x faster at T = 1024..4096 under skewed routing.
int choose_block_rows(int T, int E_local) {
  (void)E_local;
  return T <= 64 ? 16 : 128;
}

Layout make_layout(int T, int E_local, bool allow_split, int force_rows) {
  Layout L;
  const size_t tt = (size_t)(T > 0 ? T : 0);
  L.tokens = (int)tt;
  const int el = E_local > 0 ? E_local : 0;
  long pcap = (long)tt * kTopK + (long)kRowAlign * el;
  pcap = (long)align_up((size_t)pcap, 128);
  if (pcap < 128) pcap = 128;
  L.pcap = (int)pcap;
  L.max_blocks = (int)(pcap / kRowAlign);
  size_t off = 0;
  auto take = [&](size_t bytes) {
    const size_t o = off;
    off = align_up(off + bytes, 256);
    return o;
  };
  L.status = take(16);
  L.topk_idx = take(tt * kTopK * 4);
  L.topk_w = take(tt * kTopK * 4);
  L.token_rows = take(tt * kTopK * 4);
  L.expert_cnt = take((size_t)el * 4);
  L.expert_poff = take((size_t)(el + 1) * 4);
  L.n_blocks = take(16);
  L.blocks = take((size_t)L.max_blocks * 16);
  L.row_token = take((size_t)pcap * 4);
  L.row_weight = take((size_t)pcap * 4);
  L.inter = take((size_t)pcap * kInter * 2);
  const int bn = force_rows ? force_rows : choose_block_rows(T, E_local);
  const bool split = allow_split && bn == 16;
  L.pair_planes = split ? kMaxPairPlanes : 1;
  L.split_items = split ? kSplitItems : 0;
  L.pair_out = take((size_t)pcap * kHidden * 2 * L.pair_planes);
  L.splits = take(16);
  // one arrival counter per GEMM1 unit (32 per block), for the decode kernel's stream-K fix-up
  L.split_count = take(split ? (size_t)L.max_blocks * (kInter / 64) * 4 : 0);
  L.split_part = take((size_t)L.split_items * 128 * 16 * 4);
  L.blk_ready = take((size_t)L.max_blocks * 4);
  L.grid_sync = take(16);
  const bool big = bn == 128;
  L.chunk_cnt = take((tt + 1023) / 1024 * (size_t)el * 4);
  L.a_perm = take(big ? (size_t)pcap * kHidden : 0);
  L.a_scale_perm = take(big ? (size_t)pcap * kHBlocks * 4 : 0);
  L.plane_scale = take(bn == 16 ? (size_t)2 * pcap * (kInter / 64) * 4 : 0);
  L.e_local = el;
  L.total = off;
  return L;
}


// ---------------------------------------------------------------- driver ----
static PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;
static std::once_flag g_encode_once;

static bool get_encode() {
  std::call_once(g_encode_once, [] {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
  });
  return g_encode != nullptr;
}

// 2-D K-major tile map (128-byte swizzle unless stated).  inner = K extent (elements).
static int encode_2d(CUtensorMap* map, CUtensorMapDataType dtype, int elem_bytes, const void* base, uint64_t inner,
                     uint64_t rows, uint32_t box_inner, uint32_t box_rows,
                     CUtensorMapSwizzle swizzle = CU_TENSOR_MAP_SWIZZLE_128B) {
  if (!get_encode()) return FBMOE_ERR_DRIVER;
  const cuuint64_t dims[2] = {inner, rows};
  const cuuint64_t strides[1] = {inner * (uint64_t)elem_bytes};
  const cuuint32_t box[2] = {box_inner, box_rows};
  const cuuint32_t estr[2] = {1, 1};
  CUresult r = g_encode(map, dtype, 2, const_cast<void*>(base), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? FBMOE_OK : FBMOE_ERR_DRIVER;
}

static int num_sms_of_current_device() {
  static std::atomic<int> cache[kMaxDevicesTracked];  // 0 = not looked up yet
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 148;
  const bool tracked = dev >= 0 && dev < kMaxDevicesTracked;
  if (tracked) {
    const int c = cache[dev].load(std::memory_order_relaxed);
    if (c > 0) return c;
  }
  int n = 148;
  cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  if (tracked) cache[dev].store(n, std::memory_order_relaxed);
  return n;
}

static int from_cuda(cudaError_t e) { return e == cudaSuccess ? FBMOE_OK : (int)e; }

// Optional stage timing: CUDA events recorded on the forward's stream between
// the five stages, for up to `cap` forwards (host-side only, no device memory).
constexpr int kStages = 5;
struct StageProfile {
  std::mutex mu;
  bool on = false;
  int cap = 0;
  int n = 0;
  cudaEvent_t* ev = nullptr;
};
static StageProfile g_prof;

static void prof_record(int fwd, int point, cudaStream_t stream) {
  if (fwd >= 0) cudaEventRecord(g_prof.ev[fwd * (kStages + 1) + point], stream);
}

static bool aligned(const void* p, size_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

// Status sinks: workspace -> device-visible address of a pinned host word.  A
// small table under a mutex; forward_core skips the lock while it is empty.
constexpr int kMaxSinks = 64;
struct SinkTable {
  std::mutex mu;
  std::atomic<int> n{0};
  const void* ws[kMaxSinks] = {};
  uint32_t* sink[kMaxSinks] = {};
};
static SinkTable g_sinks;

uint32_t* status_sink_for(const void* workspace) {
  if (g_sinks.n.load(std::memory_order_acquire) == 0) return nullptr;
  std::lock_guard<std::mutex> lk(g_sinks.mu);
  const int n = g_sinks.n.load(std::memory_order_relaxed);
  for (int i = 0; i < n; ++i)
    if (g_sinks.ws[i] == workspace) return g_sinks.sink[i];
  return nullptr;
}

static std::atomic<int> g_test_expire{0};
bool test_expire_grid_wait() { return g_test_expire.load(std::memory_order_relaxed) != 0; }

}  // namespace fbmoe

using namespace fbmoe;

extern "C" {

size_t fbmoe_workspace_size(int T, int E_local) {
  if (T < 0 || E_local < 1 || E_local > kExperts) return 0;
  return make_layout(T, E_local).total;
}

int fbmoe_block_rows(int T, int E_local) { return choose_block_rows(T, E_local); }

int fbmoe_workspace_layout(int T, int E_local, int64_t* offsets) {
  if (offsets == nullptr) return FBMOE_ERR_NULL_POINTER;
  if (T < 0 || E_local < 1 || E_local > kExperts) return FBMOE_ERR_INVALID_ARG;
  const Layout L = make_layout(T, E_local);
  const int64_t v[FBMOE_LAYOUT_FIELDS] = {
      (int64_t)L.status,   (int64_t)L.topk_idx,  (int64_t)L.topk_w,     (int64_t)L.token_rows, (int64_t)L.expert_cnt,
      (int64_t)L.expert_poff, (int64_t)L.n_blocks, (int64_t)L.blocks,   (int64_t)L.row_token,  (int64_t)L.row_weight,
      (int64_t)L.inter,    (int64_t)L.pair_out,  (int64_t)L.total,      (int64_t)L.pcap};
  memcpy(offsets, v, sizeof v);
  return FBMOE_OK;
}

int fbmoe_route(const float* routing_logits, const void* routing_bias, int T, float routed_scaling_factor,
                int32_t* topk_idx, float* topk_weights, void* stream) {
  if (T < 0) return FBMOE_ERR_INVALID_ARG;
  if (T == 0) return FBMOE_OK;
  if (!routing_logits || !routing_bias || !topk_idx || !topk_weights) return FBMOE_ERR_NULL_POINTER;
  if (!aligned(routing_logits, 16) || !aligned(routing_bias, 16)) return FBMOE_ERR_MISALIGNED;
  return from_cuda(launch_route(routing_logits, routing_bias, T, routed_scaling_factor, topk_idx, topk_weights,
                                nullptr, reinterpret_cast<cudaStream_t>(stream)));
}

}  // extern "C"

namespace fbmoe {
int forward_core(const float* routing_logits, const void* routing_bias, const void* hidden_states,
                 const float* hidden_states_scale, const void* gemm1_weights, const float* gemm1_weights_scale,
                 const void* gemm2_weights, const float* gemm2_weights_scale, int T, int E_local,
                 int local_expert_offset, float routed_scaling_factor, void* out, bool f32_out, void* workspace,
                 size_t workspace_bytes, void* stream_, bool allow_split, const PeerScatter* scatter,
                 const int32_t* routed_idx, const float* routed_w, bool w1_packed, bool fp8_inter) {
  if (T < 0 || E_local < 1 || E_local > kExperts) return FBMOE_ERR_INVALID_ARG;
  if (T == 0) return FBMOE_OK;
  const bool scattering = scatter != nullptr && scatter->world > 0;
  // routed_idx / routed_w: routing computed elsewhere (token-dispatch expert parallelism); no router launch
  const bool routed = routed_idx != nullptr;
  if (routed && !routed_w) return FBMOE_ERR_NULL_POINTER;
  if ((!routed && (!routing_logits || !routing_bias)) || !hidden_states || !hidden_states_scale || !gemm1_weights ||
      !gemm1_weights_scale || !gemm2_weights || !gemm2_weights_scale || (!out && !scattering) || !workspace)
    return FBMOE_ERR_NULL_POINTER;
  if ((!routed && (!aligned(routing_logits, 16) || !aligned(routing_bias, 16))) || !aligned(hidden_states, 16) ||
      !aligned(gemm1_weights, 16) || !aligned(gemm2_weights, 16) || !aligned(out, 16) || !aligned(workspace, 256) ||
      !aligned(gemm1_weights_scale, 16) || !aligned(gemm2_weights_scale, 16))  // scale rows move by bulk copies
    return FBMOE_ERR_MISALIGNED;
  // the scatter lives in the row-major GEMM2's epilogue, so it forces that chain
  const int force_rows = scattering ? 128 : 0;
  const Layout L = make_layout(T, E_local, allow_split, force_rows);
  if (workspace_bytes < L.total) return FBMOE_ERR_WORKSPACE_TOO_SMALL;
  cudaStream_t stream = reinterpret_cast<cudaStream_t>(stream_);
  uint8_t* ws = reinterpret_cast<uint8_t*>(workspace);
  const int bn = force_rows ? force_rows : choose_block_rows(T, E_local);
  const int sms = num_sms_of_current_device();
  uint32_t* sink = status_sink_for(workspace);

  CUtensorMap tm_w1, tm_w2, tm_inter, tm_w2raw, tm_aperm, tm_ascale;
  // raw W1: 64-row boxes (a tile is 2 or 4 of them); pre-packed W1: one box per
  // tile, 128 rows (decode) or 256 rows (prefill)
  const uint32_t w1_box_rows = w1_packed ? (bn == 16 ? 128u : 256u) : 64u;
  int rc = encode_2d(&tm_w1, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, gemm1_weights, kHidden, (uint64_t)E_local * kGemm1N,
                     128, w1_box_rows);
  if (rc) return rc;
  rc = encode_2d(&tm_w2, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, gemm2_weights, kInter, (uint64_t)E_local * kHidden, 128,
                 128);
  if (rc) return rc;
  if (bn == 128) {
    rc = encode_2d(&tm_aperm, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, ws + L.a_perm, kHidden, (uint64_t)L.pcap, 128, 128);
    if (rc) return rc;
    // [56][pcap] fp32 scales: one box = 128 consecutive rows of one K-block (512 bytes)
    rc = encode_2d(&tm_ascale, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, ws + L.a_scale_perm, (uint64_t)L.pcap, kHBlocks,
                   128, 1, CU_TENSOR_MAP_SWIZZLE_NONE);
    if (rc) return rc;
  }
  // W2 in 64-byte (64-K) slices of 256 rows, unswizzled: converted on chip by GEMM2.
  rc = encode_2d(&tm_w2raw, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, gemm2_weights, kInter, (uint64_t)E_local * kHidden, 64,
                 256, CU_TENSOR_MAP_SWIZZLE_NONE);
  if (rc) return rc;
  // decode (bn == 16) keeps the intermediate as two fp8 planes that its GEMM2 copies
  // with cp.async (no tensor map); prefill GEMM2 loads the f16 intermediate by TMA
  if (bn != 16) {
    rc = encode_2d(&tm_inter, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, ws + L.inter, kInter, (uint64_t)L.pcap, 64,
                   (uint32_t)bn);
    if (rc) return rc;
  }
  // fp8-intermediate mode (prefill chain): e4m3 intermediate rows in 128 x 128-byte boxes,
  // their scales [16][pcap] in 128-row boxes of one K-block, raw W2 in 64-row boxes
  const bool fp8_chain = fp8_inter && bn == 128;
  CUtensorMap tm_inter8, tm_iscale, tm_w2b;
  if (fp8_chain) {
    rc = encode_2d(&tm_inter8, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, ws + L.inter, kInter, (uint64_t)L.pcap, 128, 128);
    if (rc) return rc;
    rc = encode_2d(&tm_iscale, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, ws + L.inter + fp8_inter_scale_offset(L),
                   (uint64_t)L.pcap, kIBlocks, 128, 1, CU_TENSOR_MAP_SWIZZLE_NONE);
    if (rc) return rc;
    rc = encode_2d(&tm_w2b, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, gemm2_weights, kInter, (uint64_t)E_local * kHidden, 128,
                   64);
    if (rc) return rc;
  }

  int fwd = -1;
  if (g_prof.on) {
    std::lock_guard<std::mutex> lk(g_prof.mu);
    if (g_prof.on && g_prof.n < g_prof.cap) fwd = g_prof.n++;
  }
  const int32_t* topk_idx = routed ? routed_idx : reinterpret_cast<int32_t*>(ws + L.topk_idx);
  const float* topk_w = routed ? routed_w : reinterpret_cast<float*>(ws + L.topk_w);
  prof_record(fwd, 0, stream);
  cudaError_t e = cudaSuccess;
  if (!routed && bn == 16 && T <= 16) {
    // decode: router and permutation in one CTA (its time is the "route" stage of the profile)
    e = launch_route_permute_small(routing_logits, routing_bias, T, routed_scaling_factor, E_local,
                                   local_expert_offset, bn, L, ws, stream);
    if (e != cudaSuccess) return from_cuda(e);
    prof_record(fwd, 1, stream);
  } else {
    if (!routed) {
      e = launch_route(routing_logits, routing_bias, T, routed_scaling_factor,
                       reinterpret_cast<int32_t*>(ws + L.topk_idx), reinterpret_cast<float*>(ws + L.topk_w),
                       reinterpret_cast<uint32_t*>(ws + L.status), stream);
      if (e != cudaSuccess) return from_cuda(e);
    }
    prof_record(fwd, 1, stream);
    e = launch_permute(topk_idx, topk_w, T, E_local, local_expert_offset, bn, sms, L, ws, stream);
    if (e != cudaSuccess) return from_cuda(e);
  }
  prof_record(fwd, 2, stream);
  if (bn == 16) {
    // decode: GEMM1, GEMM2 and the combine run as one kernel (its time is the
    // "gemm1" stage of the profile; "gemm2" and "combine" stay empty)
    e = launch_decode(&tm_w1, &tm_w2, reinterpret_cast<const uint8_t*>(hidden_states),
                      hidden_states_scale,
                      T, gemm1_weights_scale, gemm2_weights_scale, L, ws, out, f32_out, sms, sink, w1_packed,
                      stream);
    if (e != cudaSuccess) return from_cuda(e);
    prof_record(fwd, 3, stream);
    prof_record(fwd, 4, stream);
  } else {
    e = launch_gather_rows(reinterpret_cast<const uint8_t*>(hidden_states), hidden_states_scale, T, L, ws, stream);
    if (e != cudaSuccess) return from_cuda(e);
    e = launch_gemm1_rows(&tm_w1, &tm_aperm, &tm_ascale, gemm1_weights_scale, L, ws, sms, w1_packed, stream,
                          fp8_chain);
    if (e != cudaSuccess) return from_cuda(e);
    prof_record(fwd, 3, stream);
    if (fp8_chain)
      e = launch_gemm2_fp8_rows(&tm_w2b, &tm_inter8, &tm_iscale, gemm2_weights_scale, L, ws, sms, stream,
                                scattering ? scatter : nullptr);
    else
      e = launch_gemm2_rows(&tm_w2raw, &tm_inter, gemm2_weights_scale, L, ws, sms, stream,
                            scattering ? scatter : nullptr);
    if (e != cudaSuccess) return from_cuda(e);
    prof_record(fwd, 4, stream);
    // with the scatter, the owners' combine (moe_ep.cu) replaces the local reduce
    if (!scattering) e = launch_reduce(T, L, ws, out, f32_out, sink, stream);
  }
  prof_record(fwd, 5, stream);
  return from_cuda(e);
}

}  // namespace fbmoe

extern "C" {

int fbmoe_forward(const float* routing_logits, const void* routing_bias, const void* hidden_states,
                  const float* hidden_states_scale, const void* gemm1_weights, const float* gemm1_weights_scale,
                  const void* gemm2_weights, const float* gemm2_weights_scale, int T, int E_local,
                  int local_expert_offset, float routed_scaling_factor, void* out, void* workspace,
                  size_t workspace_bytes, void* stream) {
  return forward_core(routing_logits, routing_bias, hidden_states, hidden_states_scale, gemm1_weights,
                      gemm1_weights_scale, gemm2_weights, gemm2_weights_scale, T, E_local, local_expert_offset,
                      routed_scaling_factor, out, false, workspace, workspace_bytes, stream);
}

int fbmoe_forward_fp8_intermediate(const float* routing_logits, const void* routing_bias, const void* hidden_states,
                                   const float* hidden_states_scale, const void* gemm1_weights,
                                   const float* gemm1_weights_scale, const void* gemm2_weights,
                                   const float* gemm2_weights_scale, int T, int E_local, int local_expert_offset,
                                   float routed_scaling_factor, void* out, void* workspace, size_t workspace_bytes,
                                   void* stream) {
  return forward_core(routing_logits, routing_bias, hidden_states, hidden_states_scale, gemm1_weights,
                      gemm1_weights_scale, gemm2_weights, gemm2_weights_scale, T, E_local, local_expert_offset,
                      routed_scaling_factor, out, false, workspace, workspace_bytes, stream, true, nullptr, nullptr,
                      nullptr, false, true);
}

int fbmoe_forward_partial_f32(const float* routing_logits, const void* routing_bias, const void* hidden_states,
                              const float* hidden_states_scale, const void* gemm1_weights,
                              const float* gemm1_weights_scale, const void* gemm2_weights,
                              const float* gemm2_weights_scale, int T, int E_local, int local_expert_offset,
                              float routed_scaling_factor, float* out_f32, void* workspace, size_t workspace_bytes,
                              void* stream) {
  return forward_core(routing_logits, routing_bias, hidden_states, hidden_states_scale, gemm1_weights,
                      gemm1_weights_scale, gemm2_weights, gemm2_weights_scale, T, E_local, local_expert_offset,
                      routed_scaling_factor, out_f32, true, workspace, workspace_bytes, stream);
}

int fbmoe_profile_begin(int max_forwards) {
  if (max_forwards < 1) return FBMOE_ERR_INVALID_ARG;
  std::lock_guard<std::mutex> lk(g_prof.mu);
  if (g_prof.ev) {
    for (int i = 0; i < g_prof.cap * (kStages + 1); ++i) cudaEventDestroy(g_prof.ev[i]);
    delete[] g_prof.ev;
  }
  g_prof.ev = new cudaEvent_t[(size_t)max_forwards * (kStages + 1)];
  for (int i = 0; i < max_forwards * (kStages + 1); ++i) {
    cudaError_t e = cudaEventCreate(&g_prof.ev[i]);
    if (e != cudaSuccess) {
      for (int j = 0; j < i; ++j) cudaEventDestroy(g_prof.ev[j]);
      delete[] g_prof.ev;
      g_prof.ev = nullptr;
      g_prof.cap = 0;
      return from_cuda(e);
    }
  }
  g_prof.cap = max_forwards;
  g_prof.n = 0;
  g_prof.on = true;
  return FBMOE_OK;
}

int fbmoe_profile_end(float* stage_ms, int* n_forwards) {
  std::lock_guard<std::mutex> lk(g_prof.mu);
  g_prof.on = false;
  if (!g_prof.ev) return FBMOE_ERR_INVALID_ARG;
  int rc = FBMOE_OK;
  float sums[kStages] = {0, 0, 0, 0, 0};
  for (int f = 0; f < g_prof.n && rc == FBMOE_OK; ++f) {
    for (int s = 0; s < kStages; ++s) {
      cudaEvent_t a = g_prof.ev[f * (kStages + 1) + s], b = g_prof.ev[f * (kStages + 1) + s + 1];
      cudaError_t e = cudaEventSynchronize(b);
      float ms = 0.f;
      if (e == cudaSuccess) e = cudaEventElapsedTime(&ms, a, b);
      if (e != cudaSuccess) {
        rc = from_cuda(e);
        break;
      }
      sums[s] += ms;
    }
  }
  if (stage_ms) memcpy(stage_ms, sums, sizeof sums);
  if (n_forwards) *n_forwards = g_prof.n;
  for (int i = 0; i < g_prof.cap * (kStages + 1); ++i) cudaEventDestroy(g_prof.ev[i]);
  delete[] g_prof.ev;
  g_prof.ev = nullptr;
  g_prof.cap = 0;
  g_prof.n = 0;
  return rc;
}

int fbmoe_read_status(const void* workspace, uint32_t* status, void* stream_) {
  if (!workspace || !status) return FBMOE_ERR_NULL_POINTER;
  cudaStream_t stream = reinterpret_cast<cudaStream_t>(stream_);
  cudaError_t e = cudaMemcpyAsync(status, workspace, sizeof(uint32_t), cudaMemcpyDeviceToHost, stream);
  if (e == cudaSuccess) e = cudaStreamSynchronize(stream);
  if (e != cudaSuccess) return from_cuda(e);
  return *status ? FBMOE_ERR_DEVICE_STATUS : FBMOE_OK;
}

int fbmoe_set_status_sink(const void* workspace, uint32_t* sink) {
  if (!workspace) return FBMOE_ERR_NULL_POINTER;
  uint32_t* dev_sink = nullptr;
  if (sink) {
    cudaPointerAttributes attr;
    cudaError_t e = cudaPointerGetAttributes(&attr, sink);
    if (e != cudaSuccess) {
      (void)cudaGetLastError();
      return FBMOE_ERR_INVALID_ARG;
    }
    if (attr.type != cudaMemoryTypeHost || attr.devicePointer == nullptr) return FBMOE_ERR_INVALID_ARG;
    if (!aligned(sink, 4)) return FBMOE_ERR_MISALIGNED;
    dev_sink = static_cast<uint32_t*>(attr.devicePointer);
  }
  std::lock_guard<std::mutex> lk(g_sinks.mu);
  int n = g_sinks.n.load(std::memory_order_relaxed);
  int at = -1;
  for (int i = 0; i < n; ++i)
    if (g_sinks.ws[i] == workspace) at = i;
  if (!dev_sink) {  // unregister
    if (at >= 0) {
      g_sinks.ws[at] = g_sinks.ws[n - 1];
      g_sinks.sink[at] = g_sinks.sink[n - 1];
      g_sinks.n.store(n - 1, std::memory_order_release);
    }
    return FBMOE_OK;
  }
  if (at < 0) {
    if (n == kMaxSinks) return FBMOE_ERR_INVALID_ARG;
    at = n;
    g_sinks.ws[at] = workspace;
    g_sinks.sink[at] = dev_sink;
    g_sinks.n.store(n + 1, std::memory_order_release);
  } else {
    g_sinks.sink[at] = dev_sink;
  }
  return FBMOE_OK;
}

int fbmoe_test_expire_grid_wait(int enable) {
  g_test_expire.store(enable ? 1 : 0, std::memory_order_relaxed);
  return FBMOE_OK;
}

int fbmoe_decode_launch_mode(void) { return decode_launch_mode(); }

const char* fbmoe_error_string(int code) {
  switch (code) {
    case FBMOE_OK: return "ok";
    case FBMOE_ERR_INVALID_ARG: return "invalid argument (T < 0 or E_local outside 1..256)";
    case FBMOE_ERR_WORKSPACE_TOO_SMALL: return "workspace smaller than fbmoe_workspace_size(T, E_local)";
    case FBMOE_ERR_NULL_POINTER: return "null pointer argument";
    case FBMOE_ERR_MISALIGNED: return "misaligned pointer (tensors need 16-byte, workspace 256-byte alignment)";
    case FBMOE_ERR_DRIVER: return "cuTensorMapEncodeTiled unavailable or rejected a tensor map";
    case FBMOE_ERR_DEVICE_STATUS: return "a kernel reported a device-side error (bounded wait expired)";
    case FBMOE_ERR_NOALLOC_LIMIT: return "fbmoe_forward_noalloc supports T <= 16 and E_local <= 32 only";
    default: break;
  }
  if (code > 0) return cudaGetErrorString(static_cast<cudaError_t>(code));
  return "unknown fbmoe error";
}

int fbmoe_version(void) { return 100; }

}  // extern "C"
