// fbmoe_launch.h -- internal host-side launchers shared by the C-ABI (moe_capi.cu).
#pragma once

#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#include <atomic>

namespace fbmoe {

// Launch with programmatic stream serialization (see pdl_wait/pdl_trigger).
template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                              Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
}

// Cooperative launch (the whole grid is resident at once, or the launch fails),
// optionally also with programmatic stream serialization.
template <typename... KArgs, typename... Args>
inline cudaError_t launch_coop(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                               bool pdl, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 2 : 1;
  return cudaLaunchKernelEx(&cfg, kernel, static_cast<KArgs>(args)...);
}

// Raises a kernel's dynamic shared-memory limit on the current device once per
// device.  Safe from several host threads: the flags are atomic and the
// attribute call is idempotent, so two first calls may both make it.
constexpr int kMaxDevicesTracked = 64;
using DeviceFlags = std::atomic<bool>[kMaxDevicesTracked];
template <typename Kernel>
inline cudaError_t set_max_dynamic_smem(Kernel kernel, int bytes, DeviceFlags& done) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  const bool tracked = dev >= 0 && dev < kMaxDevicesTracked;
  if (tracked && done[dev].load(std::memory_order_acquire)) return cudaSuccess;
  e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e == cudaSuccess && tracked) done[dev].store(true, std::memory_order_release);
  return e;
}

// Offsets (bytes) of the sub-buffers inside the caller-provided workspace.
struct Layout {
  size_t status;       // uint32[4]  device status word(s)
  size_t topk_idx;     // int32[T*8] global expert ids, canonical order
  size_t topk_w;       // fp32[T*8]
  size_t token_rows;   // int32[T*8] permuted row of each (token, slot), -1 if not local
  size_t expert_cnt;   // int32[E_local]
  size_t expert_poff;  // int32[E_local+1] padded row offsets
  size_t n_blocks;     // int32[1]
  size_t blocks;       // int4[max_blocks] (expert, row0, nrows, 0)
  size_t row_token;    // int32[pcap]
  size_t row_weight;   // fp32[pcap]
  size_t inter;        // f16[pcap * 2048]   SwiGLU output, expert-contiguous rows
  size_t pair_out;     // f16[pcap * 7168]   weighted per-(token, expert) rows
  size_t chunk_cnt;    // int32[ceil(T/1024) * E_local] per-chunk expert counts (multi-CTA permute)
  size_t a_perm;       // e4m3[pcap * 7168]  token rows in permuted order (128-row blocks only)
  size_t splits;       // int32[2]: K splits of GEMM1 / GEMM2, chosen on the device per call
  size_t split_count;  // int32[max_blocks * 32]: arrivals per GEMM1 unit (stream-K fix-up)
  size_t split_part;   // fp32[kSplitItems][128][16]: GEMM1 partial sums, 2 slots per CTA
  size_t blk_ready;    // int32[max_blocks]: GEMM1 slices published per block (decode kernel)
  size_t grid_sync;    // int32[1]: CTAs of the decode kernel done with GEMM2 (zeroed by permute)
  size_t a_scale_perm;  // fp32[56 * pcap]    their 1x128 scales, [K-block][row] (128-row blocks only)
  size_t plane_scale;  // fp32[2][32][pcap]  scales of the decode kernel's fp8 intermediate planes (16-row blocks only)
  size_t total;        // bytes
  int tokens;          // T the layout was made for
  int pcap;            // row capacity (multiple of 128)
  int e_local;         // local experts the layout was made for
  int pair_planes;     // planes of pair_out (GEMM2 K splits write separate planes)
  int split_items;     // capacity of split_count / split_part (0: no split-K)
  int max_blocks;
};

// allow_split: reserve the split-K buffers used for 16-row (decode) blocks.
// force_rows: 128 selects the row-major (prefill) chain for every T.
Layout make_layout(int T, int E_local, bool allow_split = true, int force_rows = 0);

// Expert parallelism with the combine fused into GEMM2: pair row (token t, slot k)
// is stored straight into the receive buffer of the rank that owns token t
// (rows_per_rank consecutive tokens per rank), at pair[o][(t - o * rows_per_rank) * 8 + k].
// base[o] is rank o's pair region (a CUDA-IPC mapping for o != this rank).
constexpr int kMaxPeers = 8;
struct PeerScatter {
  __half* base[kMaxPeers];
  int rows_per_rank;
  int world;  // 0: no scatter, pair rows go to the local workspace
};

// Decode stream-K: capacity of fp32 partial slots (two per CTA of the decode kernel).
constexpr int kSplitItems = 1024;
constexpr int kMaxPairPlanes = 2;  // decode GEMM2 stream-K: at most 2 segments per unit
int choose_block_rows(int T, int E_local);

// Copies each routed token's row (and its 56 scales, [K-block][row]) to its
// permuted position, for the 128-row-block GEMM1 that loads A with plain TMA boxes.
cudaError_t launch_gather_rows(const uint8_t* hidden, const float* hidden_scale, int T, const Layout& L,
                               uint8_t* ws, cudaStream_t stream);

// Router: topk_idx/topk_w for T tokens; zeroes status[0].
cudaError_t launch_route(const float* logits, const void* bias_bf16, int T, float scale, int32_t* topk_idx,
                         float* topk_w, uint32_t* status, cudaStream_t stream);

// Histogram / padded offsets / deterministic permutation / GEMM block list.
// Also zeroes the decode kernel's arrival counters.
// Router + permutation in one CTA for 1 <= T <= 16 (the decode path): the same
// workspace outputs as launch_route followed by launch_permute.
cudaError_t launch_route_permute_small(const float* logits, const void* bias_bf16, int T, float scale, int E_local,
                                       int local_offset, int bn, const Layout& L, uint8_t* ws, cudaStream_t stream);

cudaError_t launch_permute(const int32_t* topk_idx, const float* topk_w, int T, int E_local, int local_offset,
                           int bn, int num_sms, const Layout& L, uint8_t* ws, cudaStream_t stream);

// Decode (16-row blocks): GEMM1 + SwiGLU, GEMM2 x routing weight and the
// per-token combine in one persistent kernel; writes out (bf16, or fp32 partial
// sums with f32_out).
// sink: host-visible status sink of the workspace (nullptr: none).
cudaError_t launch_decode(const CUtensorMap* tm_w1, const CUtensorMap* tm_w2,
                          const uint8_t* hidden, const float* hidden_scale, int T, const float* w1_scale,
                          const float* w2_scale, const Layout& L, uint8_t* ws, void* out, bool f32_out, int num_sms,
                          uint32_t* sink, bool w1_packed, cudaStream_t stream);
// 0: no decode launch yet; 1: cooperative with programmatic serialization;
// 2: cooperative; 3: plain programmatic launch sized by the occupancy query.
int decode_launch_mode();

// Status sink registered for a workspace (fbmoe_set_status_sink), or nullptr.
uint32_t* status_sink_for(const void* workspace);

// Test hook (fbmoe_test_expire_grid_wait): while set, the decode kernel's grid
// arrival waits for one arrival that never comes, with a budget of
// kTestGridWaitNs, so every CTA's bounded wait expires and reports
// kStatusTimeoutEpilogue without any fault.
bool test_expire_grid_wait();
constexpr uint64_t kTestGridWaitNs = 2000000ull;

// GEMM1 + SwiGLU for blocks of 128 rows with the tokens as the MMA M operand.
// w1_packed: tm_w1 maps the fbmoe_prepack_w1 layout with 256-row boxes (one box per
// operand tile) instead of the raw layout with 64-row boxes.
// fp8_inter: the SwiGLU output is re-quantised to e4m3 with 1x128 scales (the
// reference's numerics) into the intermediate region: e4m3 [pcap][2048] at
// L.inter, fp32 scales [16][pcap] at L.inter + fp8_inter_scale_offset(L).
cudaError_t launch_gemm1_rows(const CUtensorMap* tm_w1, const CUtensorMap* tm_aperm, const CUtensorMap* tm_ascale,
                              const float* w1_scale, const Layout& L, uint8_t* ws, int num_sms, bool w1_packed,
                              cudaStream_t stream, bool fp8_inter = false);

// Byte offset of the fp8 intermediate's scales inside the (f16-sized) intermediate region.
inline size_t fp8_inter_scale_offset(const Layout& L) { return (size_t)L.pcap * 2048; }  // pcap rows of 2048 e4m3

// GEMM2 of the fp8-intermediate mode: kind::f8f6f4 on the e4m3 intermediate
// (tm_inter8, 128 x 128-byte boxes), its scales (tm_iscale, [16][pcap]) and raw W2
// (tm_w2, 64-row x 128-byte boxes), promoted per 128-K block; f16 pair rows as
// launch_gemm2_rows writes them (or scattered to the token owners).
cudaError_t launch_gemm2_fp8_rows(const CUtensorMap* tm_w2, const CUtensorMap* tm_inter8,
                                  const CUtensorMap* tm_iscale, const float* w2_scale, const Layout& L, uint8_t* ws,
                                  int num_sms, cudaStream_t stream, const PeerScatter* scatter = nullptr);

// GEMM2 for blocks of 128 rows with the tokens as the MMA M operand; tm_w2raw
// maps W2 as unswizzled 64-byte x 256-row boxes.  Launches the pairs kernel and
// the one-block kernel; the device picks which of them does the work.
cudaError_t launch_gemm2_pairs(const CUtensorMap* tm_w2raw, const CUtensorMap* tm_inter, const float* w2_scale,
                               const Layout& L, uint8_t* ws, int num_sms, cudaStream_t stream,
                               const PeerScatter* scatter = nullptr);
cudaError_t launch_gemm2_rows(const CUtensorMap* tm_w2raw, const CUtensorMap* tm_inter, const float* w2_scale,
                              const Layout& L, uint8_t* ws, int num_sms, cudaStream_t stream,
                              const PeerScatter* scatter = nullptr);

// out[t, :] = sum of the token's pair rows, fp32 accumulation; bf16 result, or
// fp32 (f32_out) for partial sums that another stage combines across ranks.
cudaError_t launch_reduce(int T, const Layout& L, uint8_t* ws, void* out, bool f32_out, uint32_t* sink,
                          cudaStream_t stream);

// The whole forward on a caller-provided workspace (argument checks, TMA
// descriptors, the five launches); the public entry points wrap it.
int forward_core(const float* routing_logits, const void* routing_bias, const void* hidden_states,
                 const float* hidden_states_scale, const void* gemm1_weights, const float* gemm1_weights_scale,
                 const void* gemm2_weights, const float* gemm2_weights_scale, int T, int E_local,
                 int local_expert_offset, float routed_scaling_factor, void* out, bool f32_out, void* workspace,
                 size_t workspace_bytes, void* stream, bool allow_split = true,
                 const PeerScatter* scatter = nullptr, const int32_t* routed_idx = nullptr,
                 const float* routed_w = nullptr, bool w1_packed = false, bool fp8_inter = false);

}  // namespace fbmoe
