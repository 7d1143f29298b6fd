// moe_permute.cu -- per-expert histogram, padded prefix sum and deterministic
// token permutation into expert-contiguous rows, plus the GEMM block list.
//
// Counterpart of the reference's count / scan / permute kernels
// (solution/triton/main.py:1063-1238) with two differences:
//  * the order of rows inside an expert is token-ascending (deterministic; the
//    reference uses an atomic cursor, main.py:1150-1160);
//  * each expert's row segment starts at a multiple of 16 rows, so every GEMM
//    block of BN rows starts aligned, and the number of local experts is a
//    runtime value (32, 64, 128 or 256 for expert-parallel shards).
// The activations are not copied here (reference main.py:1241-1271): for small
// blocks GEMM1 gathers token rows itself; for 128-row blocks moe_gather.cu
// copies them.  Padding rows get row_token = -1.
//
// It also clears the arrival counters of the decode kernel (stream-K fix-up,
// per-block readiness, grid arrival).
//
// Tokens are processed in chunks of 1024, one CTA of 1024 threads per chunk.
// With one chunk (T <= 1024) a single CTA counts, scans and scatters.  With more,
// permute_count_kernel first writes each chunk's per-expert counts; then every
// scatter CTA derives the expert offsets (redundantly, from the small count
// matrix) and its own chunk's starting row inside each expert, so rows stay
// token-ascending across chunks.  CTA 0 alone writes the per-expert tables and
// the block list.  Within a chunk, a token's rank inside an expert is the number
// of set bits before it in that expert's 1024-bit membership mask, which is
// order-independent.
//
// Up to 16 tokens (route_permute_small_kernel): one CTA of 16 warps routes the
// tokens (a warp each, moe_route.cuh) and then permutes them, one launch instead
// of two; its top-8 goes to the workspace as the router kernel's does.
#include "fbmoe_common.cuh"
#include "fbmoe_launch.h"
#include "moe_route.cuh"

namespace fbmoe {
namespace {

constexpr int kThreads = 1024;
constexpr int kWordsPerChunk = kThreads / 32;
constexpr int kMaxLocal = 256;

struct PermuteSmem {
  int count[kMaxLocal];
  int poff[kMaxLocal + 1];
  int bstart[kMaxLocal + 1];
  int cursor[kMaxLocal];
  uint32_t bits[kMaxLocal][kWordsPerChunk];
  uint16_t wpre[kMaxLocal][kWordsPerChunk];
  int scan_tmp[2][kMaxLocal / 32];
  int n_blocks;
};

// Per-chunk expert counts: CTA c counts tokens [1024c, 1024c + 1024).
__global__ void __launch_bounds__(kThreads) permute_count_kernel(const int32_t* __restrict__ topk_idx, int T,
                                                                int E_local, int local_offset,
                                                                int32_t* __restrict__ chunk_cnt) {
  __shared__ int cnt[kMaxLocal];
  const int tid = threadIdx.x;
  pdl_wait();
  pdl_trigger();
  if (tid < kMaxLocal) cnt[tid] = 0;
  __syncthreads();
  const int t = blockIdx.x * kThreads + tid;
  if (t < T) {
#pragma unroll
    for (int k = 0; k < kTopK; ++k) {
      const int e = topk_idx[(size_t)t * kTopK + k] - local_offset;
      if ((unsigned)e < (unsigned)E_local) atomicAdd(&cnt[e], 1);
    }
  }
  __syncthreads();
  if (tid < E_local) chunk_cnt[(size_t)blockIdx.x * E_local + tid] = cnt[tid];
}

// Exclusive scan of one value per thread over threads 0..255 (8 warps).
__device__ __forceinline__ int block_excl_scan_256(int v, int* tmp, int* total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int x = v;
#pragma unroll
  for (int d = 1; d < 32; d <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, x, d);
    if (lane >= d) x += y;
  }
  if (lane == 31) tmp[warp] = x;
  named_barrier_sync(1, 256);
  int base = 0, all = 0;
#pragma unroll
  for (int w = 0; w < kMaxLocal / 32; ++w) {
    const int tw = tmp[w];
    base += (w < warp) ? tw : 0;
    all += tw;
  }
  *total = all;
  return base + x - v;
}

__global__ void __launch_bounds__(kThreads) permute_kernel(const int32_t* __restrict__ topk_idx,
                                                          const float* __restrict__ topk_w, int T, int E_local,
                                                          int local_offset, int bn, int32_t* __restrict__ expert_cnt,
                                                          int32_t* __restrict__ expert_poff,
                                                          int32_t* __restrict__ n_blocks, int4* __restrict__ blocks,
                                                          int max_blocks, int32_t* __restrict__ row_token,
                                                          float* __restrict__ row_weight,
                                                          int32_t* __restrict__ token_rows,
                                                          uint32_t* __restrict__ status, int num_sms,
                                                          int32_t* __restrict__ splits,
                                                          int32_t* __restrict__ split_count, int split_items,
                                                          int pair_planes, const int32_t* __restrict__ chunk_cnt,
                                                          int n_chunks, int32_t* __restrict__ blk_ready,
                                                          int32_t* __restrict__ grid_sync) {
  extern __shared__ __align__(16) uint8_t smem_raw[];
  PermuteSmem& S = *reinterpret_cast<PermuteSmem*>(smem_raw);
  const int tid = threadIdx.x;
  const int lane = tid & 31, warp = tid >> 5;

  pdl_wait();
  pdl_trigger();
  const int chunk = blockIdx.x;
  const bool lead = chunk == 0;  // writes the per-expert tables and the block list

  // Phase A: per-expert totals, and this chunk's starting rank inside each expert.
  if (n_chunks == 1) {
    for (int e = tid; e < kMaxLocal; e += kThreads) {
      S.count[e] = 0;
      S.cursor[e] = 0;
    }
    __syncthreads();
    for (int t = tid; t < T; t += kThreads) {
#pragma unroll
      for (int k = 0; k < kTopK; ++k) {
        const int e = topk_idx[(size_t)t * kTopK + k] - local_offset;
        if ((unsigned)e < (unsigned)E_local) atomicAdd(&S.count[e], 1);
      }
    }
  } else if (tid < kMaxLocal) {
    int tot = 0, pre = 0;
    if (tid < E_local) {
      for (int c = 0; c < n_chunks; ++c) {
        const int v = chunk_cnt[(size_t)c * E_local + tid];
        pre += c < chunk ? v : 0;
        tot += v;
      }
    }
    S.count[tid] = tot;
    S.cursor[tid] = pre;
  }
  __syncthreads();

  // Phase B: padded offsets and the GEMM block list (threads 0..255 = experts).
  if (tid < kMaxLocal) {
    const int e = tid;
    const int c = (e < E_local) ? S.count[e] : 0;
    const int padded = (c + kRowAlign - 1) / kRowAlign * kRowAlign;
    const int nb = (c + bn - 1) / bn;
    int tot_rows, tot_blocks;
    const int off = block_excl_scan_256(padded, S.scan_tmp[0], &tot_rows);
    const int boff = block_excl_scan_256(nb, S.scan_tmp[1], &tot_blocks);
    if (e < E_local) {
      S.poff[e] = off;
      S.cursor[e] += off;
      if (lead) {
        expert_cnt[e] = c;
        expert_poff[e] = off;
        for (int j = 0; j < nb; ++j) {
          const int b = boff + j;
          if (b < max_blocks) blocks[b] = make_int4(e, off + j * bn, min(bn, c - j * bn), 0);
        }
        for (int r = off + c; r < off + padded; ++r) row_token[r] = -1;  // padding rows
      }
    }
    if (e == 0 && lead) {
      expert_poff[E_local] = tot_rows;
      const int nb_all = min(tot_blocks, max_blocks);
      *n_blocks = nb_all;
      if (tot_blocks > max_blocks) atomicOr(status, kStatusBadTile);
      // planes of pair rows for the combine kernel (128-row path: always one)
      splits[0] = 1;
      splits[1] = 1;
      S.n_blocks = nb_all;
    }
  }
  __syncthreads();
  if (lead) {
    if (split_items > 0) {  // the decode kernel's stream-K arrival counters, one per GEMM1 unit
      const int units = S.n_blocks * (kInter / 64);
      for (int i = tid; i < units; i += kThreads) split_count[i] = 0;
    }
    // the decode kernel's per-block and grid arrival counters
    for (int i = tid; i < S.n_blocks; i += kThreads) blk_ready[i] = 0;
    if (tid == 0) grid_sync[0] = 0;
  }

  // Phase C: deterministic scatter of this chunk.
  {
    for (int i = tid; i < kMaxLocal * kWordsPerChunk; i += kThreads) (&S.bits[0][0])[i] = 0u;
    __syncthreads();
    const int t = chunk * kThreads + tid;
    int le[kTopK];
#pragma unroll
    for (int k = 0; k < kTopK; ++k) {
      le[k] = -1;
      if (t < T) {
        const int e = topk_idx[(size_t)t * kTopK + k] - local_offset;
        if ((unsigned)e < (unsigned)E_local) {
          le[k] = e;
          atomicOr(&S.bits[e][warp], 1u << lane);
        }
      }
    }
    __syncthreads();
    if (tid < E_local) {
      int run = 0;
      for (int w = 0; w < kWordsPerChunk; ++w) {
        S.wpre[tid][w] = (uint16_t)run;
        run += __popc(S.bits[tid][w]);
      }
    }
    __syncthreads();
    if (t < T) {
      const uint32_t below = (1u << lane) - 1u;
#pragma unroll
      for (int k = 0; k < kTopK; ++k) {
        const int e = le[k];
        int row = -1;
        if (e >= 0) {
          row = S.cursor[e] + S.wpre[e][warp] + __popc(S.bits[e][warp] & below);
          row_token[row] = t;
          row_weight[row] = topk_w[(size_t)t * kTopK + k];
        }
        token_rows[(size_t)t * kTopK + k] = row;
      }
    }
  }
}

// Decode-sized calls (T <= 64): the same outputs with 3 CTA barriers instead
// of ~10.  Thread p handles (token p / 8, slot p % 8); a token's rank inside an
// expert is the number of set bits below it in the expert's 64-bit token mask
// (token-ascending, order-independent); threads 0..255 also own one expert each
// for the padded offsets and the block list.
constexpr int kSmallT = 64;
constexpr int kSmallThreads = kSmallT * kTopK;  // 512

// The small permutation, run by all 512 threads of the calling CTA.  topk_idx /
// topk_w: global arrays written by an earlier kernel (read through L2), or, with
// kLocalTopk, this CTA's shared-memory copy.
template <bool kLocalTopk>
__device__ __forceinline__ void permute_small_body(
    const int32_t* __restrict__ topk_idx, const float* __restrict__ topk_w, int T, int E_local, int local_offset,
    int bn, int32_t* __restrict__ expert_cnt, int32_t* __restrict__ expert_poff, int32_t* __restrict__ n_blocks,
    int4* __restrict__ blocks, int max_blocks, int32_t* __restrict__ row_token, float* __restrict__ row_weight,
    int32_t* __restrict__ token_rows, uint32_t* __restrict__ status, int32_t* __restrict__ splits,
    int32_t* __restrict__ split_count, int split_items, int32_t* __restrict__ blk_ready,
    int32_t* __restrict__ grid_sync) {
  __shared__ int cnt[kMaxLocal];
  __shared__ unsigned long long mask[kMaxLocal];
  __shared__ int poff[kMaxLocal];
  __shared__ int wsum[2][kMaxLocal / 32];
  __shared__ int nblk;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  if (tid < kMaxLocal) {
    cnt[tid] = 0;
    mask[tid] = 0ull;
  }
  __syncthreads();
  const int t = tid / kTopK;
  int e = -1;
  if (t < T) {
    e = (kLocalTopk ? topk_idx[tid] : __ldcg(topk_idx + tid)) - local_offset;
    if ((unsigned)e < (unsigned)E_local) {
      atomicAdd(&cnt[e], 1);
      atomicOr(&mask[e], 1ull << t);
    } else {
      e = -1;
    }
  }
  __syncthreads();
  // padded offsets and block counts: warp-inclusive scans, then the earlier warps' totals
  int c = 0, padded = 0, nb = 0, xo = 0, xb = 0;
  if (tid < kMaxLocal) {
    c = tid < E_local ? cnt[tid] : 0;
    padded = (c + kRowAlign - 1) / kRowAlign * kRowAlign;
    nb = (c + bn - 1) / bn;
    xo = padded;
    xb = nb;
#pragma unroll
    for (int d = 1; d < 32; d <<= 1) {
      const int yo = __shfl_up_sync(0xffffffffu, xo, d), yb = __shfl_up_sync(0xffffffffu, xb, d);
      if (lane >= d) {
        xo += yo;
        xb += yb;
      }
    }
    if (lane == 31) {
      wsum[0][warp] = xo;
      wsum[1][warp] = xb;
    }
  }
  __syncthreads();
  if (tid < kMaxLocal) {
    int base_o = 0, base_b = 0, tot_o = 0, tot_b = 0;
#pragma unroll
    for (int w = 0; w < kMaxLocal / 32; ++w) {
      base_o += w < warp ? wsum[0][w] : 0;
      base_b += w < warp ? wsum[1][w] : 0;
      tot_o += wsum[0][w];
      tot_b += wsum[1][w];
    }
    const int off = base_o + xo - padded, boff = base_b + xb - nb;
    poff[tid] = off;
    if (tid < E_local) {
      expert_cnt[tid] = c;
      expert_poff[tid] = off;
      for (int j = 0; j < nb; ++j)
        if (boff + j < max_blocks) blocks[boff + j] = make_int4(tid, off + j * bn, min(bn, c - j * bn), 0);
      for (int r = off + c; r < off + padded; ++r) row_token[r] = -1;  // padding rows
    }
    if (tid == 0) {
      expert_poff[E_local] = tot_o;
      const int nb_all = min(tot_b, max_blocks);
      *n_blocks = nb_all;
      nblk = nb_all;
      if (tot_b > max_blocks) atomicOr(status, kStatusBadTile);
      splits[0] = 1;  // planes of pair rows for the 128-row combine kernel
      splits[1] = 1;
      *grid_sync = 0;
    }
  }
  __syncthreads();
  // the decode kernel's arrival counters (stream-K fix-up, per-block readiness)
  if (split_items > 0)
    for (int i = tid; i < nblk * (kInter / 64); i += kSmallThreads) split_count[i] = 0;
  for (int i = tid; i < nblk; i += kSmallThreads) blk_ready[i] = 0;
  if (t < T) {
    int row = -1;
    if (e >= 0) {
      row = poff[e] + __popcll(mask[e] & ((1ull << t) - 1ull));
      row_token[row] = t;
      row_weight[row] = kLocalTopk ? topk_w[tid] : __ldcg(topk_w + tid);
    }
    token_rows[tid] = row;
  }
}

__global__ void __launch_bounds__(kSmallThreads) permute_small_kernel(
    const int32_t* __restrict__ topk_idx, const float* __restrict__ topk_w, int T, int E_local, int local_offset,
    int bn, int32_t* __restrict__ expert_cnt, int32_t* __restrict__ expert_poff, int32_t* __restrict__ n_blocks,
    int4* __restrict__ blocks, int max_blocks, int32_t* __restrict__ row_token, float* __restrict__ row_weight,
    int32_t* __restrict__ token_rows, uint32_t* __restrict__ status, int32_t* __restrict__ splits,
    int32_t* __restrict__ split_count, int split_items, int32_t* __restrict__ blk_ready,
    int32_t* __restrict__ grid_sync) {
  pdl_wait();
  pdl_trigger();
  permute_small_body<false>(topk_idx, topk_w, T, E_local, local_offset, bn, expert_cnt, expert_poff, n_blocks, blocks,
                     max_blocks, row_token, row_weight, token_rows, status, splits, split_count, split_items,
                     blk_ready, grid_sync);
}

constexpr int kFusedT = kSmallThreads / 32;  // 16 tokens, a warp each

// Router + small permutation for T <= 16 in one CTA; the routing result stays in
// shared memory between the two (no round trip through L2).  Dynamic shared memory:
// the router's per-warp scratch (256 values, 256 ids, 256 scores, 8 picks).
__global__ void __launch_bounds__(kSmallThreads) route_permute_small_kernel(
    const float* __restrict__ logits, const __nv_bfloat16* __restrict__ bias, float scale,
    int32_t* __restrict__ topk_idx, float* __restrict__ topk_w, int T, int E_local, int local_offset,
    int bn, int32_t* __restrict__ expert_cnt, int32_t* __restrict__ expert_poff, int32_t* __restrict__ n_blocks,
    int4* __restrict__ blocks, int max_blocks, int32_t* __restrict__ row_token, float* __restrict__ row_weight,
    int32_t* __restrict__ token_rows, uint32_t* __restrict__ status, int32_t* __restrict__ splits,
    int32_t* __restrict__ split_count, int split_items, int32_t* __restrict__ blk_ready,
    int32_t* __restrict__ grid_sync) {
  extern __shared__ float route_scratch[];
  __shared__ int s_idx[kFusedT * kTopK];
  __shared__ float s_w[kFusedT * kTopK];
  const int warp = threadIdx.x >> 5;
  float* wv = route_scratch + (size_t)warp * (3 * kExperts + kTopK);
  int* wi = reinterpret_cast<int*>(wv + kExperts);
  float* wsc = wv + 2 * kExperts;
  int* wsel = reinterpret_cast<int*>(wv + 3 * kExperts);
  pdl_wait();
  pdl_trigger();
  if (threadIdx.x == 0) status[0] = 0u;
  const int t = warp;
  float x[8];
  if (t < T) route_dev::load_logits8(logits, t, x);
  float bs[8];
  route_dev::load_bias8(bias, bs);
  // the top-8 stays in shared memory for the permutation; the workspace gets a copy
  if (t < T) route_dev::route_token(x, t, bs, scale, s_idx, s_w, wv, wi, wsc, wsel);
  __syncthreads();
  if ((int)threadIdx.x < T * kTopK) {
    topk_idx[threadIdx.x] = s_idx[threadIdx.x];
    topk_w[threadIdx.x] = s_w[threadIdx.x];
  }
  permute_small_body<true>(s_idx, s_w, T, E_local, local_offset, bn, expert_cnt, expert_poff, n_blocks, blocks,
                     max_blocks, row_token, row_weight, token_rows, status, splits, split_count, split_items,
                     blk_ready, grid_sync);
}
constexpr int kFusedSmem = kFusedT * (3 * kExperts + kTopK) * 4;

}  // namespace

cudaError_t launch_route_permute_small(const float* logits, const void* bias_bf16, int T, float scale, int E_local,
                                       int local_offset, int bn, const Layout& L, uint8_t* ws, cudaStream_t stream) {
  if (T < 1 || T > kFusedT) return cudaErrorInvalidValue;
  static DeviceFlags attr_set;
  if (cudaError_t err = set_max_dynamic_smem(route_permute_small_kernel, kFusedSmem, attr_set); err != cudaSuccess) return err;
  return launch_pdl(route_permute_small_kernel, dim3(1), dim3(kSmallThreads), kFusedSmem, stream, logits,
      reinterpret_cast<const __nv_bfloat16*>(bias_bf16), scale, reinterpret_cast<int32_t*>(ws + L.topk_idx),
      reinterpret_cast<float*>(ws + L.topk_w), T, E_local, local_offset, bn,
      reinterpret_cast<int32_t*>(ws + L.expert_cnt), reinterpret_cast<int32_t*>(ws + L.expert_poff),
      reinterpret_cast<int32_t*>(ws + L.n_blocks), reinterpret_cast<int4*>(ws + L.blocks), L.max_blocks,
      reinterpret_cast<int32_t*>(ws + L.row_token), reinterpret_cast<float*>(ws + L.row_weight),
      reinterpret_cast<int32_t*>(ws + L.token_rows), reinterpret_cast<uint32_t*>(ws + L.status),
      reinterpret_cast<int32_t*>(ws + L.splits), reinterpret_cast<int32_t*>(ws + L.split_count), L.split_items,
      reinterpret_cast<int32_t*>(ws + L.blk_ready), reinterpret_cast<int32_t*>(ws + L.grid_sync));
}

cudaError_t launch_permute(const int32_t* topk_idx, const float* topk_w, int T, int E_local, int local_offset,
                           int bn, int num_sms, const Layout& L, uint8_t* ws, cudaStream_t stream) {
  const int smem = (int)sizeof(PermuteSmem);
  static DeviceFlags attr_set;
  if (cudaError_t err = set_max_dynamic_smem(permute_kernel, smem, attr_set); err != cudaSuccess) return err;
  if (T > 0 && T <= kSmallT)
    return launch_pdl(permute_small_kernel, dim3(1), dim3(kSmallThreads), 0, stream, topk_idx, topk_w, T, E_local,
        local_offset, bn, reinterpret_cast<int32_t*>(ws + L.expert_cnt), reinterpret_cast<int32_t*>(ws + L.expert_poff),
        reinterpret_cast<int32_t*>(ws + L.n_blocks), reinterpret_cast<int4*>(ws + L.blocks), L.max_blocks,
        reinterpret_cast<int32_t*>(ws + L.row_token), reinterpret_cast<float*>(ws + L.row_weight),
        reinterpret_cast<int32_t*>(ws + L.token_rows), reinterpret_cast<uint32_t*>(ws + L.status),
        reinterpret_cast<int32_t*>(ws + L.splits), reinterpret_cast<int32_t*>(ws + L.split_count), L.split_items,
        reinterpret_cast<int32_t*>(ws + L.blk_ready), reinterpret_cast<int32_t*>(ws + L.grid_sync));
  const int n_chunks = (T + kThreads - 1) / kThreads;
  int32_t* chunk_cnt = reinterpret_cast<int32_t*>(ws + L.chunk_cnt);
  if (n_chunks > 1) {
    cudaError_t err = launch_pdl(permute_count_kernel, dim3(n_chunks), dim3(kThreads), 0, stream, topk_idx, T,
                                 E_local, local_offset, chunk_cnt);
    if (err != cudaSuccess) return err;
  }
  return launch_pdl(permute_kernel, dim3(n_chunks > 0 ? n_chunks : 1), dim3(kThreads), smem, stream,
      topk_idx, topk_w, T, E_local, local_offset, bn, reinterpret_cast<int32_t*>(ws + L.expert_cnt),
      reinterpret_cast<int32_t*>(ws + L.expert_poff), reinterpret_cast<int32_t*>(ws + L.n_blocks),
      reinterpret_cast<int4*>(ws + L.blocks), L.max_blocks, reinterpret_cast<int32_t*>(ws + L.row_token),
      reinterpret_cast<float*>(ws + L.row_weight), reinterpret_cast<int32_t*>(ws + L.token_rows),
      reinterpret_cast<uint32_t*>(ws + L.status), num_sms, reinterpret_cast<int32_t*>(ws + L.splits),
      reinterpret_cast<int32_t*>(ws + L.split_count), L.split_items, L.pair_planes,
      static_cast<const int32_t*>(chunk_cnt), n_chunks, reinterpret_cast<int32_t*>(ws + L.blk_ready),
      reinterpret_cast<int32_t*>(ws + L.grid_sync));
}

}  // namespace fbmoe
