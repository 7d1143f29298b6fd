// moe_gemm2_pairs.cu -- GEMM2 x routing weight for large token blocks (prefill),
// tokens as the MMA's M operand (tcgen05 kind::f16, TMEM, TMA), sm_100a.
//
// Runs the calls whose experts have several 128-row blocks (at least 2 per active
// expert, gemm2_pairs_mode); other calls run moe_gemm2_rows.cu, which is launched
// right after this kernel.
//
// Counterpart of the reference's gemm2_kernel (solution/triton/main.py:433-600),
// and the same arithmetic as the GEMM2 phase of moe_decode.cu:
//     pair_out[r, h] = w[r] * sum_j inter[r, j] * W2[e, h, j] * s2[e, h/128, j/128].
//
// Work unit = a PAIR of row blocks of one expert (two consecutive 128-row blocks;
// an expert with an odd block count ends with a single block) x one tile of 256
// W2 rows (two 128-row scale blocks of the hidden dimension).  Per 64-K step the
// W2 tile is loaded and converted once and feeds two MMAs, one per row block:
// A = 128 intermediate rows (f16, TMA, 128-byte swizzle), B = the converted W2
// tile, D = 128 x 256 fp32 in TMEM per block (columns 0-255 and 256-511: all of
// TMEM, so the epilogue of a unit and the MMAs of the next do not overlap; the
// producers and converters keep running ahead).  Sharing the converted tile cuts
// the bytes loaded per FLOP from 32 KB to 24 KB per 128x256x64 MMA and halves
// the conversion work.  Each epilogue thread owns one token row of each block and
// writes 256 contiguous f16 outputs (512 bytes) per block.
//
// W2 dequantisation.  Per 128-row block hb the tile picks a power of two 2^k
// so that max_k s2 * 2^k lies in (32, 64]; each element becomes
// f16(fp8) * f16(s2 * 2^k) in one HMUL2 (the fp8 value is exact in f16, the
// product stays below 448 * 64), and the epilogue multiplies by 2^-k exactly.
// Two f16 roundings per weight; measured on the CPU emulation this keeps the
// worst element at 0.35x the output tolerance, the same as one fp32 rounding.
//
// Warp roles (512 threads): w0 W2 producer (TMA, raw FP8, 16 KB per step),
// w1 MMA issuer + TMEM owner, w2 intermediate producer (TMA, both blocks' rows
// of a step into one slot of its own ring), w3 idle, w4-w11 converters (256
// threads, 4 x 16-byte chunks each per step), w12-w15 epilogue (TMEM lane
// quarter = warp % 4).
//
// Epilogue stores: each warp converts 64 columns of its 32 rows at a time, stages
// them in shared memory and writes them with 8 lanes per row, so every store
// instruction covers four whole 128-byte lines (remote rows cross NVLink in full
// lines, not in 16-byte pieces).
//
// Expert parallelism (PeerScatter): the epilogue writes pair row (token t, slot k)
// into the receive buffer of the rank that owns token t, over NVLink for other
// ranks, instead of the local pair rows; the transfer overlaps the GEMM.  k is
// the slot whose token_rows entry names this row.  Each epilogue thread ends
// with a system-scope fence, so a later flag release covers its stores.
#include <math.h>

#include "fbmoe_common.cuh"
#include "fbmoe_launch.h"

namespace fbmoe {
namespace {

constexpr int kThreads = 512;
constexpr int kRows = 128;
constexpr int kN = 256;
constexpr int kNTiles = kHidden / kN;         // 28
constexpr int kKSteps = kInter / 64;          // 32 steps of 64
constexpr int kRawStages = 3;
constexpr int kConvStages = 2;
constexpr int kAStages = 2;                   // intermediate tiles in flight (their TMA latency is exposed otherwise)
constexpr int kRawBytes = kN * 64;            // 16 KB fp8
constexpr int kWBytes = kN * 128;             // 32 KB f16 W2 operand
constexpr int kABlockBytes = kRows * 128;     // 16 KB f16 intermediate operand of one row block
constexpr int kABytes = 2 * kABlockBytes;     // both blocks of a pair
constexpr uint64_t kWaitBudgetNs = 4000000000ull;
constexpr int kMaxLocal = 256;
constexpr int kOffRaw = 0;
constexpr int kOffW = kOffRaw + kRawStages * kRawBytes;
constexpr int kOffA = kOffW + kConvStages * kWBytes;
constexpr int kOffBar = kOffA + kAStages * kABytes;
constexpr int kNumBars = 2 * kRawStages + 2 * kConvStages + 2 * kAStages + 2 + 1;
constexpr int kOffMisc = kOffBar + kNumBars * 8;
// Per-expert pair tables: first block index, block count, first pair index (+ the total).
constexpr int kOffTab = (kOffMisc + 16 + 15) / 16 * 16;
constexpr int kTabBytes = (3 * kMaxLocal + 1) * 4;
// Epilogue staging: each epilogue warp's 32 rows x 64 columns (f16), rows padded
// to 144 bytes so that both the row-per-lane writes and the 8-lanes-per-row reads
// are free of bank conflicts.
constexpr int kStageStride = 144;
constexpr int kOffStage = (kOffTab + kTabBytes + 127) / 128 * 128;
constexpr int kSmemBytes = kOffStage + 4 * 32 * kStageStride + 1024;
static_assert(kSmemBytes <= 227 * 1024, "shared memory over the per-CTA limit");

struct Ring {
  int slot = 0;
  uint32_t phase = 0;
  int n;
  __device__ explicit Ring(int n_) : n(n_) {}
  __device__ void next() {
    if (++slot == n) {
      slot = 0;
      phase ^= 1u;
    }
  }
};

// Pair tables in shared memory: blocks are laid out expert by expert, nb_e =
// ceil(rows_e / 128) of them (the permutation's block list); expert e's pairs
// are its blocks (2j, 2j + 1), the last one single when nb_e is odd.
struct PairTab {
  const int* boff;   // [E] first block of expert e
  const int* nblk;   // [E] blocks of expert e
  const int* poff;   // [E + 1] first pair of expert e; poff[E] = pairs in total
  int E;
  int nb;            // blocks in the list (the permutation caps it at max_blocks)
  // pair p -> (first block, second block or -1)
  __device__ int2 at(int p) const {
    int lo = 0, hi = E - 1;  // the last expert e with poff[e] <= p
    while (lo < hi) {
      const int mid = (lo + hi + 1) >> 1;
      if (poff[mid] <= p) lo = mid;
      else hi = mid - 1;
    }
    const int b0 = boff[lo] + 2 * (p - poff[lo]);
    const int b1 = (b0 + 1 < boff[lo] + nblk[lo] && b0 + 1 < nb) ? b0 + 1 : -1;
    return make_int2(b0, b1);
  }
};

__global__ void __launch_bounds__(kThreads, 1)
    gemm2_pairs_kernel(const __grid_constant__ CUtensorMap tm_w2raw, const __grid_constant__ CUtensorMap tm_inter,
                      const float* __restrict__ w2_scale, const int32_t* __restrict__ n_blocks_ptr,
                      const int4* __restrict__ blocks, const int32_t* __restrict__ expert_cnt,
                      const float* __restrict__ row_weight, __half* __restrict__ pair_out,
                      uint32_t* __restrict__ status, const int32_t* __restrict__ row_token,
                      const int32_t* __restrict__ token_rows, const PeerScatter ps, int T, int e_local, int pcap) {
  // Calls with few blocks per expert run the one-block kernel launched after this one.
  {
    __shared__ int red[16];
    __shared__ int s_pairs;
    if (threadIdx.x < 256) {
      const bool pm = gemm2_pairs_mode(expert_cnt, e_local, *n_blocks_ptr, red);
      if (threadIdx.x == 0) s_pairs = pm ? 1 : 0;
    }
    __syncthreads();
    if (!s_pairs) {
      pdl_trigger();
      pdl_wait();  // complete only after the grids before it (the next kernel relies on it)
      return;
    }
  }
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sRaw = sm + kOffRaw;
  uint8_t* sW = sm + kOffW;
  uint8_t* sA = sm + kOffA;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + kOffBar);
  uint64_t* raw_full = bars;
  uint64_t* raw_empty = bars + kRawStages;
  uint64_t* w_full = bars + 2 * kRawStages;                    // converters wrote the f16 W2 slot
  uint64_t* c_empty = bars + 2 * kRawStages + kConvStages;     // MMA done with the f16 W2 slot
  uint64_t* a_full = bars + 2 * kRawStages + 2 * kConvStages;  // intermediate rows landed
  uint64_t* a_empty = a_full + kAStages;                       // MMA done with the intermediate slot
  uint64_t* tfull = a_empty + kAStages;                        // a unit's accumulators are complete
  uint64_t* tempty = tfull + 1;                                // the epilogue has read them
  uint64_t* drain = tfull + 2;
  uint32_t* sTmem = reinterpret_cast<uint32_t*>(sm + kOffMisc);
  volatile int* sAbort = reinterpret_cast<volatile int*>(sm + kOffMisc + 4);
  int* sBoff = reinterpret_cast<int*>(sm + kOffTab);
  int* sNblk = sBoff + kMaxLocal;
  int* sPoff = sNblk + kMaxLocal;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kRawStages; ++s) {
      mbar_init(&raw_full[s], 1);
      mbar_init(&raw_empty[s], 8);
    }
    for (int s = 0; s < kConvStages; ++s) {
      mbar_init(&w_full[s], 8);
      mbar_init(&c_empty[s], 1);
    }
    for (int s = 0; s < kAStages; ++s) {
      mbar_init(&a_full[s], 1);
      mbar_init(&a_empty[s], 1);
    }
    mbar_init(tfull, 1);
    mbar_init(tempty, 4);
    mbar_init(drain, 1);
    *sAbort = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tm_w2raw);
    tma_prefetch_desc(&tm_inter);
  }
  if (warp == 1) {
    tmem_alloc(sTmem, 512);
    tmem_relinquish();
  }
  // The pair tables from the per-expert row counts (threads 0..255, one expert
  // each; blocks and counts come from the permute kernel, which finished before
  // GEMM1 let this grid launch).
  const int nb_all = *n_blocks_ptr;
  if (threadIdx.x < kMaxLocal) {
    const int e = threadIdx.x;
    const int c = e < e_local ? expert_cnt[e] : 0;
    const int nbk = (c + kRows - 1) / kRows;
    const int np = (nbk + 1) / 2;
    // two inclusive warp scans, then the 8 warps' totals
    int xb = nbk, xp = np;
#pragma unroll
    for (int d = 1; d < 32; d <<= 1) {
      const int yb = __shfl_up_sync(0xffffffffu, xb, d), yp = __shfl_up_sync(0xffffffffu, xp, d);
      if (lane >= d) {
        xb += yb;
        xp += yp;
      }
    }
    sNblk[e] = nbk;
    // each warp's totals, then every thread adds the totals of the warps before its own
    const int tb = __shfl_sync(0xffffffffu, xb, 31), tp = __shfl_sync(0xffffffffu, xp, 31);
    __shared__ int wtot[2][kMaxLocal / 32];
    if (lane == 0) {
      wtot[0][warp] = tb;
      wtot[1][warp] = tp;
    }
    named_barrier_sync(1, kMaxLocal);
    int base_b = 0, base_p = 0, all_p = 0;
#pragma unroll
    for (int w = 0; w < kMaxLocal / 32; ++w) {
      base_b += w < warp ? wtot[0][w] : 0;
      base_p += w < warp ? wtot[1][w] : 0;
      all_p += wtot[1][w];
    }
    sBoff[e] = xb - nbk + base_b;
    sPoff[e] = xp - np + base_p;
    if (e == 0) sPoff[kMaxLocal] = all_p;
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  // The block list and row weights come from the permute kernel, which finished
  // before GEMM1 let this grid launch; only the intermediate rows (GEMM1's output)
  // need the wait, done by the thread that loads them.
  pdl_trigger();
  const uint32_t tmem_base = *sTmem;
  const int E = e_local < kMaxLocal ? e_local : kMaxLocal;
  const PairTab tab{sBoff, sNblk, sPoff, E, nb_all};
  // a block list the permutation had to cut short (status already flagged) runs no unit
  const bool whole = E > 0 && sBoff[E - 1] + sNblk[E - 1] == nb_all;
  const int n_units = whole ? sPoff[kMaxLocal] * kNTiles : 0;

  auto fail = [&](uint32_t bit) {
    *sAbort = 1;
    atomicOr(status, bit);
  };

  if (warp == 0 || warp == 2) {
    // ------------------------------------------------------------ producers
    if (lane == 0) {
      const bool w2_side = (warp == 0);
      if (!w2_side) {
        pdl_wait();
        fence_proxy_async_global();
      }
      const int n = w2_side ? kRawStages : kAStages;
      uint64_t* fullb = w2_side ? raw_full : a_full;
      uint64_t* emptyb = w2_side ? raw_empty : a_empty;
      Ring ring(n);
      bool ok = true;
      uint32_t issued_mask = 0, parity_mask = 0;
      for (int u = blockIdx.x; u < n_units && ok; u += gridDim.x) {
        const int2 pr = tab.at(u / kNTiles);
        const int4 blk0 = dbg_block(blocks[pr.x], kRows, e_local, pcap, status);
        const int r1 = pr.y >= 0 ? dbg_block(blocks[pr.y], kRows, e_local, pcap, status).y : -1;
        const int nt = u % kNTiles;
        for (int ks = 0; ks < kKSteps; ++ks) {
          if (!mbar_wait(&emptyb[ring.slot], ring.phase ^ 1u, sAbort, kWaitBudgetNs)) {
            ok = false;
            fail(kStatusTimeoutProducer);
            break;
          }
          if (w2_side) {
            mbar_arrive_expect_tx(&fullb[ring.slot], kRawBytes);
            tma_load_2d_nohint(sRaw + ring.slot * kRawBytes, &tm_w2raw, &fullb[ring.slot], ks * 64,
                               blk0.x * kHidden + nt * kN);
          } else {
            uint8_t* dst = sA + ring.slot * kABytes;
            mbar_arrive_expect_tx(&fullb[ring.slot], r1 >= 0 ? kABytes : kABlockBytes);
            tma_load_2d_nohint(dst, &tm_inter, &fullb[ring.slot], ks * 64, blk0.y);
            if (r1 >= 0) tma_load_2d_nohint(dst + kABlockBytes, &tm_inter, &fullb[ring.slot], ks * 64, r1);
          }
          issued_mask |= 1u << ring.slot;
          parity_mask = (parity_mask & ~(1u << ring.slot)) | (ring.phase << ring.slot);
          ring.next();
        }
      }
      for (int s = 0; s < n; ++s)
        if ((issued_mask >> s) & 1u)
          if (!mbar_wait_drain(&fullb[s], (parity_mask >> s) & 1u, kWaitBudgetNs))
            fail(kStatusTimeoutDrain);
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = umma_idesc(0u, kRows, kN);  // f16 x f16 -> fp32
      Ring ring(kConvStages), ar(kAStages);
      uint32_t ug = 0;
      bool ok = true, any = false;
      for (int u = blockIdx.x; u < n_units && ok; u += gridDim.x, ++ug) {
        const bool two = tab.at(u / kNTiles).y >= 0;
        // the epilogue has read the previous unit's accumulators
        if (!mbar_wait(tempty, (ug & 1u) ^ 1u, sAbort, kWaitBudgetNs)) {
          ok = false;
          fail(kStatusTimeoutMma);
          break;
        }
        tc_fence_after();
        for (int ks = 0; ks < kKSteps; ++ks) {
          if (!mbar_wait(&w_full[ring.slot], ring.phase, sAbort, kWaitBudgetNs) ||
              !mbar_wait(&a_full[ar.slot], ar.phase, sAbort, kWaitBudgetNs)) {
            ok = false;
            fail(kStatusTimeoutMma);
            break;
          }
          tc_fence_after();
          const uint64_t bdesc = umma_desc_sw128(smem_u32(sW + ring.slot * kWBytes));
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            if (h == 1 && !two) break;
            const uint64_t adesc = umma_desc_sw128(smem_u32(sA + ar.slot * kABytes + h * kABlockBytes));
#pragma unroll
            for (int k = 0; k < 4; ++k)
              mma_f16(tmem_base + h * kN, adesc + 2 * k, bdesc + 2 * k, idesc, (ks | k) ? 1u : 0u);
          }
          tc_commit(&c_empty[ring.slot]);
          tc_commit(&a_empty[ar.slot]);
          any = true;
          ring.next();
          ar.next();
        }
        if (!ok) break;
        tc_commit(tfull);
      }
      if (any) {
        tc_commit(drain);
        mbar_wait_drain(drain, 0, kWaitBudgetNs);
      }
    }
    __syncwarp();
  } else if (warp >= 4 && warp < 12) {
    // ------------------------------------------------------------ converters
    const int tid = threadIdx.x - 128;  // 0..255
    Ring rr(kRawStages), cr(kConvStages);
    bool ok = true;
    for (int u = blockIdx.x; u < n_units && ok; u += gridDim.x) {
      const int4 blk = dbg_block(blocks[tab.at(u / kNTiles).x], kRows, e_local, pcap, status);
      const int nt = u % kNTiles;
      const float* s_lo = w2_scale + ((size_t)blk.x * kHBlocks + 2 * nt) * kIBlocks;  // rows 0..127
      const float* s_hi = s_lo + kIBlocks;                                           // rows 128..255
      const int k_lo = w2_block_exponent(s_lo), k_hi = w2_block_exponent(s_hi);
      // lanes 0-15 hold the first block's 16 scales, lanes 16-31 the second's
      const float lane_scale = __ldg((lane < 16 ? s_lo : s_hi) + (lane & 15));
      for (int ks = 0; ks < kKSteps; ++ks) {
        if (!mbar_wait(&raw_full[rr.slot], rr.phase, sAbort, kWaitBudgetNs) ||
            !mbar_wait(&c_empty[cr.slot], cr.phase ^ 1u, sAbort, kWaitBudgetNs)) {
          ok = false;
          if (lane == 0) fail(kStatusTimeoutConvert);
          break;
        }
        const __half h_lo = __float2half_rn(ldexpf(__shfl_sync(0xffffffffu, lane_scale, ks / 2), k_lo));
        const __half h_hi = __float2half_rn(ldexpf(__shfl_sync(0xffffffffu, lane_scale, 16 + ks / 2), k_hi));
        const uint8_t* raw = sRaw + rr.slot * kRawBytes;
        uint8_t* wt = sW + cr.slot * kWBytes;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int c = tid + 256 * i;  // 16-byte chunk of the raw tile
          const int r = c >> 2, part = c & 3;
          const __half2 sc2 = __half2half2(r < 128 ? h_lo : h_hi);
          const uint4 q = *reinterpret_cast<const uint4*>(raw + c * 16);
          const uint32_t w[4] = {q.x, q.y, q.z, q.w};
          uint32_t o[8];
#pragma unroll
          for (int h = 0; h < 4; ++h) {
            const __half2_raw a = __nv_cvt_fp8x2_to_halfraw2((__nv_fp8x2_storage_t)(w[h] & 0xFFFFu), __NV_E4M3);
            const __half2_raw b = __nv_cvt_fp8x2_to_halfraw2((__nv_fp8x2_storage_t)(w[h] >> 16), __NV_E4M3);
            const __half2 pa = __hmul2(*reinterpret_cast<const __half2*>(&a), sc2);
            const __half2 pb = __hmul2(*reinterpret_cast<const __half2*>(&b), sc2);
            o[2 * h] = *reinterpret_cast<const uint32_t*>(&pa);
            o[2 * h + 1] = *reinterpret_cast<const uint32_t*>(&pb);
          }
          *reinterpret_cast<uint4*>(wt + sw128_offset(r, 2 * part)) = make_uint4(o[0], o[1], o[2], o[3]);
          *reinterpret_cast<uint4*>(wt + sw128_offset(r, 2 * part + 1)) = make_uint4(o[4], o[5], o[6], o[7]);
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          mbar_arrive(&raw_empty[rr.slot]);
          mbar_arrive(&w_full[cr.slot]);
        }
        rr.next();
        cr.next();
      }
    }
  } else if (warp >= 12) {
    // ------------------------------------------------------------ epilogue
    const int q = warp & 3;
    const int row = q * 32 + lane;
    const uint32_t lane_base = (uint32_t)(q * 32) << 16;
    uint8_t* stage = sm + kOffStage + q * 32 * kStageStride;
    uint32_t ug = 0;
    bool ok = true;
    for (int u = blockIdx.x; u < n_units && ok; u += gridDim.x, ++ug) {
      const int2 pr = tab.at(u / kNTiles);
      const int nt = u % kNTiles;
      if (!mbar_wait(tfull, ug & 1u, sAbort, kWaitBudgetNs)) {
        ok = false;
        if (lane == 0) fail(kStatusTimeoutEpilogue);
        break;
      }
      tc_fence_after();
      bool sat = false;
      for (int h = 0; h < 2; ++h) {
        const int b = h == 0 ? pr.x : pr.y;
        if (b < 0) break;
        const int4 blk = dbg_block(blocks[b], kRows, e_local, pcap, status);
        const int r0 = blk.y, nrows = blk.z;
        const float* s_lo = w2_scale + ((size_t)blk.x * kHBlocks + 2 * nt) * kIBlocks;
        const float wr = row < nrows ? __ldg(row_weight + r0 + row) : 0.0f;
        const float f_lo = ldexpf(wr, -w2_block_exponent(s_lo));
        const float f_hi = ldexpf(wr, -w2_block_exponent(s_lo + kIBlocks));
        __half* drow = pair_out + (size_t)(r0 + row) * kHidden;
        bool has_dst = row < nrows;
        if (ps.world > 0 && has_dst) {
          const int r = r0 + row;
          const int t = dbg_token(__ldg(row_token + r), T, status);
          const int4* tr4 = reinterpret_cast<const int4*>(token_rows + (size_t)t * kTopK);
          const int4 ra = __ldg(tr4), rb = __ldg(tr4 + 1);
          const int k = ra.x == r ? 0 : ra.y == r ? 1 : ra.z == r ? 2 : ra.w == r ? 3
                      : rb.x == r ? 4 : rb.y == r ? 5 : rb.z == r ? 6 : rb.w == r ? 7 : -1;
          const int o = t / ps.rows_per_rank;
          if (k < 0 || o >= ps.world) {
            atomicOr(status, kStatusBadSlot);
            has_dst = false;
          } else {
            drow = ps.base[o] + ((size_t)(t - o * ps.rows_per_rank) * kTopK + k) * kHidden;
          }
        }
        drow += nt * kN;
#pragma unroll 1
        for (int g = 0; g < kN / 64; ++g) {
#pragma unroll
          for (int cc = 0; cc < 4; ++cc) {
            const int c = 4 * g + cc;
            float p[16];
            tmem_ld16(tmem_base + lane_base + h * kN + 16 * c, p);
            tmem_wait_ld();
            const float f = c < 8 ? f_lo : f_hi;
            uint32_t w[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) {
              const __half a = to_half_sat(p[2 * i] * f, sat), bb = to_half_sat(p[2 * i + 1] * f, sat);
              w[i] = (uint32_t)__half_as_ushort(a) | ((uint32_t)__half_as_ushort(bb) << 16);
            }
            uint4* st = reinterpret_cast<uint4*>(stage + lane * kStageStride + cc * 32);
            st[0] = make_uint4(w[0], w[1], w[2], w[3]);
            st[1] = make_uint4(w[4], w[5], w[6], w[7]);
          }
          __syncwarp();
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            const int rr = 4 * j + (lane >> 3), ch = lane & 7;
            __half* rp = reinterpret_cast<__half*>(__shfl_sync(0xffffffffu, reinterpret_cast<unsigned long long>(drow), rr));
            const int rd = __shfl_sync(0xffffffffu, has_dst ? 1 : 0, rr);
            const uint4 v = *reinterpret_cast<const uint4*>(stage + rr * kStageStride + ch * 16);
            if (rd) *reinterpret_cast<uint4*>(rp + g * 64 + ch * 8) = v;
          }
          __syncwarp();
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(tempty);
      if (sat) atomicOr(status, kStatusSaturated);
    }
    if (ps.world > 0) __threadfence_system();  // peer stores ordered before the signal that follows
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, 512);
  }
}

}  // namespace

cudaError_t launch_gemm2_pairs(const CUtensorMap* tm_w2raw, const CUtensorMap* tm_inter, const float* w2_scale,
                              const Layout& L, uint8_t* ws, int num_sms, cudaStream_t stream,
                              const PeerScatter* scatter) {
  static DeviceFlags attr_set;
  if (cudaError_t err = set_max_dynamic_smem(gemm2_pairs_kernel, kSmemBytes, attr_set); err != cudaSuccess) return err;
  PeerScatter ps{};
  if (scatter != nullptr) ps = *scatter;
  const long max_units = (long)(L.max_blocks + 1) / 2 * kNTiles + (long)L.e_local * kNTiles;
  int grid = (int)(max_units < num_sms ? max_units : num_sms);
  if (grid < 1) grid = 1;
  return launch_pdl(gemm2_pairs_kernel, dim3(grid), dim3(kThreads), kSmemBytes, stream, *tm_w2raw, *tm_inter, w2_scale,
                    reinterpret_cast<const int32_t*>(ws + L.n_blocks), reinterpret_cast<const int4*>(ws + L.blocks),
                    reinterpret_cast<const int32_t*>(ws + L.expert_cnt),
                    reinterpret_cast<const float*>(ws + L.row_weight), reinterpret_cast<__half*>(ws + L.pair_out),
                    reinterpret_cast<uint32_t*>(ws + L.status), reinterpret_cast<const int32_t*>(ws + L.row_token),
                    reinterpret_cast<const int32_t*>(ws + L.token_rows), ps, L.tokens, L.e_local, L.pcap);
}

}  // namespace fbmoe
