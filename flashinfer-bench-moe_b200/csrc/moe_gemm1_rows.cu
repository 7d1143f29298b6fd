// moe_gemm1_rows.cu -- GEMM1 + SwiGLU for large token blocks (prefill), with
// the tokens as the MMA's M operand (tcgen05 kind::f8f6f4, TMEM, TMA), sm_100a;
// and, in the fp8-intermediate mode, GEMM2 on fp8 operands through the same
// pipeline.
//
// Counterpart of the reference's gemm1_kernel + act_quant_kernel (solution/
// triton/main.py:41-223, 1426-1602), and the same arithmetic as the GEMM1 phase
// of moe_decode.cu: per permuted row r (token t) of expert e,
//     G1[r, n] = sum_k A[t, k] * a_scale[k/128, t] * W1[e, n, k] * s1[e, n/128, k/128]
//     inter[r, j] = silu(G1[r, 2048 + j]) * G1[r, j]      (f16, clamped to +-65504)
//
// Orientation.  A = 128 token rows (one block of the permuted list), read by TMA
// as one 128 x 128-byte box from the permuted copy of the activations (see
// moe_gather.cu for why the rows are copied first); B = 256 W1 rows: the 128 rows of one scale
// block of the first half stacked on the matching 128 rows of the second half
// (TMA).  D = 128 x 256 fp32 in TMEM.  Each thread of the epilogue owns one token
// row, so the per-128-K promotion is ONE multiply-add per element with a
// per-thread factor (a_scale[row] * s1[block]) instead of a per-column factor,
// and SwiGLU pairs columns c and 128 + c inside a thread.
//
// One work unit = (block of <=128 rows) x (tile j of 128 intermediate columns),
// 56 K-blocks.  Each K-block is MMA'd into one of two 256-column TMEM buffers
// (all 512 columns) while the epilogue promotes the other.
//
// Warp roles (576 threads): w0 producer (TMA for the activation and W1 tiles),
// w1 MMA issuer + TMEM owner, w2-w17 epilogue: 16 warps, four per SM
// sub-partition so that their TMEM-load latencies overlap; warp w reads TMEM
// lanes 32*(w%4)..+31 and owns 32 of the 128 output columns of the tile
// (64 fp32 accumulators per thread, 96 registers per thread).
//
// FP8-intermediate mode (the reference's numerics, selected per call):
// * GEMM1 (kOutFp8): the SwiGLU output is re-quantised per row and 128-column
//   block, scale = amax / 448 (1 for an all-zero block), q = e4m3(y / scale) --
//   the reference's act_quant rule (main.py:1476-1488) -- into an fp8
//   intermediate [pcap][2048] plus scales [16][pcap].  The four warps that own a
//   block's 128 columns of a row exchange their partial amax through shared memory.
// * GEMM2 (kPairOut): A = 128 rows of that fp8 intermediate, B = 256 W2 rows (two
//   128-row scale blocks), 16 K-blocks, promoted with a_scale[row] * s2[block];
//   the epilogue multiplies by the routing weight and stores f16 pair rows (to
//   the token owner's buffer when scattering), as gemm2_rows_kernel does.
#include "fbmoe_common.cuh"
#include "fbmoe_launch.h"

namespace fbmoe {
namespace {

enum RowsMode : int { kOutF16 = 0, kOutFp8 = 1, kPairOut = 2 };

template <int M>
struct RowsCfg {
  static constexpr int kKBlocks = M == kPairOut ? kIBlocks : kHBlocks;  // 16 or 56 K-blocks of 128
  static constexpr int kTiles = M == kPairOut ? kHidden / 256 : kInter / 128;  // 28 or 16 tiles per row block
};

constexpr int kThreads = 576;
constexpr int kEpiWarps = 16;
constexpr int kRows = 128;                       // token rows per block (== block_rows 128)
constexpr int kStages = 4;
constexpr int kABytes = kRows * 128;             // 16 KB of gathered token rows
constexpr int kBBytes = 256 * 128;               // 32 KB of W1 rows
constexpr uint64_t kWaitBudgetNs = 4000000000ull;
constexpr int kOffA = 0;
constexpr int kOffB = kOffA + kStages * kABytes;
constexpr int kScaleSlots = 8;                   // ring of per-K-block row-scale vectors
constexpr int kOffAS = kOffB + kStages * kBBytes;            // fp32 [8][128] row scales
constexpr int kOffWS = kOffAS + kScaleSlots * kRows * 4;    // fp32 [2][2][56] weight scales of a unit
constexpr int kOffAmax = kOffWS + 2 * 2 * kHBlocks * 4;     // fp32 [2][4][128] partial amax (kOutFp8)
constexpr int kOffBar = kOffAmax + 2 * 4 * kRows * 4;
constexpr int kNumBars = 2 * kStages + 4 + 1 + kScaleSlots + 2 + 2;
constexpr int kOffMisc = kOffBar + kNumBars * 8;
constexpr int kSmemBytes = kOffMisc + 16 + 1024;
static_assert(kSmemBytes <= 227 * 1024, "shared memory over the per-CTA limit");

// Outputs of the three modes (unused fields are null).
struct RowsOut {
  __half* inter;                 // kOutF16: f16 intermediate [pcap][2048]
  uint8_t* inter8;               // kOutFp8: e4m3 intermediate [pcap][2048]
  float* iscale;                 // kOutFp8: its scales [16][pcap]
  const float* row_weight;       // kPairOut: routing weight per permuted row
  __half* pair_out;              // kPairOut: pair rows [pcap][7168] (no scatter)
  const int32_t* row_token;      // kPairOut with scatter: token of each row
  const int32_t* token_rows;     // kPairOut with scatter: the token's 8 slot rows
  PeerScatter ps;
  int T;
};

template <int M>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_rows_fp8_kernel(const __grid_constant__ CUtensorMap tm_w, const __grid_constant__ CUtensorMap tm_a,
                         const __grid_constant__ CUtensorMap tm_ascale, const float* __restrict__ w_scale,
                         const int32_t* __restrict__ n_blocks_ptr, const int4* __restrict__ blocks,
                         const RowsOut out, uint32_t* __restrict__ status, int e_local, int pcap, int w1_packed) {
  using Cfg = RowsCfg<M>;
  constexpr int kKB = Cfg::kKBlocks;
  constexpr int kTiles = Cfg::kTiles;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = sm + kOffA;
  uint8_t* sB = sm + kOffB;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + kOffBar);
  uint64_t* full = bars;
  uint64_t* empty = bars + kStages;
  uint64_t* tfull = bars + 2 * kStages;
  uint64_t* tempty = tfull + 2;
  uint64_t* drain = tfull + 4;
  uint64_t* sfull = drain + 1;               // row scales of K-block x landed in slot x % 8
  uint64_t* wfull = sfull + kScaleSlots;     // weight scales of a unit landed in slot (unit % 2)
  float* sAS = reinterpret_cast<float*>(sm + kOffAS);
  float* sWS = reinterpret_cast<float*>(sm + kOffWS);
  float* sAmax = reinterpret_cast<float*>(sm + kOffAmax);
  uint32_t* sTmem = reinterpret_cast<uint32_t*>(sm + kOffMisc);
  volatile int* sAbort = reinterpret_cast<volatile int*>(sm + kOffMisc + 4);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);   // producer's expect_tx arrive (weight tiles + row tiles)
      mbar_init(&empty[s], 1);  // tcgen05.commit
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], kEpiWarps);  // one arrive per epilogue warp
    }
    mbar_init(drain, 1);
    for (int s = 0; s < kScaleSlots; ++s) mbar_init(&sfull[s], 1);
    mbar_init(&wfull[0], 1);
    mbar_init(&wfull[1], 1);
    mbar_init(&wfull[2], kEpiWarps);  // amax_ready of the kOutFp8 epilogue, by unit parity
    mbar_init(&wfull[3], kEpiWarps);
    *sAbort = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tm_w);
    tma_prefetch_desc(&tm_a);
    tma_prefetch_desc(&tm_ascale);
  }
  if (warp == 1) {
    tmem_alloc(sTmem, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  pdl_wait();
  pdl_trigger();
  fence_proxy_async_global();
  const uint32_t tmem_base = *sTmem;
  const int n_units = (*n_blocks_ptr) * kTiles;

  auto fail = [&](uint32_t bit) {
    *sAbort = 1;
    atomicOr(status, bit);
  };

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    // Operand tiles into stage x % 4, the K-block's 128 row scales into slot
    // x % 8 and, at a unit's first K-block, its weight scales into slot unit % 2.
    // Slot reuse is safe without extra barriers: loads for K-block x start only
    // after MMA x - 4 completed, which needed the epilogue done with x - 6 (two
    // TMEM buffers); slot x % 8 last held x - 8, and unit slots are kKB >= 16
    // K-blocks apart.
    int stage = 0;
    uint32_t phase = 0;
    bool ok = true;
    uint32_t issued_mask = 0, parity_mask = 0;  // per stage: ever issued / parity of the last issue
    int x = 0, ui = 0;
    for (int u = blockIdx.x; u < n_units && ok; u += gridDim.x, ++ui) {
      const int4 blk = dbg_block(blocks[u / kTiles], kRows, e_local, pcap, status);
      const int j = u % kTiles;
      const int e = blk.x, r0 = blk.y;
      // B rows of the tile: GEMM1 raw W1 = rows 128j.. of both halves; GEMM2 = 256 consecutive W2 rows
      const int wrow = M == kPairOut ? e * kHidden + 256 * j : e * kGemm1N + 128 * j;
      for (int kb = 0; kb < kKB; ++kb, ++x) {
        if (!mbar_wait(&empty[stage], phase ^ 1u, sAbort, kWaitBudgetNs)) {
          ok = false;
          if (lane == 0) fail(kStatusTimeoutProducer);
          break;
        }
        if (lane == 0) {
          if (kb == 0) {
            uint64_t* wb = &wfull[ui & 1];
            float* wdst = sWS + (ui & 1) * 2 * kHBlocks;
            // the unit's two 128-row weight scale blocks, kKB scales each
            const float* w0 = M == kPairOut ? w_scale + ((size_t)e * kHBlocks + 2 * j) * kIBlocks
                                            : w_scale + ((size_t)e * (kGemm1N / kBlk) + j) * kHBlocks;
            const float* w1 = M == kPairOut ? w0 + kIBlocks
                                            : w_scale + ((size_t)e * (kGemm1N / kBlk) + kIBlocks + j) * kHBlocks;
            mbar_arrive_expect_tx(wb, 2 * kKB * 4);
            bulk_load_1d(wdst, w0, kKB * 4, wb);
            bulk_load_1d(wdst + kHBlocks, w1, kKB * 4, wb);
          }
          uint64_t* sb = &sfull[x & (kScaleSlots - 1)];
          mbar_arrive_expect_tx(sb, kRows * 4);
          tma_load_2d_nohint(sAS + (x & (kScaleSlots - 1)) * kRows, &tm_ascale, sb, r0, kb);
          mbar_arrive_expect_tx(&full[stage], kABytes + kBBytes);
          tma_load_2d_nohint(sA + stage * kABytes, &tm_a, &full[stage], kb * kBlk, r0);
          uint8_t* b = sB + stage * kBBytes;
          if (M != kPairOut && w1_packed) {
            // packed rows [256j, 256j + 256): X1 2j, X2 2j, X1 2j+1, X2 2j+1 (64 rows each), one box
            tma_load_2d_nohint(b, &tm_w, &full[stage], kb * kBlk, e * kGemm1N + 256 * j);
          } else if (M == kPairOut) {
            tma_load_2d_nohint(b, &tm_w, &full[stage], kb * kBlk, wrow);
            tma_load_2d_nohint(b + 64 * 128, &tm_w, &full[stage], kb * kBlk, wrow + 64);
            tma_load_2d_nohint(b + 128 * 128, &tm_w, &full[stage], kb * kBlk, wrow + 128);
            tma_load_2d_nohint(b + 192 * 128, &tm_w, &full[stage], kb * kBlk, wrow + 192);
          } else {
            tma_load_2d_nohint(b, &tm_w, &full[stage], kb * kBlk, wrow);
            tma_load_2d_nohint(b + 64 * 128, &tm_w, &full[stage], kb * kBlk, wrow + 64);
            tma_load_2d_nohint(b + 128 * 128, &tm_w, &full[stage], kb * kBlk, wrow + kInter);
            tma_load_2d_nohint(b + 192 * 128, &tm_w, &full[stage], kb * kBlk, wrow + kInter + 64);
          }
        }
        issued_mask |= 1u << stage;
        parity_mask = (parity_mask & ~(1u << stage)) | (phase << stage);
        if (++stage == kStages) {
          stage = 0;
          phase ^= 1u;
        }
      }
    }
    __syncwarp();
    if (lane == 0) {
      // every issued load lands before the CTA exits
      for (int s = 0; s < kStages; ++s)
        if ((issued_mask >> s) & 1u)
          if (!mbar_wait_drain(&full[s], (parity_mask >> s) & 1u, kWaitBudgetNs))
            fail(kStatusTimeoutDrain);
      for (int k = 1; k <= kScaleSlots && k <= x; ++k) {
        const int y = x - k;  // the last K-blocks issued, one per slot
        if (!mbar_wait_drain(&sfull[y & (kScaleSlots - 1)], (uint32_t)(y >> 3) & 1u, kWaitBudgetNs))
          fail(kStatusTimeoutDrain);
      }
      for (int k = 1; k <= 2 && k <= ui; ++k) {
        const int v = ui - k;
        if (!mbar_wait_drain(&wfull[v & 1], (uint32_t)(v >> 1) & 1u, kWaitBudgetNs))
          fail(kStatusTimeoutDrain);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = umma_idesc(0u, 128, 256);
      int stage = 0;
      uint32_t phase = 0;
      uint32_t kbg = 0;
      bool ok = true;
      bool any = false;
      for (int u = blockIdx.x; u < n_units && ok; u += gridDim.x) {
        for (int kb = 0; kb < kKB; ++kb) {
          const uint32_t buf = kbg & 1u;
          if (!mbar_wait(&tempty[buf], ((kbg >> 1) & 1u) ^ 1u, sAbort, kWaitBudgetNs) ||
              !mbar_wait(&full[stage], phase, sAbort, kWaitBudgetNs)) {
            ok = false;
            fail(kStatusTimeoutMma);
            break;
          }
          tc_fence_after();
          const uint64_t adesc = umma_desc_sw128(smem_u32(sA + stage * kABytes));
          const uint64_t bdesc = umma_desc_sw128(smem_u32(sB + stage * kBBytes));
          const uint32_t d = tmem_base + buf * 256;
#pragma unroll
          for (int k = 0; k < 4; ++k) mma_f8f6f4(d, adesc + 2 * k, bdesc + 2 * k, idesc, k > 0 ? 1u : 0u);
          tc_commit(&empty[stage]);
          tc_commit(&tfull[buf]);
          any = true;
          ++kbg;
          if (++stage == kStages) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      if (any) {
        tc_commit(drain);
        mbar_wait_drain(drain, 0, kWaitBudgetNs);
      }
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------ epilogue
    const int q = warp & 3;            // TMEM lane quarter
    const int g = (warp - 2) >> 2;     // output columns [32g, 32g+32) of each 128-column half of the tile
    const int row = q * 32 + lane;     // token row in the block == TMEM lane
    const uint32_t lane_base = (uint32_t)(q * 32) << 16;
    // TMEM columns of this warp's 32 first-half and 32 second-half columns: raw layout
    // 0-127 | 128-255; packed W1 layout in 64-column runs X1 | X2 | X1 | X2
    const bool packed = M != kPairOut && w1_packed;
    const uint32_t x1_col = packed ? (uint32_t)((g >> 1) * 128 + (g & 1) * 32) : (uint32_t)(32 * g);
    const uint32_t x2_col = packed ? x1_col + 64u : (uint32_t)(128 + 32 * g);
    uint64_t* amax_ready = wfull + 2;  // kOutFp8: the 16 warps' partial amax of a unit are in shared memory
    uint32_t kbg = 0;
    bool ok = true;
    int ui = 0;
    for (int u = blockIdx.x; u < n_units && ok; u += gridDim.x, ++ui) {
      const int4 blk = dbg_block(blocks[u / kTiles], kRows, e_local, pcap, status);
      const int j = u % kTiles;
      const int r0 = blk.y, nrows = blk.z;
      // this unit's weight scales: [0, kKB) first 128-row block, [56, 56 + kKB) second
      if (!mbar_wait(&wfull[ui & 1], (uint32_t)(ui >> 1) & 1u, sAbort, kWaitBudgetNs)) {
        if (lane == 0) fail(kStatusTimeoutEpilogue);
        break;
      }
      const float* wsu = sWS + (ui & 1) * 2 * kHBlocks;
      // packed accumulators: acc[k] = columns (2k, 2k+1) of this warp's 32 first-half
      // columns (k < 16) or second-half columns (k >= 16)
      uint64_t acc[32];
#pragma unroll
      for (int i = 0; i < 32; ++i) acc[i] = 0ull;
      for (int kb = 0; kb < kKB; ++kb) {
        const uint32_t slot = kbg & (kScaleSlots - 1);
        if (!mbar_wait(&sfull[slot], (kbg >> 3) & 1u, sAbort, kWaitBudgetNs)) {
          ok = false;
          if (lane == 0) fail(kStatusTimeoutEpilogue);
          break;
        }
        // rows past the block's end use whatever scale the box held (zero-filled
        // past the buffer); their results are never stored
        const float a_s = sAS[slot * kRows + row];
        const float w_1 = wsu[kb], w_2 = wsu[kHBlocks + kb];
        const uint32_t buf = kbg & 1u;
        if (!mbar_wait(&tfull[buf], (kbg >> 1) & 1u, sAbort, kWaitBudgetNs)) {
          ok = false;
          if (lane == 0) fail(kStatusTimeoutEpilogue);
          break;
        }
        tc_fence_after();
        const uint32_t t0 = tmem_base + lane_base + buf * 256;
        const uint64_t f1 = f32x2_pack(a_s * w_1, a_s * w_1), f2 = f32x2_pack(a_s * w_2, a_s * w_2);
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          // chunks 0-1: first-half columns (f1); 2-3: second half (f2)
          uint64_t p[8];
          tmem_ld16_pairs(t0 + (c < 2 ? x1_col + 16 * c : x2_col + 16 * (c - 2)), p);
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 8; ++i) f32x2_fma(acc[8 * c + i], p[i], c < 2 ? f1 : f2);
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&tempty[buf]);
        ++kbg;
      }
      if (!ok) break;
      if constexpr (M == kOutF16) {
        if (row < nrows) {
          bool sat = false;
          uint4* dst = reinterpret_cast<uint4*>(out.inter + (size_t)(r0 + row) * kInter + 128 * j + 32 * g);
#pragma unroll
          for (int v = 0; v < 4; ++v) {
            uint32_t w[4];
#pragma unroll
            for (int h = 0; h < 4; ++h) {
              const int k = 4 * v + h;  // columns 2k, 2k+1
              float x1a, x1b, x2a, x2b;
              f32x2_unpack(acc[k], x1a, x1b);
              f32x2_unpack(acc[16 + k], x2a, x2b);
              const float ya = x2a / (1.0f + expf(-x2a)) * x1a;
              const float yb = x2b / (1.0f + expf(-x2b)) * x1b;
              const __half ha = to_half_sat(ya, sat), hb = to_half_sat(yb, sat);
              w[h] = (uint32_t)__half_as_ushort(ha) | ((uint32_t)__half_as_ushort(hb) << 16);
            }
            dst[v] = make_uint4(w[0], w[1], w[2], w[3]);
          }
          if (sat) atomicOr(status, kStatusSaturated);
        }
      } else if constexpr (M == kOutFp8) {
        float y[32];
        float m = 0.0f;
#pragma unroll
        for (int k = 0; k < 16; ++k) {
          float x1a, x1b, x2a, x2b;
          f32x2_unpack(acc[k], x1a, x1b);
          f32x2_unpack(acc[16 + k], x2a, x2b);
          y[2 * k] = x2a / (1.0f + expf(-x2a)) * x1a;
          y[2 * k + 1] = x2b / (1.0f + expf(-x2b)) * x1b;
          m = fmaxf(m, fmaxf(fabsf(y[2 * k]), fabsf(y[2 * k + 1])));
        }
        // block amax over the four warps that own the row's 128 columns
        float* am = sAmax + (ui & 1) * 4 * kRows;
        am[g * kRows + row] = m;
        __syncwarp();
        if (lane == 0) mbar_arrive(&amax_ready[ui & 1]);
        if (!mbar_wait(&amax_ready[ui & 1], (uint32_t)(ui >> 1) & 1u, sAbort, kWaitBudgetNs)) {
          if (lane == 0) fail(kStatusTimeoutEpilogue);
          break;
        }
        const float bm = fmaxf(fmaxf(am[row], am[kRows + row]), fmaxf(am[2 * kRows + row], am[3 * kRows + row]));
        if (row < nrows) {
          const E4m3Scale qs = e4m3_block_scale(bm);
          const float s = qs.s;
          uint32_t w[8];
#pragma unroll
          for (int i = 0; i < 8; ++i)
            w[i] = e4m3x2_quotient(y[4 * i], y[4 * i + 1], qs) | (e4m3x2_quotient(y[4 * i + 2], y[4 * i + 3], qs) << 16);
          uint4* dst = reinterpret_cast<uint4*>(out.inter8 + (size_t)(r0 + row) * kInter + 128 * j + 32 * g);
          dst[0] = make_uint4(w[0], w[1], w[2], w[3]);
          dst[1] = make_uint4(w[4], w[5], w[6], w[7]);
          if (g == 0) out.iscale[(size_t)j * pcap + r0 + row] = s;
          if (!(m <= 3.0e38f)) atomicOr(status, kStatusSaturated);  // non-finite SwiGLU output
        }
      } else {
        // kPairOut: routing weight, f16 pair row (this rank's buffer or the token owner's)
        const float wr = row < nrows ? __ldg(out.row_weight + r0 + row) : 0.0f;
        __half* drow = out.pair_out + (size_t)(r0 + row) * kHidden;
        bool has_dst = row < nrows;
        if (out.ps.world > 0 && has_dst) {
          const int r = r0 + row;
          const int t = dbg_token(__ldg(out.row_token + r), out.T, status);
          const int4* tr4 = reinterpret_cast<const int4*>(out.token_rows + (size_t)t * kTopK);
          const int4 ra = __ldg(tr4), rb = __ldg(tr4 + 1);
          const int k = ra.x == r ? 0 : ra.y == r ? 1 : ra.z == r ? 2 : ra.w == r ? 3
                      : rb.x == r ? 4 : rb.y == r ? 5 : rb.z == r ? 6 : rb.w == r ? 7 : -1;
          const int o = t / out.ps.rows_per_rank;
          if (k < 0 || o >= out.ps.world) {
            atomicOr(status, kStatusBadSlot);
            has_dst = false;
          } else {
            drow = out.ps.base[o] + ((size_t)(t - o * out.ps.rows_per_rank) * kTopK + k) * kHidden;
          }
        }
        if (has_dst) {
          bool sat = false;
          drow += 256 * j;
#pragma unroll
          for (int half = 0; half < 2; ++half) {
            uint4* dst = reinterpret_cast<uint4*>(drow + 128 * half + 32 * g);
#pragma unroll
            for (int v = 0; v < 4; ++v) {
              uint32_t w[4];
#pragma unroll
              for (int h = 0; h < 4; ++h) {
                float a, b;
                f32x2_unpack(acc[16 * half + 4 * v + h], a, b);
                const __half ha = to_half_sat(a * wr, sat), hb = to_half_sat(b * wr, sat);
                w[h] = (uint32_t)__half_as_ushort(ha) | ((uint32_t)__half_as_ushort(hb) << 16);
              }
              dst[v] = make_uint4(w[0], w[1], w[2], w[3]);
            }
          }
          if (sat) atomicOr(status, kStatusSaturated);
        }
      }
    }
    if (M == kPairOut && out.ps.world > 0) __threadfence_system();  // peer stores before the signal that follows
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, 512);
  }
}

template <int M>
cudaError_t launch_rows(const CUtensorMap* tm_w, const CUtensorMap* tm_a, const CUtensorMap* tm_ascale,
                        const float* w_scale, const Layout& L, uint8_t* ws, int num_sms, bool w1_packed,
                        const RowsOut& out, cudaStream_t stream) {
  static DeviceFlags attr_set;
  if (cudaError_t err = set_max_dynamic_smem(gemm_rows_fp8_kernel<M>, kSmemBytes, attr_set); err != cudaSuccess)
    return err;
  const long max_units = (long)L.max_blocks * RowsCfg<M>::kTiles;
  int grid = (int)(max_units < num_sms ? max_units : num_sms);
  if (grid < 1) grid = 1;
  return launch_pdl(gemm_rows_fp8_kernel<M>, dim3(grid), dim3(kThreads), kSmemBytes, stream, *tm_w, *tm_a,
                    *tm_ascale, w_scale, reinterpret_cast<const int32_t*>(ws + L.n_blocks),
                    reinterpret_cast<const int4*>(ws + L.blocks), out, reinterpret_cast<uint32_t*>(ws + L.status),
                    L.e_local, L.pcap, w1_packed ? 1 : 0);
}

}  // namespace

cudaError_t launch_gemm1_rows(const CUtensorMap* tm_w1, const CUtensorMap* tm_aperm, const CUtensorMap* tm_ascale,
                              const float* w1_scale, const Layout& L, uint8_t* ws, int num_sms, bool w1_packed,
                              cudaStream_t stream, bool fp8_inter) {
  RowsOut out{};
  if (fp8_inter) {
    out.inter8 = ws + L.inter;
    out.iscale = reinterpret_cast<float*>(ws + L.inter + fp8_inter_scale_offset(L));
    return launch_rows<kOutFp8>(tm_w1, tm_aperm, tm_ascale, w1_scale, L, ws, num_sms, w1_packed, out, stream);
  }
  out.inter = reinterpret_cast<__half*>(ws + L.inter);
  return launch_rows<kOutF16>(tm_w1, tm_aperm, tm_ascale, w1_scale, L, ws, num_sms, w1_packed, out, stream);
}

cudaError_t launch_gemm2_fp8_rows(const CUtensorMap* tm_w2, const CUtensorMap* tm_inter8,
                                  const CUtensorMap* tm_iscale, const float* w2_scale, const Layout& L, uint8_t* ws,
                                  int num_sms, cudaStream_t stream, const PeerScatter* scatter) {
  RowsOut out{};
  out.row_weight = reinterpret_cast<const float*>(ws + L.row_weight);
  out.pair_out = reinterpret_cast<__half*>(ws + L.pair_out);
  out.row_token = reinterpret_cast<const int32_t*>(ws + L.row_token);
  out.token_rows = reinterpret_cast<const int32_t*>(ws + L.token_rows);
  if (scatter != nullptr) out.ps = *scatter;
  out.T = L.tokens;
  return launch_rows<kPairOut>(tm_w2, tm_inter8, tm_iscale, w2_scale, L, ws, num_sms, false, out, stream);
}

}  // namespace fbmoe
