// moe_gemm1_rows.cu -- GEMM1 + SwiGLU for large token blocks (prefill), with
// the tokens as the MMA's M operand (tcgen05 kind::f8f6f4, TMEM, TMA), sm_100a.
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
#include "fbmoe_common.cuh"
#include "fbmoe_launch.h"

namespace fbmoe {
namespace {

constexpr int kThreads = 576;
constexpr int kEpiWarps = 16;
constexpr int kRows = 128;                       // token rows per block (== block_rows 128)
constexpr int kTiles = kInter / 128;             // 16 tiles of 128 intermediate columns
constexpr int kStages = 4;
constexpr int kABytes = kRows * 128;             // 16 KB of gathered token rows
constexpr int kBBytes = 256 * 128;               // 32 KB of W1 rows
constexpr uint64_t kWaitBudgetNs = 4000000000ull;
constexpr int kOffA = 0;
constexpr int kOffB = kOffA + kStages * kABytes;
constexpr int kScaleSlots = 8;                   // ring of per-K-block row-scale vectors
constexpr int kOffAS = kOffB + kStages * kBBytes;            // fp32 [8][128] row scales
constexpr int kOffWS = kOffAS + kScaleSlots * kRows * 4;    // fp32 [2][112] W1 scales of a unit
constexpr int kOffBar = kOffWS + 2 * 2 * kHBlocks * 4;
constexpr int kNumBars = 2 * kStages + 4 + 1 + kScaleSlots + 2;
constexpr int kOffMisc = kOffBar + kNumBars * 8;
constexpr int kSmemBytes = kOffMisc + 16 + 1024;
static_assert(kSmemBytes <= 227 * 1024, "shared memory over the per-CTA limit");

__global__ void __launch_bounds__(kThreads, 1)
    gemm1_rows_kernel(const __grid_constant__ CUtensorMap tm_w1, const __grid_constant__ CUtensorMap tm_aperm,
                      const __grid_constant__ CUtensorMap tm_ascale, const float* __restrict__ w1_scale,
                      const int32_t* __restrict__ n_blocks_ptr, const int4* __restrict__ blocks,
                      __half* __restrict__ inter,
                      uint32_t* __restrict__ status, int e_local, int pcap, int w1_packed) {
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
  uint64_t* wfull = sfull + kScaleSlots;     // W1 scales of a unit landed in slot (unit % 2)
  float* sAS = reinterpret_cast<float*>(sm + kOffAS);
  float* sWS = reinterpret_cast<float*>(sm + kOffWS);
  uint32_t* sTmem = reinterpret_cast<uint32_t*>(sm + kOffMisc);
  volatile int* sAbort = reinterpret_cast<volatile int*>(sm + kOffMisc + 4);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);   // producer's expect_tx arrive (W1 tiles + row gathers)
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
    *sAbort = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tm_w1);
    tma_prefetch_desc(&tm_aperm);
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
    // x % 8 and, at a unit's first K-block, its W1 scales into slot unit % 2.
    // Slot reuse is safe without extra barriers: loads for K-block x start only
    // after MMA x - 4 completed, which needed the epilogue done with x - 6 (two
    // TMEM buffers); slot x % 8 last held x - 8, and unit slots are 56 K-blocks apart.
    int stage = 0;
    uint32_t phase = 0;
    bool ok = true;
    uint32_t issued_mask = 0, parity_mask = 0;  // per stage: ever issued / parity of the last issue
    int x = 0, ui = 0;
    for (int u = blockIdx.x; u < n_units && ok; u += gridDim.x, ++ui) {
      const int4 blk = dbg_block(blocks[u / kTiles], kRows, e_local, pcap, status);
      const int j = u % kTiles;
      const int e = blk.x, r0 = blk.y;
      const int wrow = e * kGemm1N + 128 * j;
      for (int kb = 0; kb < kHBlocks; ++kb, ++x) {
        if (!mbar_wait(&empty[stage], phase ^ 1u, sAbort, kWaitBudgetNs)) {
          ok = false;
          if (lane == 0) fail(kStatusTimeoutProducer);
          break;
        }
        if (lane == 0) {
          if (kb == 0) {
            uint64_t* wb = &wfull[ui & 1];
            float* wdst = sWS + (ui & 1) * 2 * kHBlocks;
            mbar_arrive_expect_tx(wb, 2 * kHBlocks * 4);
            bulk_load_1d(wdst, w1_scale + ((size_t)e * (kGemm1N / kBlk) + j) * kHBlocks, kHBlocks * 4, wb);
            bulk_load_1d(wdst + kHBlocks, w1_scale + ((size_t)e * (kGemm1N / kBlk) + kIBlocks + j) * kHBlocks,
                         kHBlocks * 4, wb);
          }
          uint64_t* sb = &sfull[x & (kScaleSlots - 1)];
          mbar_arrive_expect_tx(sb, kRows * 4);
          tma_load_2d_nohint(sAS + (x & (kScaleSlots - 1)) * kRows, &tm_ascale, sb, r0, kb);
          mbar_arrive_expect_tx(&full[stage], kABytes + kBBytes);
          tma_load_2d_nohint(sA + stage * kABytes, &tm_aperm, &full[stage], kb * kBlk, r0);
          uint8_t* b = sB + stage * kBBytes;
          if (w1_packed) {
            // packed rows [256j, 256j + 256): X1 2j, X2 2j, X1 2j+1, X2 2j+1 (64 rows each), one box
            tma_load_2d_nohint(b, &tm_w1, &full[stage], kb * kBlk, e * kGemm1N + 256 * j);
          } else {
            tma_load_2d_nohint(b, &tm_w1, &full[stage], kb * kBlk, wrow);
            tma_load_2d_nohint(b + 64 * 128, &tm_w1, &full[stage], kb * kBlk, wrow + 64);
            tma_load_2d_nohint(b + 128 * 128, &tm_w1, &full[stage], kb * kBlk, wrow + kInter);
            tma_load_2d_nohint(b + 192 * 128, &tm_w1, &full[stage], kb * kBlk, wrow + kInter + 64);
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
        for (int kb = 0; kb < kHBlocks; ++kb) {
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
    const int g = (warp - 2) >> 2;     // output columns [32g, 32g+32) of the tile
    const int row = q * 32 + lane;     // token row in the block == TMEM lane
    const uint32_t lane_base = (uint32_t)(q * 32) << 16;
    // TMEM columns of this warp's 32 X1 and 32 X2 columns: raw layout X1 0-127 | X2 128-255;
    // packed layout in 64-column runs X1 | X2 | X1 | X2
    const uint32_t x1_col = w1_packed ? (uint32_t)((g >> 1) * 128 + (g & 1) * 32) : (uint32_t)(32 * g);
    const uint32_t x2_col = w1_packed ? x1_col + 64u : (uint32_t)(128 + 32 * g);
    uint32_t kbg = 0;
    bool ok = true;
    int ui = 0;
    for (int u = blockIdx.x; u < n_units && ok; u += gridDim.x, ++ui) {
      const int4 blk = dbg_block(blocks[u / kTiles], kRows, e_local, pcap, status);
      const int j = u % kTiles;
      const int r0 = blk.y, nrows = blk.z;
      // this unit's W1 scales: [0, 56) first half, [56, 112) second half
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
      for (int kb = 0; kb < kHBlocks; ++kb) {
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
      if (row < nrows) {
        bool sat = false;
        uint4* dst = reinterpret_cast<uint4*>(inter + (size_t)(r0 + row) * kInter + 128 * j + 32 * g);
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
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, 512);
  }
}

}  // namespace

cudaError_t launch_gemm1_rows(const CUtensorMap* tm_w1, const CUtensorMap* tm_aperm, const CUtensorMap* tm_ascale,
                              const float* w1_scale, const Layout& L, uint8_t* ws, int num_sms, bool w1_packed,
                              cudaStream_t stream) {
  static DeviceFlags attr_set;
  if (cudaError_t err = set_max_dynamic_smem(gemm1_rows_kernel, kSmemBytes, attr_set); err != cudaSuccess) return err;
  const long max_units = (long)L.max_blocks * kTiles;
  int grid = (int)(max_units < num_sms ? max_units : num_sms);
  if (grid < 1) grid = 1;
  return launch_pdl(gemm1_rows_kernel, dim3(grid), dim3(kThreads), kSmemBytes, stream, *tm_w1, *tm_aperm,
                    *tm_ascale, w1_scale, reinterpret_cast<const int32_t*>(ws + L.n_blocks),
                    reinterpret_cast<const int4*>(ws + L.blocks), reinterpret_cast<__half*>(ws + L.inter),
                    reinterpret_cast<uint32_t*>(ws + L.status), L.e_local, L.pcap, w1_packed ? 1 : 0);
}

}  // namespace fbmoe
