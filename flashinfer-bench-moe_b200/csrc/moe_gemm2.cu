// moe_gemm2.cu -- grouped GEMM2 with the routing-weighted epilogue
// (tcgen05 + TMEM + TMA), sm_100a.
//
// Reference counterpart: gemm2_kernel (Triton, solution/triton/main.py:433-600):
//     O[r, h] = w[r] * sum_j inter[r, j] * W2[e, h, j] * s2[e, h/128, j/128]
// written as one row per (token, local expert) pair.
//
// W2 arrives as FP8 with fp32 128x128 block scales.  Because the intermediate
// is f16, this GEMM runs as a kind::f16 (f16 x f16 -> fp32) MMA: converter
// warps dequantise each 128x128 W2 tile on chip (fp8 * s2 in fp32, rounded
// once to f16) into the UMMA operand layout.  With the scale folded into the
// operand no promotion is needed; TMEM accumulates the full K = 2048.
// The weighted pair rows are written as f16 (clamped to +-65504, flagged) and
// summed in fp32 by the combine kernel.
//
// Orientation (swap-AB): A = 128 rows of W2 (one 128-row scale block of the
// hidden dimension), B = BN intermediate rows of one expert (TMA, two 64-column
// boxes per K-block).  One work unit = (block of BN rows) x (slice of 128 hidden
// columns); its accumulator is double-buffered in TMEM so the epilogue of one
// unit overlaps the MMAs of the next.
//
// Split-K (decode): with splits[1] = S > 1 each unit's 16 K-blocks are shared
// by S work items; item s writes plane s of pair_out and the combine kernel adds
// the planes.
//
// Three shared-memory rings: a ring of raw FP8 W2 tiles (16 KB each; the bytes
// that stream from HBM), a ring of converted f16 W2 tiles (3 deep for small
// blocks, so the converters run two stages ahead of the MMA), and a
// deep ring of intermediate rows (their L2 latency must not sit on the critical
// path: with the rows in the converted ring, decode ran at ~10 GB/s per SM).
//
// Warp roles (384 threads): w0 W2 producer (TMA), w1 MMA issuer + TMEM owner,
// w2 intermediate producer (TMA), w3 idle, w4-w7 converters (one W2 row each),
// w8-w11 epilogue.
#include "fbmoe_common.cuh"
#include "fbmoe_launch.h"

namespace fbmoe {
namespace {

constexpr int kG2Threads = 384;
constexpr int kG2Slices = kHidden / 128;  // 56
constexpr uint64_t kWaitBudgetNs = 4000000000ull;

template <int BN>
struct G2Cfg {
  static constexpr int kRawStages = BN <= 32 ? 4 : 3;
  static constexpr int kConvStages = BN <= 32 ? 3 : 2;
  static constexpr int kBStages = BN <= 16 ? 6 : BN <= 32 ? 4 : BN <= 64 ? 4 : 2;
  static constexpr int kRawBytes = 128 * 128;      // fp8 W2 tile
  static constexpr int kAhBytes = 2 * 128 * 128;   // f16 W2 tile (two 64-K halves)
  static constexpr int kBBytes = BN * 256;         // f16 intermediate rows (two 64-K halves)
  static constexpr int kTmemCols = (2 * BN < 32) ? 32 : 2 * BN;
  static constexpr int kOffRaw = 0;
  static constexpr int kOffAh = kOffRaw + kRawStages * kRawBytes;
  static constexpr int kOffB = kOffAh + kConvStages * kAhBytes;
  static constexpr int kOffBar = kOffB + kBStages * kBBytes;
  static constexpr int kNumBars = 2 * kRawStages + 2 * kConvStages + 2 * kBStages + 4 + 1;
  static constexpr int kOffMisc = kOffBar + kNumBars * 8;
  static constexpr int kBytes = kOffMisc + 16 + 1024;
};

// 4 fp8 (e4m3) -> 4 f16, each times `scale` (exact widening, fp32 multiply, one rounding).
__device__ __forceinline__ uint2 fp8x4_to_f16x4(uint32_t q, float scale) {
  const __half2_raw h01 = __nv_cvt_fp8x2_to_halfraw2((__nv_fp8x2_storage_t)(q & 0xFFFFu), __NV_E4M3);
  const __half2_raw h23 = __nv_cvt_fp8x2_to_halfraw2((__nv_fp8x2_storage_t)(q >> 16), __NV_E4M3);
  const float2 f01 = __half22float2(*reinterpret_cast<const __half2*>(&h01));
  const float2 f23 = __half22float2(*reinterpret_cast<const __half2*>(&h23));
  const __half2 o01 = __floats2half2_rn(f01.x * scale, f01.y * scale);
  const __half2 o23 = __floats2half2_rn(f23.x * scale, f23.y * scale);
  return make_uint2(*reinterpret_cast<const uint32_t*>(&o01), *reinterpret_cast<const uint32_t*>(&o23));
}

// Ring position: slot and phase parity of successive uses of a ring of n slots.
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

template <int BN>
__global__ void __launch_bounds__(kG2Threads, 1)
    gemm2_combine_kernel(const __grid_constant__ CUtensorMap tm_w2, const __grid_constant__ CUtensorMap tm_inter,
                         const float* __restrict__ w2_scale, const int32_t* __restrict__ n_blocks_ptr,
                         const int4* __restrict__ blocks, const float* __restrict__ row_weight,
                         __half* __restrict__ pair_out, uint32_t* __restrict__ status,
                         const int32_t* __restrict__ splits, size_t plane_elems) {
  using C = G2Cfg<BN>;
  constexpr int SR = C::kRawStages;
  constexpr int SC = C::kConvStages;
  constexpr int SB = C::kBStages;
  // Decode-sized blocks read each W2 tile about once: stream it past L2.
  constexpr bool kStreamWeights = (BN <= 16);
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sRaw = sm + C::kOffRaw;
  uint8_t* sAh = sm + C::kOffAh;
  uint8_t* sB = sm + C::kOffB;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + C::kOffBar);
  uint64_t* raw_full = bars;                   // raw W2 tile landed (TMA)
  uint64_t* raw_empty = bars + SR;             // converters done reading it
  uint64_t* a_full = bars + 2 * SR;            // f16 W2 tile written by the converters
  uint64_t* c_empty = bars + 2 * SR + SC;       // MMA done with the converted slot
  uint64_t* b_full = bars + 2 * SR + 2 * SC;    // intermediate rows landed (TMA)
  uint64_t* b_empty = b_full + SB;              // MMA done with the intermediate slot
  uint64_t* tfull = b_empty + SB;
  uint64_t* tempty = tfull + 2;
  uint64_t* drain = tfull + 4;
  uint32_t* sTmem = reinterpret_cast<uint32_t*>(sm + C::kOffMisc);
  volatile int* sAbort = reinterpret_cast<volatile int*>(sm + C::kOffMisc + 4);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < SR; ++s) {
      mbar_init(&raw_full[s], 1);
      mbar_init(&raw_empty[s], 4);
    }
    for (int s = 0; s < SC; ++s) {
      mbar_init(&a_full[s], 4);
      mbar_init(&c_empty[s], 1);
    }
    for (int s = 0; s < SB; ++s) {
      mbar_init(&b_full[s], 1);
      mbar_init(&b_empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], 4);
    }
    mbar_init(drain, 1);
    *sAbort = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tm_w2);
    tma_prefetch_desc(&tm_inter);
  }
  if (warp == 1) {
    tmem_alloc(sTmem, C::kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  // The block list and row weights come from the permute kernel, which finished
  // before GEMM1 let this grid launch; only the intermediate rows (GEMM1's
  // output) need the wait, done by the thread that loads them.
  pdl_trigger();
  const uint32_t tmem_base = *sTmem;
  const int n_units = (*n_blocks_ptr) * kG2Slices;
  const int n_split = splits[1];                  // K splits per unit (1 unless decode)
  const int nk = kIBlocks / n_split;              // K-blocks per work item
  const int n_items = n_units * n_split;

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
      const uint64_t pol = w2_side ? l2_policy_evict_first() : l2_policy_evict_last();
      const int n = w2_side ? SR : SB;
      uint64_t* fullb = w2_side ? raw_full : b_full;
      uint64_t* emptyb = w2_side ? raw_empty : b_empty;
      Ring ring(n);
      bool ok = true;
      uint32_t last_parity[SR > SB ? SR : SB];
      for (int s = 0; s < n; ++s) last_parity[s] = 0xFFFFFFFFu;
      for (int it = blockIdx.x; it < n_items && ok; it += gridDim.x) {
        const int u = it / n_split, sp = it % n_split;
        const int4 blk = blocks[u / kG2Slices];
        const int h = u % kG2Slices;
        const int e = blk.x, r0 = blk.y;
        for (int kb = sp * nk; kb < (sp + 1) * nk; ++kb) {
          if (!mbar_wait(&emptyb[ring.slot], ring.phase ^ 1u, sAbort, kWaitBudgetNs)) {
            ok = false;
            fail(kStatusTimeoutProducer);
            break;
          }
          if (w2_side) {
            mbar_arrive_expect_tx(&fullb[ring.slot], C::kRawBytes);
            if (kStreamWeights)
              tma_load_2d(sRaw + ring.slot * C::kRawBytes, &tm_w2, &fullb[ring.slot], kb * kBlk,
                          e * kHidden + h * 128, pol);
            else
              tma_load_2d_nohint(sRaw + ring.slot * C::kRawBytes, &tm_w2, &fullb[ring.slot], kb * kBlk,
                                 e * kHidden + h * 128);
          } else {
            uint8_t* b = sB + ring.slot * C::kBBytes;
            mbar_arrive_expect_tx(&fullb[ring.slot], C::kBBytes);
            tma_load_2d(b, &tm_inter, &fullb[ring.slot], kb * kBlk, r0, pol);
            tma_load_2d(b + BN * 128, &tm_inter, &fullb[ring.slot], kb * kBlk + 64, r0, pol);
          }
          last_parity[ring.slot] = ring.phase;
          ring.next();
        }
      }
      // every issued TMA load lands before the CTA exits
      for (int s = 0; s < n; ++s)
        if (last_parity[s] != 0xFFFFFFFFu)
          if (!mbar_wait(&fullb[s], last_parity[s], sAbort, kWaitBudgetNs) && !*sAbort) fail(kStatusTimeoutDrain);
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = umma_idesc(0u, 128, BN);  // f16 x f16
      Ring ring(SC), bring(SB);
      uint32_t ug = 0;
      bool ok = true;
      bool any = false;
      for (int it = blockIdx.x; it < n_items && ok; it += gridDim.x, ++ug) {
        const uint32_t buf = ug & 1u;
        if (!mbar_wait(&tempty[buf], ((ug >> 1) & 1u) ^ 1u, sAbort, kWaitBudgetNs)) {
          ok = false;
          fail(kStatusTimeoutMma);
          break;
        }
        tc_fence_after();
        const uint32_t d = tmem_base + buf * BN;
        for (int kb = 0; kb < nk; ++kb) {
          if (!mbar_wait(&a_full[ring.slot], ring.phase, sAbort, kWaitBudgetNs) ||
              !mbar_wait(&b_full[bring.slot], bring.phase, sAbort, kWaitBudgetNs)) {
            ok = false;
            fail(kStatusTimeoutMma);
            break;
          }
          tc_fence_after();
#pragma unroll
          for (int half = 0; half < 2; ++half) {
            const uint64_t adesc = umma_desc_sw128(smem_u32(sAh + ring.slot * C::kAhBytes + half * 128 * 128));
            const uint64_t bdesc = umma_desc_sw128(smem_u32(sB + bring.slot * C::kBBytes + half * BN * 128));
#pragma unroll
            for (int j = 0; j < 4; ++j)
              mma_f16(d, adesc + 2 * j, bdesc + 2 * j, idesc, (kb | half | j) ? 1u : 0u);
          }
          tc_commit(&c_empty[ring.slot]);
          tc_commit(&b_empty[bring.slot]);
          any = true;
          ring.next();
          bring.next();
        }
        if (!ok) break;
        tc_commit(&tfull[buf]);
      }
      if (any) {
        tc_commit(drain);
        mbar_wait(drain, 0, sAbort, kWaitBudgetNs);
      }
    }
    __syncwarp();
  } else if (warp >= 4 && warp < 8) {
    // ------------------------------------------------------------ converters
    const int r = threadIdx.x - 128;  // W2 row within the tile
    Ring rr(SR), cr(SC);
    bool ok = true;
    for (int it = blockIdx.x; it < n_items && ok; it += gridDim.x) {
      const int u = it / n_split, sp = it % n_split;
      const int4 blk = blocks[u / kG2Slices];
      const int h = u % kG2Slices;
      const float* sc = w2_scale + ((size_t)blk.x * kHBlocks + h) * kIBlocks;
      // the unit's 16 scales, one per lane: no global load on the per-stage path
      const float lane_scale = __ldg(sc + (lane & (kIBlocks - 1)));
      for (int kb = sp * nk; kb < (sp + 1) * nk; ++kb) {
        if (!mbar_wait(&raw_full[rr.slot], rr.phase, sAbort, kWaitBudgetNs) ||
            !mbar_wait(&c_empty[cr.slot], cr.phase ^ 1u, sAbort, kWaitBudgetNs)) {
          ok = false;
          if (lane == 0) fail(kStatusTimeoutConvert);
          break;
        }
        const float scale = __shfl_sync(0xffffffffu, lane_scale, kb);
        const uint8_t* raw = sRaw + rr.slot * C::kRawBytes;
        uint8_t* ah = sAh + cr.slot * C::kAhBytes;
#pragma unroll
        for (int c = 0; c < 8; ++c) {
          const uint4 q = *reinterpret_cast<const uint4*>(raw + sw128_offset(r, c));
          const uint2 o0 = fp8x4_to_f16x4(q.x, scale);
          const uint2 o1 = fp8x4_to_f16x4(q.y, scale);
          const uint2 o2 = fp8x4_to_f16x4(q.z, scale);
          const uint2 o3 = fp8x4_to_f16x4(q.w, scale);
          uint8_t* dst = ah + (c >> 2) * (128 * 128);
          const int c2 = (c & 3) * 2;
          *reinterpret_cast<uint4*>(dst + sw128_offset(r, c2)) = make_uint4(o0.x, o0.y, o1.x, o1.y);
          *reinterpret_cast<uint4*>(dst + sw128_offset(r, c2 + 1)) = make_uint4(o2.x, o2.y, o3.x, o3.y);
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          mbar_arrive(&raw_empty[rr.slot]);
          mbar_arrive(&a_full[cr.slot]);
        }
        rr.next();
        cr.next();
      }
    }
  } else if (warp >= 8) {
    // ------------------------------------------------------------ epilogue
    const int ew = warp - 8;
    const int hrow = ew * 32 + lane;
    const uint32_t lane_base = (uint32_t)(ew * 32) << 16;
    uint32_t ug = 0;
    bool ok = true;
    for (int it = blockIdx.x; it < n_items && ok; it += gridDim.x, ++ug) {
      const int u = it / n_split, sp = it % n_split;
      const int4 blk = blocks[u / kG2Slices];
      const int h = u % kG2Slices;
      const int r0 = blk.y, nrows = blk.z;
      const uint32_t buf = ug & 1u;
      if (!mbar_wait(&tfull[buf], (ug >> 1) & 1u, sAbort, kWaitBudgetNs)) {
        ok = false;
        if (lane == 0) fail(kStatusTimeoutEpilogue);
        break;
      }
      tc_fence_after();
      __half* dst = pair_out + (size_t)sp * plane_elems + (size_t)r0 * kHidden + h * 128 + hrow;
      const float* wrow = row_weight + r0;
      bool sat = false;
#pragma unroll
      for (int c = 0; c < BN / 16; ++c) {
        float p[16];
        tmem_ld16(tmem_base + lane_base + buf * BN + c * 16, p);
        tmem_wait_ld();
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const int t = c * 16 + i;
          if (t < nrows) dst[(size_t)t * kHidden] = to_half_sat(p[i] * __ldg(wrow + t), sat);
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty[buf]);
      if (sat) atomicOr(status, kStatusSaturated);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, C::kTmemCols);
  }
}

template <int BN>
cudaError_t launch_g2(const CUtensorMap* tm_w2, const CUtensorMap* tm_inter, const float* w2_scale,
                      const Layout& L, uint8_t* ws, int num_sms, cudaStream_t stream) {
  using C = G2Cfg<BN>;
  static_assert(C::kBytes <= 227 * 1024, "GEMM2 shared memory over the per-CTA limit");
  static bool attr_set[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 64 && !attr_set[dev]) {
    cudaError_t err =
        cudaFuncSetAttribute(gemm2_combine_kernel<BN>, cudaFuncAttributeMaxDynamicSharedMemorySize, C::kBytes);
    if (err != cudaSuccess) return err;
    attr_set[dev] = true;
  }
  long max_units = (long)L.max_blocks * kG2Slices;
  int grid = (int)(max_units < num_sms ? max_units : num_sms);
  if (grid < 1) grid = 1;
  return launch_pdl(gemm2_combine_kernel<BN>, dim3(grid), dim3(kG2Threads), C::kBytes, stream, *tm_w2, *tm_inter,
                    w2_scale, reinterpret_cast<const int32_t*>(ws + L.n_blocks),
                    reinterpret_cast<const int4*>(ws + L.blocks), reinterpret_cast<const float*>(ws + L.row_weight),
                    reinterpret_cast<__half*>(ws + L.pair_out), reinterpret_cast<uint32_t*>(ws + L.status),
                    reinterpret_cast<const int32_t*>(ws + L.splits), (size_t)L.pcap * kHidden);
}

}  // namespace

cudaError_t launch_gemm2(const CUtensorMap* tm_w2, const CUtensorMap* tm_inter, const float* w2_scale,
                         int E_local, int bn, const Layout& L, uint8_t* ws, int num_sms, cudaStream_t stream) {
  (void)E_local;
  switch (bn) {
    case 16: return launch_g2<16>(tm_w2, tm_inter, w2_scale, L, ws, num_sms, stream);
    case 128: return launch_g2<128>(tm_w2, tm_inter, w2_scale, L, ws, num_sms, stream);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace fbmoe
