// moe_gemm2.cu -- grouped GEMM2 with the routing-weighted epilogue
// (tcgen05 + TMEM + TMA), sm_100a.
//
// Reference counterpart: gemm2_kernel (Triton, solution/triton/main.py:433-600):
//     O[r, h] = w[r] * sum_j inter[r, j] * W2[e, h, j] * s2[e, h/128, j/128]
// written as one bf16 row per (token, local expert) pair.
//
// W2 arrives as FP8 with fp32 128x128 block scales.  Because the intermediate
// is bf16, this GEMM runs as a kind::f16 (bf16 x bf16 -> fp32) MMA: converter
// warps dequantise each 128x128 W2 tile on chip (fp8 * s2 in fp32, rounded
// once to bf16) into the UMMA operand layout.  With the scale folded into the
// operand no promotion is needed; TMEM accumulates the full K = 2048.
//
// Orientation (swap-AB): A = 128 rows of W2 (one 128-row scale block of the
// hidden dimension), B = BN intermediate rows of one expert (TMA, two 64-column
// boxes per K-block).  One work unit = (block of BN rows) x (slice of 128 hidden
// columns); its accumulator is double-buffered in TMEM so the epilogue of one
// unit overlaps the MMAs of the next.
//
// Warp roles (384 threads): w0 producer (TMA), w1 MMA issuer + TMEM owner,
// w2-w3 idle, w4-w7 converters (one W2 row each), w8-w11 epilogue.
#include "fbmoe_common.cuh"
#include "fbmoe_launch.h"

namespace fbmoe {
namespace {

constexpr int kG2Threads = 384;
constexpr int kG2Slices = kHidden / 128;  // 56
constexpr uint64_t kWaitBudgetNs = 4000000000ull;

template <int BN>
struct G2Cfg {
  static constexpr int kStages = BN <= 32 ? 4 : 3;
  static constexpr int kRawBytes = 128 * 128;      // fp8 W2 tile
  static constexpr int kAbfBytes = 2 * 128 * 128;  // bf16 W2 tile (two 64-K halves)
  static constexpr int kBBytes = BN * 256;         // bf16 intermediate rows (two 64-K halves)
  static constexpr int kTmemCols = (2 * BN < 32) ? 32 : 2 * BN;
  static constexpr int kOffRaw = 0;
  static constexpr int kOffAbf = kOffRaw + kStages * kRawBytes;
  static constexpr int kOffB = kOffAbf + kStages * kAbfBytes;
  static constexpr int kOffW = kOffB + kStages * kBBytes;
  static constexpr int kOffBar = (kOffW + BN * 4 + 7) / 8 * 8;
  static constexpr int kNumBars = 3 * kStages + 4 + 1;
  static constexpr int kOffMisc = kOffBar + kNumBars * 8;
  static constexpr int kBytes = kOffMisc + 16 + 1024;
};

// 4 fp8 (e4m3) -> 4 bf16, each times `scale` (fp32 multiply, one rounding).
__device__ __forceinline__ uint2 fp8x4_to_bf16x4(uint32_t q, float scale) {
  const __half2_raw h01 = __nv_cvt_fp8x2_to_halfraw2((__nv_fp8x2_storage_t)(q & 0xFFFFu), __NV_E4M3);
  const __half2_raw h23 = __nv_cvt_fp8x2_to_halfraw2((__nv_fp8x2_storage_t)(q >> 16), __NV_E4M3);
  const float2 f01 = __half22float2(*reinterpret_cast<const __half2*>(&h01));
  const float2 f23 = __half22float2(*reinterpret_cast<const __half2*>(&h23));
  const __nv_bfloat162 b01 = __floats2bfloat162_rn(f01.x * scale, f01.y * scale);
  const __nv_bfloat162 b23 = __floats2bfloat162_rn(f23.x * scale, f23.y * scale);
  return make_uint2(*reinterpret_cast<const uint32_t*>(&b01), *reinterpret_cast<const uint32_t*>(&b23));
}

template <int BN>
__global__ void __launch_bounds__(kG2Threads, 1)
    gemm2_combine_kernel(const __grid_constant__ CUtensorMap tm_w2, const __grid_constant__ CUtensorMap tm_inter,
                         const float* __restrict__ w2_scale, const int32_t* __restrict__ n_blocks_ptr,
                         const int4* __restrict__ blocks, const float* __restrict__ row_weight,
                         __nv_bfloat16* __restrict__ pair_out, uint32_t* __restrict__ status) {
  using C = G2Cfg<BN>;
  constexpr int S = C::kStages;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sRaw = sm + C::kOffRaw;
  uint8_t* sAbf = sm + C::kOffAbf;
  uint8_t* sB = sm + C::kOffB;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + C::kOffBar);
  uint64_t* full = bars;            // TMA landed (raw W2 + B)
  uint64_t* conv = bars + S;        // bf16 W2 written
  uint64_t* empty = bars + 2 * S;   // MMA done with the stage
  uint64_t* tfull = bars + 3 * S;
  uint64_t* tempty = bars + 3 * S + 2;
  uint64_t* drain = bars + 3 * S + 4;
  uint32_t* sTmem = reinterpret_cast<uint32_t*>(sm + C::kOffMisc);
  volatile int* sAbort = reinterpret_cast<volatile int*>(sm + C::kOffMisc + 4);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&conv[s], 4);
      mbar_init(&empty[s], 1);
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
  const uint32_t tmem_base = *sTmem;
  const int n_units = (*n_blocks_ptr) * kG2Slices;

  auto fail = [&](uint32_t bit) {
    *sAbort = 1;
    atomicOr(status, bit);
  };

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      const uint64_t pol_w = l2_policy_evict_first();
      const uint64_t pol_a = l2_policy_evict_last();
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      uint32_t last_parity[S];
      for (int s = 0; s < S; ++s) last_parity[s] = 0xFFFFFFFFu;
      for (int u = blockIdx.x; u < n_units && ok; u += gridDim.x) {
        const int4 blk = blocks[u / kG2Slices];
        const int h = u % kG2Slices;
        const int e = blk.x, r0 = blk.y;
        for (int kb = 0; kb < kIBlocks; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1u, sAbort, kWaitBudgetNs)) {
            ok = false;
            fail(kStatusTimeoutProducer);
            break;
          }
          mbar_arrive_expect_tx(&full[stage], C::kRawBytes + C::kBBytes);
          tma_load_2d(sRaw + stage * C::kRawBytes, &tm_w2, &full[stage], kb * kBlk, e * kHidden + h * 128, pol_w);
          uint8_t* b = sB + stage * C::kBBytes;
          tma_load_2d(b, &tm_inter, &full[stage], kb * kBlk, r0, pol_a);
          tma_load_2d(b + BN * 128, &tm_inter, &full[stage], kb * kBlk + 64, r0, pol_a);
          last_parity[stage] = phase;
          if (++stage == S) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      for (int s = 0; s < S; ++s)
        if (last_parity[s] != 0xFFFFFFFFu)
          if (!mbar_wait(&full[s], last_parity[s], sAbort, kWaitBudgetNs) && !*sAbort) fail(kStatusTimeoutDrain);
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = umma_idesc(1u, 128, BN);  // bf16 x bf16
      int stage = 0;
      uint32_t phase = 0;
      uint32_t ug = 0;
      bool ok = true;
      bool any = false;
      for (int u = blockIdx.x; u < n_units && ok; u += gridDim.x, ++ug) {
        const uint32_t buf = ug & 1u;
        if (!mbar_wait(&tempty[buf], ((ug >> 1) & 1u) ^ 1u, sAbort, kWaitBudgetNs)) {
          ok = false;
          fail(kStatusTimeoutMma);
          break;
        }
        tc_fence_after();
        const uint32_t d = tmem_base + buf * BN;
        for (int kb = 0; kb < kIBlocks; ++kb) {
          if (!mbar_wait(&conv[stage], phase, sAbort, kWaitBudgetNs) ||
              !mbar_wait(&full[stage], phase, sAbort, kWaitBudgetNs)) {
            ok = false;
            fail(kStatusTimeoutMma);
            break;
          }
          tc_fence_after();
#pragma unroll
          for (int half = 0; half < 2; ++half) {
            const uint64_t adesc = umma_desc_sw128(smem_u32(sAbf + stage * C::kAbfBytes + half * 128 * 128));
            const uint64_t bdesc = umma_desc_sw128(smem_u32(sB + stage * C::kBBytes + half * BN * 128));
#pragma unroll
            for (int j = 0; j < 4; ++j)
              mma_f16(d, adesc + 2 * j, bdesc + 2 * j, idesc, (kb | half | j) ? 1u : 0u);
          }
          tc_commit(&empty[stage]);
          any = true;
          if (++stage == S) {
            stage = 0;
            phase ^= 1u;
          }
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
    int stage = 0;
    uint32_t phase = 0;
    bool ok = true;
    for (int u = blockIdx.x; u < n_units && ok; u += gridDim.x) {
      const int4 blk = blocks[u / kG2Slices];
      const int h = u % kG2Slices;
      const float* sc = w2_scale + ((size_t)blk.x * kHBlocks + h) * kIBlocks;
      for (int kb = 0; kb < kIBlocks; ++kb) {
        if (!mbar_wait(&full[stage], phase, sAbort, kWaitBudgetNs)) {
          ok = false;
          if (lane == 0) fail(kStatusTimeoutConvert);
          break;
        }
        const float scale = __ldg(sc + kb);
        const uint8_t* raw = sRaw + stage * C::kRawBytes;
        uint8_t* abf = sAbf + stage * C::kAbfBytes;
#pragma unroll
        for (int c = 0; c < 8; ++c) {
          const uint4 q = *reinterpret_cast<const uint4*>(raw + sw128_offset(r, c));
          const uint2 o0 = fp8x4_to_bf16x4(q.x, scale);
          const uint2 o1 = fp8x4_to_bf16x4(q.y, scale);
          const uint2 o2 = fp8x4_to_bf16x4(q.z, scale);
          const uint2 o3 = fp8x4_to_bf16x4(q.w, scale);
          uint8_t* dst = abf + (c >> 2) * (128 * 128);
          const int c2 = (c & 3) * 2;
          *reinterpret_cast<uint4*>(dst + sw128_offset(r, c2)) = make_uint4(o0.x, o0.y, o1.x, o1.y);
          *reinterpret_cast<uint4*>(dst + sw128_offset(r, c2 + 1)) = make_uint4(o2.x, o2.y, o3.x, o3.y);
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(&conv[stage]);
        if (++stage == S) {
          stage = 0;
          phase ^= 1u;
        }
      }
    }
  } else if (warp >= 8) {
    // ------------------------------------------------------------ epilogue
    const int ew = warp - 8;
    const int hrow = ew * 32 + lane;
    const uint32_t lane_base = (uint32_t)(ew * 32) << 16;
    uint32_t ug = 0;
    bool ok = true;
    for (int u = blockIdx.x; u < n_units && ok; u += gridDim.x, ++ug) {
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
      __nv_bfloat16* dst = pair_out + (size_t)r0 * kHidden + h * 128 + hrow;
      const float* wrow = row_weight + r0;
#pragma unroll
      for (int c = 0; c < BN / 16; ++c) {
        float p[16];
        tmem_ld16(tmem_base + lane_base + buf * BN + c * 16, p);
        tmem_wait_ld();
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const int t = c * 16 + i;
          if (t < nrows) dst[(size_t)t * kHidden] = __float2bfloat16_rn(p[i] * __ldg(wrow + t));
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty[buf]);
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
  gemm2_combine_kernel<BN><<<grid, kG2Threads, C::kBytes, stream>>>(
      *tm_w2, *tm_inter, w2_scale, reinterpret_cast<const int32_t*>(ws + L.n_blocks),
      reinterpret_cast<const int4*>(ws + L.blocks), reinterpret_cast<const float*>(ws + L.row_weight),
      reinterpret_cast<__nv_bfloat16*>(ws + L.pair_out), reinterpret_cast<uint32_t*>(ws + L.status));
  return cudaGetLastError();
}

}  // namespace

cudaError_t launch_gemm2(const CUtensorMap* tm_w2, const CUtensorMap* tm_inter, const float* w2_scale,
                         int E_local, int bn, const Layout& L, uint8_t* ws, int num_sms, cudaStream_t stream) {
  (void)E_local;
  switch (bn) {
    case 16: return launch_g2<16>(tm_w2, tm_inter, w2_scale, L, ws, num_sms, stream);
    case 32: return launch_g2<32>(tm_w2, tm_inter, w2_scale, L, ws, num_sms, stream);
    case 64: return launch_g2<64>(tm_w2, tm_inter, w2_scale, L, ws, num_sms, stream);
    case 128: return launch_g2<128>(tm_w2, tm_inter, w2_scale, L, ws, num_sms, stream);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace fbmoe
