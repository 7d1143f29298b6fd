// fbmoe_common.cuh -- shared constants and sm_100a primitives (mbarrier, TMA,
// cp.async, tcgen05/TMEM) for the fused FP8 block-scale MoE kernels.
//
// Every wait in these kernels is bounded by wall time (%globaltimer): on expiry
// the waiting thread records an error code in the caller-visible status word,
// raises a per-CTA abort flag, and the kernel unwinds (drains its own copies,
// frees TMEM) instead of hanging the GPU.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_fp8.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace fbmoe {

// DeepSeek-V3 MoE geometry (reference solution/triton/main.py:2459-2490).
constexpr int kHidden = 7168;        // H
constexpr int kInter = 2048;         // I
constexpr int kGemm1N = 2 * kInter;  // 4096 rows of W13
constexpr int kExperts = 256;        // E_global
constexpr int kTopK = 8;
constexpr int kGroups = 8;
constexpr int kGroupSize = 32;
constexpr int kTopKGroups = 4;
constexpr int kBlk = 128;                 // quantisation block
constexpr int kHBlocks = kHidden / kBlk;  // 56
constexpr int kIBlocks = kInter / kBlk;   // 16
constexpr int kRowAlign = 16;             // per-expert row segments are padded to this

// Device status word bits (ORed together).
enum StatusBits : uint32_t {
  kStatusTimeoutProducer = 1u << 0,
  kStatusTimeoutMma = 1u << 1,
  kStatusTimeoutEpilogue = 1u << 2,
  kStatusTimeoutConvert = 1u << 3,
  kStatusBadTile = 1u << 4,
  kStatusTimeoutDrain = 1u << 5,
  kStatusSaturated = 1u << 6,  // an f16 intermediate/pair value was clamped to +-65504
  kStatusTimeoutPeer = 1u << 7,  // expert parallelism: a peer's pair rows did not arrive in time
  kStatusBadSlot = 1u << 8,      // expert parallelism: a pair row's (token, slot) was not found
  kStatusDebugIndex = 1u << 9,   // debug-check build: an index read from the workspace was out of range
};

// ---------------------------------------------------------- debug checks ----
// Debug-check build (-DFBMOE_DEBUG_CHECKS, libfbmoe_debug.so): every index a
// kernel reads back from the workspace -- the token of a permuted row, the
// permuted row of a (token, slot), a GEMM block's expert and row range -- is
// range-checked before it addresses memory.  A bad value sets kStatusDebugIndex
// and is replaced by a harmless one (token 0, no row, an empty block), so the
// access it would have made is skipped or stays in bounds and the pipelines keep
// their protocol.  The checks never trap.  In the normal build they compile to
// nothing.  This is the stand-in for a memory checker on hardware where none runs.
#ifdef FBMOE_DEBUG_CHECKS
constexpr bool kDebugChecks = true;
#else
constexpr bool kDebugChecks = false;
#endif

// A token index in [0, n): otherwise 0.
__device__ __forceinline__ int dbg_token(int v, int n, uint32_t* status) {
  if (kDebugChecks && (unsigned)v >= (unsigned)n) {
    atomicOr(status, kStatusDebugIndex);
    return 0;
  }
  return v;
}
// A row index in [0, n) or -1 (none): otherwise -1.
__device__ __forceinline__ int dbg_row(int v, int n, uint32_t* status) {
  if (kDebugChecks && v != -1 && (unsigned)v >= (unsigned)n) {
    atomicOr(status, kStatusDebugIndex);
    return -1;
  }
  return v;
}
// A GEMM block (expert, first row, rows): expert in [0, e_local), rows in
// [1, max_rows], all inside [0, pcap): otherwise an empty block of expert 0.
__device__ __forceinline__ int4 dbg_block(int4 b, int max_rows, int e_local, int pcap, uint32_t* status) {
  if (kDebugChecks && ((unsigned)b.x >= (unsigned)e_local || b.y < 0 || b.z < 1 || b.z > max_rows ||
                       b.y + b.z > pcap)) {
    atomicOr(status, kStatusDebugIndex);
    return make_int4(0, 0, 0, 0);
  }
  return b;
}

constexpr float kF16Max = 65504.0f;

// fp32 -> f16 (round to nearest) with saturation; NaN stays NaN.  `sat` is set
// when a finite value had to be clamped.
__device__ __forceinline__ __half to_half_sat(float x, bool& sat) {
  if (fabsf(x) > kF16Max) {
    sat = true;
    x = copysignf(kF16Max, x);
  }
  return __float2half_rn(x);
}

// ---------------------------------------------------------------- timing ----
__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// -------------------------------------------------- programmatic dependent launch
// Kernels of the forward are launched with programmatic stream serialization:
// a kernel may start while its predecessor is still running.  pdl_wait() blocks
// the calling thread until the predecessor grid has completed and its writes are
// visible; pdl_trigger() lets the successor grid be scheduled.  The invariant the
// kernels rely on: anything a kernel reads before its own pdl_wait() was written
// by a grid at least two launches back in the stream (which has completed,
// because the predecessor itself waited for it before it could finish).  Most
// kernels trigger only after their wait; gemm2_rows_kernel triggers first (its
// successor, the reduce or the expert-parallel flag release, waits before reading).
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
// After pdl_wait, before TMA (async proxy) reads of what the predecessor wrote.
__device__ __forceinline__ void fence_proxy_async_global() {
  asm volatile("fence.proxy.async.global;" ::: "memory");
}

// ---------------------------------------------------------------- smem ------
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ---------------------------------------------------------------- mbarrier --
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.shared::cta.b64 st, [%0];\n\t}" ::"r"(smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n\t}" ::"r"(
                   smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// try_wait with a suspend-time hint: a thread whose phase is not complete sleeps
// in hardware until the phase completes or `hint_ns` passes, instead of
// re-issuing the test (spinning waiters compete with the epilogue for issue slots).
__device__ __forceinline__ bool mbar_try_wait_sleep(uint64_t* bar, uint32_t parity, uint32_t hint_ns) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity), "r"(hint_ns)
      : "memory");
  return ok != 0;
}

// Wait for the phase with the given parity to complete.  Returns false when the
// wall-time budget runs out or another role of this CTA raised the abort flag
// (checked every 16 sleeps of at most 20 us).
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, volatile int* abort_flag,
                                          uint64_t budget_ns) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  for (uint32_t it = 1;; ++it) {
    if (mbar_try_wait_sleep(bar, parity, 20000u)) return true;
    if ((it & 15u) == 0) {
      if (*abort_flag) return false;
      if (globaltimer_ns() - t0 > budget_ns) return false;
    }
  }
}

// Wait for copies this CTA issued itself (TMA loads, MMA completion) before the
// shared memory or tensor memory they target is reused or released.  Unlike
// mbar_wait it ignores the CTA abort flag: after an abort the copies already in
// flight still land within microseconds, and a CTA must not retire before they
// do.  Bounded by `budget_ns`; returns false if the budget ran out.
__device__ __forceinline__ bool mbar_wait_drain(uint64_t* bar, uint32_t parity, uint64_t budget_ns) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  for (uint32_t it = 1;; ++it) {
    if (mbar_try_wait_sleep(bar, parity, 20000u)) return true;
    if ((it & 15u) == 0 && globaltimer_ns() - t0 > budget_ns) return false;
  }
}

// At the end of a forward's last kernel: if the status word is non-zero, copy it
// to the caller's host-visible sink (pinned host memory registered with
// fbmoe_set_status_sink), so the host learns of a device-side error without a
// synchronising read.  Racing CTAs may store different non-zero words; any of
// them marks the call as failed.
__device__ __forceinline__ void forward_status_to_sink(uint32_t* status, uint32_t* sink) {
  if (sink == nullptr) return;
  // A relaxed gpu-scope load reads the word at L2: it sees this CTA's own earlier
  // atomicOr (ordered by the caller's CTA barrier) and whatever other CTAs have
  // made visible; each CTA that sets a bit also forwards it at its own end.  (An
  // atomicOr(status, 0) from every CTA would serialise at one L2 address.)
  uint32_t s;
  asm volatile("ld.relaxed.gpu.global.b32 %0, [%1];" : "=r"(s) : "l"(status) : "memory");
  if (s != 0u) {
    *reinterpret_cast<volatile uint32_t*>(sink) = s;
    __threadfence_system();
  }
}

// ---------------------------------------------------------------- fences ----
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void named_barrier_sync(uint32_t id, uint32_t nthreads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

// Named barrier that also ORs a flag over the participating threads, so that a
// group of warps takes the same branch after a failed (timed-out) wait.
__device__ __forceinline__ bool named_barrier_or(uint32_t id, uint32_t nthreads, bool flag) {
  uint32_t out;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\tsetp.ne.u32 p, %1, 0;\n\t"
      "bar.red.or.pred q, %2, %3, p;\n\tselp.u32 %0, 1, 0, q;\n\t}"
      : "=r"(out)
      : "r"((uint32_t)flag), "r"(id), "r"(nthreads)
      : "memory");
  return out != 0;
}

// ---------------------------------------------------------------- TMA -------
__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// 2-D tiled bulk tensor load global -> this CTA's shared memory, completion on an mbarrier.
// x = innermost coordinate (elements), y = row.  x * elem_size must be a multiple of 16.
__device__ __forceinline__ void tma_load_2d(void* smem_dst, const CUtensorMap* map, uint64_t* bar, int32_t x,
                                            int32_t y, uint64_t cache_hint) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%3, %4}], [%2], %5;" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y), "l"(cache_hint)
      : "memory");
}

// Same, without an L2 cache hint.
__device__ __forceinline__ void tma_load_2d_nohint(void* smem_dst, const CUtensorMap* map, uint64_t* bar, int32_t x,
                                                   int32_t y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y)
      : "memory");
}

// Prefetch one tile of a tensor map into L2 (no shared-memory destination and no
// completion to wait for).  x * element size must be a multiple of 16 bytes.
__device__ __forceinline__ void tma_prefetch_l2_2d(const CUtensorMap* map, int32_t x, int32_t y) {
  asm volatile("cp.async.bulk.prefetch.tensor.2d.L2.global.tile [%0, {%1, %2}];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(x), "r"(y)
               : "memory");
}

// L2 eviction policies (createpolicy).
// 1-D bulk copy global -> shared (both 16-byte aligned, bytes a multiple of 16),
// completing as transaction bytes on `bar`.
__device__ __forceinline__ void bulk_load_1d(void* smem_dst, const void* gsrc, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(smem_dst)),
      "l"(gsrc), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ uint64_t l2_policy_evict_first() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}
__device__ __forceinline__ uint64_t l2_policy_evict_last() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
  return p;
}

// ---------------------------------------------------------------- cp.async --
// 16-byte copy; src_bytes = 0 writes zeros (used for padding columns).
__device__ __forceinline__ void cp_async_16(uint32_t smem_dst, const void* gsrc, uint32_t src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_dst), "l"(gsrc), "r"(src_bytes)
               : "memory");
}
__device__ __forceinline__ void cp_async_4(uint32_t smem_dst, const void* gsrc, uint32_t src_bytes) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;" ::"r"(smem_dst), "l"(gsrc), "r"(src_bytes)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait_group() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }

// ---------------------------------------------------------------- tcgen05 ---
// TMEM allocation (whole warp).  The allocated base address is written to smem.
__device__ __forceinline__ void tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// Arrive on an mbarrier once all previously issued tcgen05.mma of this thread complete.
__device__ __forceinline__ void tc_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

// D[tmem] (+)= A[smem] * B[smem]^T, FP8 (E4M3 x E4M3) with fp32 accumulation.
__device__ __forceinline__ void mma_f8f6f4(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                           uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// D[tmem] (+)= A[smem] * B[smem]^T, BF16 x BF16 with fp32 accumulation.
__device__ __forceinline__ void mma_f16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                        uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Warp-collective TMEM load: 32 lanes x 16 consecutive fp32 columns.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float (&v)[16]) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}
// The same load, returned as 8 packed pairs of fp32 for the f32x2 FMA below.
__device__ __forceinline__ void tmem_ld16_pairs(uint32_t taddr, uint64_t (&v)[8]) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
#pragma unroll
  for (int i = 0; i < 8; ++i) asm("mov.b64 %0, {%1, %2};" : "=l"(v[i]) : "r"(r[2 * i]), "r"(r[2 * i + 1]));
}

// W2 dequantisation to f16 (both GEMM2 kernels).  Per 128-row block of W2 the
// kernels pick a power of two 2^k with max_k s2 * 2^k in [32, 64); each element
// becomes f16(fp8) * f16(s2 * 2^k) in one HMUL2 (the fp8 value is exact in f16,
// the product stays below 448 * 64) and the epilogue multiplies by 2^-k exactly.
// This returns k for the 16 scales of one block.
__device__ __forceinline__ int w2_block_exponent(const float* s16) {
  float m = 0.0f;
#pragma unroll
  for (int i = 0; i < kIBlocks; ++i) m = fmaxf(m, fabsf(__ldg(s16 + i)));
  if (!(m > 0.0f) || !isfinite(m)) return 0;
  int ex;
  frexpf(m, &ex);  // m = f * 2^ex, f in [0.5, 1)
  int k = 6 - ex;  // m * 2^k in [32, 64)
  return k < -60 ? -60 : (k > 60 ? 60 : k);
}

// ---------------------------------------------------- packed fp32 (f32x2) ----
// sm_100 executes two IEEE fp32 FMAs (round-to-nearest, the same result as two
// fmaf calls) per fma.rn.f32x2 instruction; the promotion epilogues use it to
// halve their instruction count.
__device__ __forceinline__ uint64_t f32x2_pack(float lo, float hi) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}
__device__ __forceinline__ void f32x2_unpack(uint64_t v, float& lo, float& hi) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
}
__device__ __forceinline__ void f32x2_fma(uint64_t& acc, uint64_t x, uint64_t y) {
  asm("fma.rn.f32x2 %0, %1, %2, %0;" : "+l"(acc) : "l"(x), "l"(y));
}
__device__ __forceinline__ uint64_t f32x2_mul(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}

// ----------------------------------------------- prefill GEMM2 mode ----
// Prefill GEMM2 runs as one of two kernels chosen on the device from the routing:
// both are launched, one after the other, and the one not chosen only waits for
// its grid dependency and returns.  Experts' 128-row blocks are worked in pairs
// (moe_gemm2_pairs.cu) when the blocks number at least 2 per active expert
// (measured: 13-15 % faster GEMM2 under skewed routing, 3.5 % faster per call at
// config 3's 2.96 blocks per expert); with about one block per expert, units stay
// single and one block per unit keeps the accumulators double-buffered
// (moe_gemm2_rows.cu).  A block list the permutation cut short
// goes to the one-block kernel.  Run by threads 0..255 of the CTA (named barrier
// 1); every one of them gets the same answer.  red: 16 ints of shared memory.
__device__ __forceinline__ bool gemm2_pairs_mode(const int32_t* __restrict__ expert_cnt, int e_local, int nb_all,
                                                 int* red) {
  const int e = threadIdx.x, lane = e & 31, warp = e >> 5;
  const int c = e < e_local ? expert_cnt[e] : 0;
  const int nb = __reduce_add_sync(0xffffffffu, (c + 127) / 128);
  const int act = __reduce_add_sync(0xffffffffu, c > 0 ? 1 : 0);
  if (lane == 0) {
    red[warp] = nb;
    red[8 + warp] = act;
  }
  named_barrier_sync(1, 256);
  int tot_nb = 0, tot_act = 0;
#pragma unroll
  for (int w = 0; w < 8; ++w) {
    tot_nb += red[w];
    tot_act += red[8 + w];
  }
  return tot_nb == nb_all && tot_act > 0 && tot_nb >= 2 * tot_act;
}

// ------------------------------------------- 1x128 e4m3 quantisation -------
// e4m3(RN(a / s)) and e4m3(RN(b / s)), saturating, packed with a in the low
// byte -- bit-identical to converting the IEEE quotients -- given the block's
// E4m3Scale.  y0 = RN(x * r), r = RN(1 / s), lies within 3 fp32 ulps of
// RN(x / s); the conversion is monotonic, so when y0 - 4 ulps and y0 + 4 ulps
// convert to the same e4m3 value, so does RN(x / s).  Otherwise (an e4m3
// rounding midpoint or zero within reach, NaN) the pair is divided exactly.  On
// bf16 data about 0.5 % of the elements land that close to a midpoint (a short
// ratio x / amax lands on one exactly).
struct E4m3Scale {
  float s;    // amax / 448 (1 for an all-zero block), the stored scale
  float r;    // RN(1 / s)
  bool fast;  // r is a finite normal number
};
__device__ __forceinline__ uint32_t e4m3x2_of(float a, float b) {
  return (uint32_t)__nv_cvt_float2_to_fp8x2(make_float2(a, b), __NV_SATFINITE, __NV_E4M3);
}
__device__ __forceinline__ uint32_t e4m3x2_quotient(float a, float b, const E4m3Scale& q) {
  float ya, yb;
  f32x2_unpack(f32x2_mul(f32x2_pack(a, b), f32x2_pack(q.r, q.r)), ya, yb);
  const uint32_t ua = __float_as_uint(ya), ub = __float_as_uint(yb);
  const uint32_t lower = e4m3x2_of(__uint_as_float(ua - 4u), __uint_as_float(ub - 4u));
  const uint32_t upper = e4m3x2_of(__uint_as_float(ua + 4u), __uint_as_float(ub + 4u));
  if (lower == upper && q.fast) return lower;
  return e4m3x2_of(__fdiv_rn(a, q.s), __fdiv_rn(b, q.s));
}
// The 1x128 rule's scale for a block with the given amax.
__device__ __forceinline__ E4m3Scale e4m3_block_scale(float amax) {
  E4m3Scale q;
  q.s = amax > 0.0f ? __fdiv_rn(amax, 448.0f) : 1.0f;
  q.r = __frcp_rn(q.s);
  q.fast = q.s >= 1.0e-36f && q.s <= 1.0e36f;
  return q;
}

// Warp-collective TMEM load: 32 lanes x 4 consecutive fp32 columns.
__device__ __forceinline__ void tmem_ld4(uint32_t taddr, float (&v)[4]) {
  uint32_t r[4];
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x4.b32 {%0, %1, %2, %3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(taddr));
#pragma unroll
  for (int i = 0; i < 4; ++i) v[i] = __uint_as_float(r[i]);
}

// Warp-collective TMEM load of 32 consecutive fp32 columns as 16 packed pairs.
__device__ __forceinline__ void tmem_ld32_pairs(uint32_t taddr, uint64_t (&v)[16]) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
#pragma unroll
  for (int i = 0; i < 16; ++i) asm("mov.b64 %0, {%1, %2};" : "=l"(v[i]) : "r"(r[2 * i]), "r"(r[2 * i + 1]));
}

// Warp-collective TMEM load: 32 lanes x 32 consecutive fp32 columns.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&v)[32]) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}
// Warp-collective TMEM store: 32 lanes x 32 consecutive 32-bit columns.
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&v)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16, "
      "%17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};" ::"r"(taddr),
      "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]), "r"(v[9]),
      "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15]), "r"(v[16]), "r"(v[17]), "r"(v[18]),
      "r"(v[19]), "r"(v[20]), "r"(v[21]), "r"(v[22]), "r"(v[23]), "r"(v[24]), "r"(v[25]), "r"(v[26]), "r"(v[27]),
      "r"(v[28]), "r"(v[29]), "r"(v[30]), "r"(v[31])
      : "memory");
}
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// f16 x f16 -> fp32 MMA with the A operand (M rows = TMEM lanes, K packed two
// per 32-bit column) in tensor memory and B in shared memory.
__device__ __forceinline__ void mma_f16_tmem_a(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                               uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// UMMA shared-memory matrix descriptor, K-major operand with 128-byte swizzle:
// rows of 128 bytes, 8-row (1024-byte) swizzle atoms stacked along M/N.
__device__ __forceinline__ uint64_t umma_desc_sw128(uint32_t smem_addr) {
  uint64_t d = 0;
  d |= (uint64_t)((smem_addr >> 4) & 0x3FFFu);    // start address
  d |= (uint64_t)(1u) << 16;                      // leading byte offset (unused for swizzled K-major)
  d |= (uint64_t)((1024u >> 4) & 0x3FFFu) << 32;  // stride byte offset: next 8-row atom
  d |= (uint64_t)1u << 46;                        // descriptor version (sm_100)
  d |= (uint64_t)2u << 61;                        // layout: SWIZZLE_128B
  return d;
}

// Instruction descriptor: fp32 accumulate, K-major A and B, shape M x N.
// a_b_format: 0 = E4M3 (kind::f8f6f4) or F16 (kind::f16); 1 = BF16 (kind::f16).
__host__ __device__ constexpr uint32_t umma_idesc(uint32_t a_b_format, int M, int N) {
  return (1u << 4)                          // D format F32
         | (a_b_format << 7)                // A format
         | (a_b_format << 10)               // B format
         | ((uint32_t)(N >> 3) << 17)       // N
         | ((uint32_t)(M >> 4) << 24);      // M
}

// Offset (bytes) of the 16-byte chunk `c` of row `r` in a 128B-swizzled K-major tile.
__host__ __device__ __forceinline__ uint32_t sw128_offset(uint32_t r, uint32_t c) {
  return r * 128u + ((c ^ (r & 7u)) << 4);
}

}  // namespace fbmoe
