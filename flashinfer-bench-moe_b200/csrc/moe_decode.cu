// moe_decode.cu -- the expert computation of a decode-sized call (16-row
// blocks, T <= 64) as ONE persistent kernel: GEMM1 + SwiGLU, GEMM2 x routing
// weight and the per-token combine (tcgen05 + TMEM + TMA), sm_100a.
//
// Reference counterparts: gemm1_kernel + act_quant_kernel (solution/triton/
// main.py:41-223, 1426-1602), gemm2_kernel (main.py:433-600) and
// reduce_add_kernel (main.py:1604-1714).  Per local expert e, permuted row r
// (token t) and hidden column h:
//     G1[r, n]    = sum_k A[t, k] * a_scale[k/128, t] * W1[e, n, k] * s1[e, n/128, k/128]
//     inter[r, j] = silu(G1[r, 2048 + j]) * G1[r, j]
//     pair[r, h]  = w[r] * sum_j inter[r, j] * W2[e, h, j] * s2[e, h/128, j/128]   (f16)
//     out[t, h]   = sum over t's local slots of pair[r, h]            (fp32 sum, bf16)
// The intermediate is stored as two fp8 planes per row and 64-column chunk: q0 =
// e4m3(y * 448 / amax) with scale amax / 448, then the same for the residual
// y - q0 * s0 (not the reference's single re-quantisation, which puts about 10%
// of output elements outside atol 1e-2 / rtol 2e-2; two planes stay within
// ~0.12x of the tolerance in host emulation).  A non-finite SwiGLU output sets
// kStatusSaturated.
//
// Why one kernel.  At decode sizes the call streams the active experts' weights
// (44 MB each) and little else; separate GEMM1 / GEMM2 / combine launches cost a
// grid drain, a launch and a prologue each, and GEMM2 could not start streaming
// W2 before the last GEMM1 CTA retired.  Here every CTA runs its GEMM1 work items,
// then its GEMM2 items: W2 tiles stream in at once, and only the intermediate
// rows of a block wait for that block's 32 GEMM1 slices (a per-block counter
// that GEMM1 raises after publishing them).  The combine runs after one grid-wide
// arrival (every CTA has written its pair rows) and is spread over all threads.
// The grid is at most one CTA per SM with one CTA resident per SM, nothing in
// GEMM1 waits on GEMM2 and every CTA reaches the grid arrival, so every wait
// ends; every wait is also bounded in wall time.
//
// Orientation (swap-AB) in both GEMMs: weight rows are the MMA's M = 128 operand
// and the <= 16 token rows of a block its N operand.
//
// GEMM1 phase.  Work unit = (block of 16 rows of one expert) x (slice g of 64
// output columns); the A tile stacks W1 rows [64g, 64g+64) (h1 half) on rows
// [2048+64g, 2048+64g+64) (silu half); the B tile gathers the block's token rows
// with cp.async (no permuted copy of the activations).  Every 128-K block is
// MMA'd into its own TMEM buffer and promoted by s1 * a_scale into fp32
// registers (the per-128-K block scales are applied exactly).  Four sets of four
// epilogue warps take the K-blocks kb = j (mod 4), so four K-blocks are in flight
// in the epilogue; their partial sums are added in set order.  Work is balanced
// "stream-K" style: the phase's K-blocks, flattened unit-major, are cut into one
// contiguous range per CTA (see Partition); a unit cut by range boundaries is
// computed in segments whose fp32 partials the segment that arrives last adds in
// segment order (deterministic).
// Warps: w0 producer (TMA + cp.async), w1 MMA issuer, w2-w3 idle, w4-w19 epilogue.
//
// GEMM2 phase.  Work unit = (block) x (slice h of 128 hidden columns): A = 128
// raw fp8 W2 rows (TMA ring), exact; B = the block's two intermediate planes
// (2 x 16 rows, fp8, the block's rows copied with cp.async), resident in shared
// memory for the CTA's units of that block.  Per K-block one kind::f8f6f4 MMA per 64-K chunk (N = 32: both planes)
// into one of 8 TMEM slots, one commit per K-block; promotion warps add
// D * s2 * plane_scale in fp32 registers per chunk and plane.  Stream-K as in
// GEMM1, with ranges of >= 16 K-blocks, so a unit has at most two segments;
// segment s writes plane s of the pair rows and the combine adds a unit's planes.
// Warps: w0 W2 producer (TMA), w1 MMA issuer, w2 planes producer (waits for the
// block's GEMM1 slices, then cp.async), w3 idle, w4-w19 promotion; then all
// threads combine.
#include <cstdlib>

#include "fbmoe_common.cuh"
#include "fbmoe_launch.h"

namespace fbmoe {
namespace {

constexpr int BN = 16;                      // rows per block
constexpr int kThreads = 640;               // 20 warps
constexpr uint64_t kWaitBudgetNs = 4000000000ull;
constexpr int kG1Slices = kInter / 64;      // 32 slices of 64 intermediate columns
constexpr int kG2Slices = kHidden / 128;    // 56 slices of 128 hidden columns

// ---- GEMM1 phase layout (offsets inside the shared region)
constexpr int kSets = 4;                    // epilogue warp sets
constexpr int kEpi1Threads = 128 * kSets;
// TMEM partial buffers: all 512 columns, so the MMA can run up to 32 K-blocks
// (two split-K items) ahead of the promotion epilogue, whose per-item fix-up
// (partials to L2, fence, counter) would otherwise stall the weight stream.
constexpr int kBufs1 = 32;
// 10 stages = 160 KB of W1 in flight per SM: HBM streaming at ~2 us loaded latency
// needs roughly 90 KB per SM, and more absorbs the latency spread.
constexpr int kStages1 = 10;
// A stage's cp.async row copies are signalled complete kLag stages after they
// are issued, so up to kLag stages of row copies are in flight.
constexpr int kLag = kStages1 - 2;
constexpr int kA1Bytes = 128 * 128;
constexpr int kB1Bytes = BN * 128;
constexpr int kXchStride = BN + 1;
constexpr int kP1A = 0;
constexpr int kP1B = kP1A + kStages1 * kA1Bytes;
constexpr int kP1AScale = kP1B + kStages1 * kB1Bytes;
constexpr int kP1WScale = kP1AScale + kHBlocks * BN * 4;
constexpr int kP1Xch = kP1WScale + 2 * kHBlocks * 4;
constexpr int kP1Tok = kP1Xch + kSets * 128 * kXchStride * 4;
constexpr int kP1End = kP1Tok + BN * 4;
// ---- GEMM2 phase layout
// A = the W2 tile (fp8, 128 rows x 128 K) from a TMA ring; B = the block's
// intermediate as two fp8 planes (see gemm2_phase), resident in shared memory
// for all of the CTA's units of that block: per K-block 32 rows (plane 0 then
// plane 1, 16 token rows each) x 128 bytes, 128-byte swizzle, plus the planes'
// fp32 scales.  Tensor memory: 16 accumulator buffers of 32 columns.
constexpr int kRawStages = 9;
constexpr int kRawBytes = 128 * 128;        // fp8 W2 tile
constexpr int kPlaneRows = 2 * BN;          // two planes of BN token rows
constexpr int kPlaneKBytes = kPlaneRows * 128;
// K-block slots of tensor memory: a W2 tile's two 64-K chunks accumulate into the
// slot's two 32-column halves, signalled by one commit per K-block (tcgen05.commit
// is the expensive part of issuing at these sizes; the raw W2 stage is released by
// the promotion warps once the slot's commit shows its MMAs done).
constexpr int kSlots2 = 8;
// Every promotion warp waits on every buffer use in order, so each parity wait is
// for the phase right after the one the same waiter last saw (a parity wait cannot
// alias a phase two completions ahead).
constexpr int kCols2 = kPlaneRows;          // accumulator columns per chunk (a slot holds two chunks)
constexpr int kChunks = kInter / 64;         // 64-column chunks of the intermediate (plane scale blocks)
constexpr int kP2Raw = 0;
constexpr int kP2Planes = kP2Raw + kRawStages * kRawBytes;
constexpr int kP2PScale = kP2Planes + kIBlocks * kPlaneKBytes;
constexpr int kP2End = kP2PScale + 2 * BN * kChunks * 4;
constexpr int kRegion = ((kP1End > kP2End ? kP1End : kP2End) + 1023) / 1024 * 1024;
// ---- barriers and flags (not reused across phases)
constexpr int kNumBars1 = 2 * kStages1 + 2 * kBufs1 + 1;
constexpr int kNumBars2 = 2 * kRawStages + 2 + 2 * kSlots2 + 1;
constexpr int kOffBar = kRegion;
constexpr int kOffMisc = kOffBar + (kNumBars1 + kNumBars2) * 8;
constexpr int kSmemBytes = kOffMisc + 32 + 1024;  // + alignment slack
constexpr int kTmemCols = 512;                    // one CTA per SM holds all of TMEM
static_assert(kSmemBytes <= 227 * 1024, "decode kernel shared memory over the per-CTA limit");
static_assert(kHBlocks % kSets == 0, "K-blocks must split evenly over the epilogue sets");
static_assert(kBufs1 % kSets == 0, "a buffer belongs to one epilogue set");
static_assert(kBufs1 * BN <= kTmemCols && kSlots2 * 2 * kCols2 <= kTmemCols, "TMEM allocation");
static_assert(kP2Planes % 1024 == 0, "the planes are 128-byte swizzle atoms");

struct DecodeArgs {
  CUtensorMap tm_w1;     // W1 rows x 7168 K, 128-byte x 64-row boxes
  CUtensorMap tm_w2;     // W2 rows x 2048 K, 128-byte x 128-row boxes
  const uint8_t* hidden;
  const float* hidden_scale;
  const float* w1_scale;
  const float* w2_scale;
  const int32_t* n_blocks;
  const int4* blocks;
  const int32_t* row_token;
  const float* row_weight;
  const int32_t* token_rows;
  int streamk;           // 1: K-block-granular partition with split-K fix-ups; 0: whole units
  int32_t* split_count;
  float* split_part;
  int32_t* blk_ready;
  int32_t* grid_sync;
  uint8_t* planes;         // [2][pcap][2048] fp8: the intermediate as two planes (GEMM1 -> GEMM2)
  float* plane_scale;      // [2][32][pcap] fp32: their per-(64-column chunk, row) scales
  __half* pair_out;
  void* out;
  uint32_t* status;
  uint32_t* sink;          // host-visible copy of a non-zero status word (nullptr: none)
  size_t plane_elems;
  int T;
  int pcap;                // row capacity of the workspace (bounds of the debug checks)
  int e_local;
  int w1_packed;           // W1 in the fbmoe_prepack_w1 layout (tm_w1 then has 128-row boxes)
  int f32_out;
  int grid_extra;          // arrivals the combine waits for beyond gridDim.x (0; 1 only under the test hook)
  uint64_t grid_wait_ns;   // budget of the grid arrival wait
};

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

__device__ __forceinline__ int ld_relaxed_gpu(const int32_t* p) {
  int v;
  asm volatile("ld.relaxed.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void fence_acq_rel_gpu() { asm volatile("fence.acq_rel.gpu;" ::: "memory"); }
__device__ __forceinline__ int atom_add_acq_rel_gpu(int32_t* p, int v) {
  int old;
  asm volatile("atom.acq_rel.gpu.global.add.s32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(v) : "memory");
  return old;
}
__device__ __forceinline__ void red_release_gpu_add(int32_t* p, int v) {
  asm volatile("red.release.gpu.global.add.s32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Wait until *p >= target (a counter raised by release-adds of other CTAs), then
// acquire: relaxed polling (no sleep: the counter is one L2 line and one thread per
// CTA polls it) and one acquire fence once the target is seen.  Returns false when
// `abort` is raised or the wall-time budget runs out.
__device__ __forceinline__ bool wait_counter(const int32_t* p, int target, volatile int* abort, uint64_t budget_ns) {
  const uint64_t t0 = globaltimer_ns();
  for (uint32_t it = 1; ld_relaxed_gpu(p) < target; ++it) {
    if ((it & 31u) == 0 && (*abort || globaltimer_ns() - t0 > budget_ns)) return false;
  }
  fence_acq_rel_gpu();
  return true;
}

// Balanced partition of one phase's K-blocks over the CTAs that take part
// ("stream-K"): the phase's units are flattened unit-major (unit u holds K-blocks
// [u*len, u*len + len)) and CTA c owns the range [begin(c), begin(c+1)).  A unit
// cut by range boundaries is computed in segments on different CTAs and fixed up
// in segment order (deterministic).  With unit_aligned the boundaries fall on
// unit boundaries, so no unit is cut (used when no split-K buffers exist).
struct Partition {
  int total;         // units * len
  int len;           // K-blocks per unit
  int g;             // CTAs that take part
  bool unit_aligned;
  __device__ int begin(int c) const {
    if (c >= g) return total;
    if (unit_aligned) return (int)(((long long)c * (total / len)) / g) * len;
    return (int)(((long long)c * total) / g);
  }
  // the CTA whose range holds K-block x
  __device__ int owner(int x) const {
    if (unit_aligned) {
      const long long nu = total / len;
      return (int)((((long long)(x / len) + 1) * g + nu - 1) / nu) - 1;
    }
    return (int)((((long long)x + 1) * g + total - 1) / total) - 1;
  }
  __device__ int first_owner(int u) const { return owner(u * len); }
  __device__ int nseg(int u) const { return owner(u * len + len - 1) - owner(u * len) + 1; }
};

// The segment of unit x / len that starts at K-block x and ends before `end`.
struct Seg {
  int u, kb0, kb1;
};
__device__ __forceinline__ Seg seg_at(const Partition& P, int x, int end) {
  Seg sg;
  sg.u = x / P.len;
  sg.kb0 = x % P.len;
  sg.kb1 = min(P.len, sg.kb0 + (end - x));
  return sg;
}

// Phase partitions.  Stream-K: GEMM1 ranges hold >= 8 K-blocks (a unit has up to 8
// segments; a CTA writes at most 2 partials: its first and its last unit); GEMM2
// ranges hold >= 16 K-blocks = one unit, so a unit has at most 2 segments = planes.
constexpr int kSegBatch = 4;  // fix-up: segment partials loaded per L2 round trip
__device__ __forceinline__ Partition gemm1_partition(int nb, bool streamk) {
  const int units = nb * kG1Slices, total = units * kHBlocks;
  const int g = streamk ? max(1, min((int)gridDim.x, total / 8)) : max(1, min((int)gridDim.x, units));
  return Partition{total, kHBlocks, g, !streamk};
}
__device__ __forceinline__ Partition gemm2_partition(int nb, bool streamk) {
  const int units = nb * kG2Slices, total = units * kIBlocks;
  const int g = streamk ? max(1, min((int)gridDim.x, total / kIBlocks)) : max(1, min((int)gridDim.x, units));
  return Partition{total, kIBlocks, g, !streamk};
}
// fp32 partial slot of CTA c's segment of unit u: 2c for its first unit, 2c + 1 for its last.
__device__ __forceinline__ int partial_slot(const Partition& P, int c, int u) {
  return 2 * c + (u == P.begin(c) / P.len ? 0 : 1);
}

// ============================================================== GEMM1 phase
__device__ __forceinline__ void gemm1_phase(const DecodeArgs& a, uint8_t* sm, uint64_t* bars, uint32_t tmem_base,
                                            int nb, volatile int* sAbort, volatile int* sLast) {
  constexpr int S = kStages1;
  uint8_t* sA = sm + kP1A;
  uint8_t* sB = sm + kP1B;
  float* sAScale = reinterpret_cast<float*>(sm + kP1AScale);  // [56][BN]
  float* sWScale = reinterpret_cast<float*>(sm + kP1WScale);  // [2][56]
  float* sXch = reinterpret_cast<float*>(sm + kP1Xch);        // [sets][128][BN+1] partial sums
  int* sTok = reinterpret_cast<int*>(sm + kP1Tok);            // [BN]
  uint64_t* full = bars;
  uint64_t* empty = bars + S;
  uint64_t* tfull = bars + 2 * S;
  uint64_t* tempty = tfull + kBufs1;
  uint64_t* drain = tempty + kBufs1;
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const Partition P = gemm1_partition(nb, a.streamk != 0);
  const int x_beg = P.begin(blockIdx.x), x_end = P.begin(blockIdx.x + 1);
  auto fail = [&](uint32_t bit) {
    *sAbort = 1;
    atomicOr(a.status, bit);
  };

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    const uint64_t pol_w = l2_policy_evict_first();  // each weight tile is read about once
    int stage = 0;
    uint32_t phase = 0;
    long issued = 0;
    bool ok = true;
    uint32_t last_parity[S];
#pragma unroll
    for (int s = 0; s < S; ++s) last_parity[s] = 0xFFFFFFFFu;
    for (int x = x_beg; x < x_end && ok;) {
      const Seg sg = seg_at(P, x, x_end);
      x += sg.kb1 - sg.kb0;
      const int u = sg.u;
      const int4 blk = dbg_block(a.blocks[u / kG1Slices], BN, a.e_local, a.pcap, a.status);
      const int g = u % kG1Slices;
      const int e = blk.x, r0 = blk.y, nrows = blk.z;
      // token row pointers for the rows this lane copies: rows (lane>>3) + 4j
      constexpr int kRowsPerLane = BN / 4;
      const uint8_t* src[kRowsPerLane];
#pragma unroll
      for (int j = 0; j < kRowsPerLane; ++j) {
        const int row = (lane >> 3) + 4 * j;
        src[j] = (row < nrows) ? a.hidden + (size_t)dbg_token(a.row_token[r0 + row], a.T, a.status) * kHidden +
                                     (lane & 7) * 16
                               : a.hidden;
      }
      const int wrow1 = e * kGemm1N + 64 * g;
      const int wrow2 = wrow1 + kInter;
      for (int kb = sg.kb0; kb < sg.kb1; ++kb) {
        if (!mbar_wait(&empty[stage], phase ^ 1u, sAbort, kWaitBudgetNs)) {
          ok = false;
          if (lane == 0) fail(kStatusTimeoutProducer);
          break;
        }
        if (lane == 0) {
          mbar_arrive_expect_tx(&full[stage], kA1Bytes);
          if (a.w1_packed) {
            // packed rows [128g, 128g + 128) = this slice of both halves, one box
            tma_load_2d(sA + stage * kA1Bytes, &a.tm_w1, &full[stage], kb * kBlk, e * kGemm1N + 128 * g, pol_w);
          } else {
            tma_load_2d(sA + stage * kA1Bytes, &a.tm_w1, &full[stage], kb * kBlk, wrow1, pol_w);
            tma_load_2d(sA + stage * kA1Bytes + 64 * 128, &a.tm_w1, &full[stage], kb * kBlk, wrow2, pol_w);
          }
        }
        last_parity[stage] = phase;
        const uint32_t bdst = smem_u32(sB + stage * kB1Bytes);
#pragma unroll
        for (int j = 0; j < kRowsPerLane; ++j) {
          const int row = (lane >> 3) + 4 * j;
          cp_async_16(bdst + sw128_offset(row, lane & 7), src[j] + kb * kBlk, row < nrows ? 16u : 0u);
        }
        cp_async_commit();
        ++issued;
        if (issued > kLag) {
          cp_async_wait_group<kLag>();
          fence_proxy_async_smem();
          __syncwarp();
          int ps = stage - kLag;
          if (ps < 0) ps += S;
          if (lane == 0) mbar_arrive(&full[ps]);
        }
        if (++stage == S) {
          stage = 0;
          phase ^= 1u;
        }
      }
    }
    // complete the last kLag stages (or fewer)
    cp_async_wait_all();
    fence_proxy_async_smem();
    __syncwarp();
    if (lane == 0) {
      const long tail = issued < kLag ? issued : kLag;
      for (long i = tail; i >= 1; --i) {
        int ps = stage - (int)i;
        while (ps < 0) ps += S;
        mbar_arrive(&full[ps]);
      }
      // drain: every issued TMA load must have landed before the smem is reused
      for (int s = 0; s < S; ++s)
        if (last_parity[s] != 0xFFFFFFFFu)
          if (!mbar_wait_drain(&full[s], last_parity[s], kWaitBudgetNs)) fail(kStatusTimeoutDrain);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = umma_idesc(0u, 128, BN);
      int stage = 0;
      uint32_t phase = 0;
      uint32_t kbg = 0;
      bool ok = true;
      bool any = false;
      for (int x = x_beg; x < x_end && ok;) {
        const Seg sg = seg_at(P, x, x_end);
        x += sg.kb1 - sg.kb0;
        for (int l = 0; l < sg.kb1 - sg.kb0; ++l) {
          const uint32_t buf = kbg % kBufs1;
          if (!mbar_wait(&tempty[buf], ((kbg / kBufs1) & 1u) ^ 1u, sAbort, kWaitBudgetNs) ||
              !mbar_wait(&full[stage], phase, sAbort, kWaitBudgetNs)) {
            ok = false;
            fail(kStatusTimeoutMma);
            break;
          }
          tc_fence_after();
          const uint64_t adesc = umma_desc_sw128(smem_u32(sA + stage * kA1Bytes));
          const uint64_t bdesc = umma_desc_sw128(smem_u32(sB + stage * kB1Bytes));
          const uint32_t d = tmem_base + buf * BN;
#pragma unroll
          for (int j = 0; j < 4; ++j) mma_f8f6f4(d, adesc + 2 * j, bdesc + 2 * j, idesc, j > 0 ? 1u : 0u);
          tc_commit(&empty[stage]);
          tc_commit(&tfull[buf]);
          any = true;
          ++kbg;
          if (++stage == S) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      if (any) {
        // all issued MMAs complete before TMEM and shared memory are reused
        tc_commit(drain);
        mbar_wait_drain(drain, 0, kWaitBudgetNs);
      }
    }
    __syncwarp();
  } else if (warp >= 4) {
    // ------------------------------------------------------------ epilogue
    constexpr int G = kSets;
    const int set = (warp - 4) >> 2;   // this warp's K-block residue class
    const int ew = warp & 3;           // TMEM lane quarter
    const int row = ew * 32 + lane;    // A row == TMEM lane
    const int etid = threadIdx.x - 128;
    const uint32_t lane_base = (uint32_t)(ew * 32) << 16;
    uint32_t kbg = 0;                  // K-blocks this CTA processed before the current item
    bool ok = true;
    for (int x = x_beg; x < x_end && ok;) {
      const Seg sg = seg_at(P, x, x_end);
      x += sg.kb1 - sg.kb0;
      const int u = sg.u, nk = sg.kb1 - sg.kb0;
      const int nseg = P.nseg(u);
      const int4 blk = dbg_block(a.blocks[u / kG1Slices], BN, a.e_local, a.pcap, a.status);
      const int g = u % kG1Slices;
      const int e = blk.x, r0 = blk.y, nrows = blk.z;
      if (etid < BN) sTok[etid] = (etid < nrows) ? dbg_token(a.row_token[r0 + etid], a.T, a.status) : -1;
      if (etid < 2 * kHBlocks) {
        const int h = etid / kHBlocks, kb = etid % kHBlocks;
        const int nbk = h * (kInter / kBlk) + g / 2;
        sWScale[etid] = a.w1_scale[((size_t)e * (kGemm1N / kBlk) + nbk) * kHBlocks + kb];
      }
      named_barrier_sync(1, kEpi1Threads);
      for (int i = etid; i < kHBlocks * BN; i += kEpi1Threads) {
        const int kb = i / BN, t = i % BN;
        const int tok = sTok[t];
        sAScale[i] = tok >= 0 ? a.hidden_scale[(size_t)kb * a.T + tok] : 0.0f;
      }
      named_barrier_sync(1, kEpi1Threads);

      float acc[BN];
#pragma unroll
      for (int t = 0; t < BN; ++t) acc[t] = 0.0f;
      const float* wsc = sWScale + (ew < 2 ? 0 : kHBlocks);
      bool bad = false;
      // this set takes the item's K-blocks whose CTA-wide index is = set (mod G)
      for (int l = (set - (int)(kbg % G) + G) % G; l < nk; l += G) {
        const uint32_t kgl = kbg + l;
        const uint32_t buf = kgl % kBufs1;
        if (!mbar_wait(&tfull[buf], (kgl / kBufs1) & 1u, sAbort, kWaitBudgetNs)) {
          bad = true;
          if (lane == 0) fail(kStatusTimeoutEpilogue);
          break;
        }
        tc_fence_after();
        const int kb = sg.kb0 + l;
        const float ws = wsc[kb];
        const float* asc = sAScale + kb * BN;
        float p[16];
        tmem_ld16(tmem_base + lane_base + buf * BN, p);
        tmem_wait_ld();
#pragma unroll
        for (int i = 0; i < 16; ++i) acc[i] = fmaf(p[i], ws * asc[i], acc[i]);
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&tempty[buf]);
      }
      kbg += nk;
      // Each set publishes its partial sums; they are added in set order.
      if (!bad) {
        float* mine = sXch + (size_t)(set * 128 + row) * kXchStride;
#pragma unroll
        for (int t = 0; t < BN; ++t) mine[t] = acc[t];
      }
      if (named_barrier_or(1, kEpi1Threads, bad)) {
        ok = false;
        break;
      }
      bool last = true;
      if (nseg > 1) {
        // publish this segment's partial, then find out whether it completes the unit
        float* part = a.split_part + (size_t)partial_slot(P, blockIdx.x, u) * 128 * BN;
        for (int i = etid; i < 128 * BN; i += kEpi1Threads) {
          const int r = i / BN, t = i % BN;
          float v = 0.0f;
#pragma unroll
          for (int j = 0; j < G; ++j) v += sXch[(size_t)(j * 128 + r) * kXchStride + t];
          part[i] = v;
        }
        // One thread's acq_rel add after the barrier publishes all 512 threads'
        // partials (release) and, for the last arriver, makes the other segments'
        // partials visible to all of them after the next barrier (acquire); no
        // per-thread fence.
        named_barrier_sync(1, kEpi1Threads);
        if (etid == 0) *sLast = (atom_add_acq_rel_gpu(&a.split_count[u], 1) == nseg - 1) ? 1 : 0;
        named_barrier_sync(1, kEpi1Threads);
        last = *sLast != 0;
      }
      if (last) {
        // SwiGLU: rows 0..63 (first half) pair with rows 64..127 (silu half).  Warp
        // w takes token row t = w, lane l its columns 2l and 2l + 1 of the slice.  The
        // row's 64 values are stored as two fp8 planes with one scale each (GEMM2's B
        // operand, see gemm2_phase): s0 = amax / 448, q0 = e4m3(y * 448 / amax), then
        // the same for the residual y - q0 * s0.
        const int c0 = P.first_owner(u);
        const int t = etid >> 5;  // 16 warps, 16 token rows
        const int r = 2 * lane;
        float y[2] = {0.0f, 0.0f};
        if (t < nrows) {
          float x1[2] = {0.0f, 0.0f}, x2[2] = {0.0f, 0.0f};
          if (nseg == 1) {
#pragma unroll
            for (int cc = 0; cc < 2; ++cc)
#pragma unroll
              for (int j = 0; j < G; ++j) {
                x1[cc] += sXch[(size_t)(j * 128 + r + cc) * kXchStride + t];
                x2[cc] += sXch[(size_t)(j * 128 + 64 + r + cc) * kXchStride + t];
              }
          } else {
            // the partials of up to four segments are loaded before any is added (one
            // L2 round trip per four segments, not per segment), then summed in
            // segment order (deterministic)
            for (int q0 = 0; q0 < nseg; q0 += kSegBatch) {
              float p1[kSegBatch][2], p2[kSegBatch][2];
#pragma unroll
              for (int q = 0; q < kSegBatch; ++q) {
                if (q0 + q < nseg) {
                  const float* pq = a.split_part + (size_t)partial_slot(P, c0 + q0 + q, u) * 128 * BN;
#pragma unroll
                  for (int cc = 0; cc < 2; ++cc) {
                    p1[q][cc] = __ldcg(pq + (r + cc) * BN + t);
                    p2[q][cc] = __ldcg(pq + (64 + r + cc) * BN + t);
                  }
                }
              }
#pragma unroll
              for (int q = 0; q < kSegBatch; ++q)
                if (q0 + q < nseg)
#pragma unroll
                  for (int cc = 0; cc < 2; ++cc) {
                    x1[cc] += p1[q][cc];
                    x2[cc] += p2[q][cc];
                  }
            }
          }
#pragma unroll
          for (int cc = 0; cc < 2; ++cc) y[cc] = x2[cc] / (1.0f + expf(-x2[cc])) * x1[cc];
        }
        if (!isfinite(y[0]) || !isfinite(y[1])) {
          atomicOr(a.status, kStatusSaturated);
          y[0] = isfinite(y[0]) ? y[0] : 0.0f;
          y[1] = isfinite(y[1]) ? y[1] : 0.0f;
        }
#pragma unroll
        for (int pl = 0; pl < 2; ++pl) {
          float m = fmaxf(fabsf(y[0]), fabsf(y[1]));
#pragma unroll
          for (int d = 16; d >= 1; d >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, d));
          const float sc = m > 0.0f ? m * (1.0f / 448.0f) : 1.0f;
          const float inv = m > 0.0f ? __fdividef(448.0f, m) : 1.0f;
          uint32_t packed = 0;
#pragma unroll
          for (int cc = 0; cc < 2; ++cc) {
            const float v = fminf(fmaxf(y[cc] * inv, -448.0f), 448.0f);
            const __nv_fp8_storage_t f8 = __nv_cvt_float_to_fp8(v, __NV_SATFINITE, __NV_E4M3);
            packed |= (uint32_t)f8 << (8 * cc);
            const __half_raw hr = __nv_cvt_fp8_to_halfraw(f8, __NV_E4M3);
            y[cc] -= __half2float(*reinterpret_cast<const __half*>(&hr)) * sc;  // residual for plane 1
          }
          if (t < nrows) {
            const size_t prow = (size_t)pl * a.pcap + r0 + t;
            *reinterpret_cast<uint16_t*>(a.planes + prow * kInter + 64 * g + r) = (uint16_t)packed;
            if (lane == 0) a.plane_scale[((size_t)pl * kChunks + g) * a.pcap + r0 + t] = sc;
          }
        }
        if (nseg > 1 && etid == 0) a.split_count[u] = 0;  // ready for the next call
      }
      named_barrier_sync(1, kEpi1Threads);
      // one more of this block's 32 slices is published (GEMM2 waits for all 32): the
      // release-add after the barrier covers every thread's plane stores
      if (last && etid == 0) red_release_gpu_add(&a.blk_ready[u / kG1Slices], 1);
    }
  }
}

// ============================================================== GEMM2 phase
// GEMM1 stored each block's intermediate as two fp8 planes, per (token row,
// 64-column chunk) with its own scale (q0 * s0 + q1 * s1 ~ the fp32 SwiGLU output,
// the 1x64 block rule applied to the value and then to its residual).  GEMM2 runs
// as kind::f8f6f4 straight on the fp8 W2 tile -- no dequantisation of W2 -- with
// the two planes stacked as the N = 32 operand, and is promoted per 64-K chunk by
// the W2 block scale times each plane's scale:
//     acc[t] += s2[h, kb] * (s0[t, c] * D[:, t] + s1[t, c] * D[:, 16 + t])
// W2 enters exactly (fp8 times its fp32 scale); two planes keep about eight
// significant bits of every intermediate value relative to its chunk's largest.
// Measured on the host against the fp32 intermediate, the worst pair-row element is
// within 0.13x the output tolerance (0.08x for the f16 intermediate with f16 W2 this
// replaces, 0.40x for bf16, 5.8x for a single fp8 plane).
//
// Warps: w0 W2 producer (TMA ring); w2 copies a block's planes and scales (cp.async
// by the whole warp, once per block, after GEMM1 published the block's 32 slices and the MMAs on the
// previous block's planes completed); w1 MMA issuer; w4-w19 promote every chunk,
// each warp four token rows of its TMEM lane quarter, and at a unit's end multiply
// by the routing weights and store the f16 pair rows of the segment's plane.
__device__ __forceinline__ void gemm2_phase(const DecodeArgs& a, uint8_t* sm, uint64_t* bars, uint32_t tmem_base,
                                            int nb, volatile int* sAbort) {
  constexpr int SR = kRawStages;
  uint8_t* sRaw = sm + kP2Raw;
  uint8_t* sPlanes = sm + kP2Planes;
  const float* sPScale = reinterpret_cast<const float*>(sm + kP2PScale);  // [2 planes][32 chunks][16 rows]
  uint64_t* raw_full = bars;                  // W2 tile landed (TMA)
  uint64_t* raw_empty = bars + SR;            // MMA done with it (a promotion thread, after the slot's commit)
  uint64_t* planes_full = bars + 2 * SR;      // a block's planes and scales copied (cp.async, one arrive)
  uint64_t* planes_empty = planes_full + 1;   // MMA done with them (another block follows)
  uint64_t* tfull = planes_full + 2;
  uint64_t* tempty = tfull + kSlots2;
  uint64_t* drain = tempty + kSlots2;
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const Partition P = gemm2_partition(nb, a.streamk != 0);
  const int x_beg = P.begin(blockIdx.x), x_end = P.begin(blockIdx.x + 1);
  auto fail = [&](uint32_t bit) {
    *sAbort = 1;
    atomicOr(a.status, bit);
  };

  if (warp == 0) {
    // ------------------------------------------------------------ W2 producer
    if (lane == 0) {
      const uint64_t pol = l2_policy_evict_first();
      Ring ring(SR);
      bool ok = true;
      uint32_t last_parity[SR];
      for (int s = 0; s < SR; ++s) last_parity[s] = 0xFFFFFFFFu;
      for (int x = x_beg; x < x_end && ok;) {
        const Seg sg = seg_at(P, x, x_end);
        x += sg.kb1 - sg.kb0;
        const int4 blk = dbg_block(a.blocks[sg.u / kG2Slices], BN, a.e_local, a.pcap, a.status);
        const int wrow = blk.x * kHidden + (sg.u % kG2Slices) * 128;
        for (int kb = sg.kb0; kb < sg.kb1; ++kb) {
          if (!mbar_wait(&raw_empty[ring.slot], ring.phase ^ 1u, sAbort, kWaitBudgetNs)) {
            ok = false;
            fail(kStatusTimeoutProducer);
            break;
          }
          mbar_arrive_expect_tx(&raw_full[ring.slot], kRawBytes);
          tma_load_2d(sRaw + ring.slot * kRawBytes, &a.tm_w2, &raw_full[ring.slot], kb * kBlk, wrow, pol);
          last_parity[ring.slot] = ring.phase;
          ring.next();
        }
      }
      // every issued TMA load lands before the CTA exits
      for (int s = 0; s < SR; ++s)
        if (last_parity[s] != 0xFFFFFFFFu)
          if (!mbar_wait_drain(&raw_full[s], last_parity[s], kWaitBudgetNs)) fail(kStatusTimeoutDrain);
    }
    __syncwarp();
  } else if (warp == 2) {
    // ------------------------------------------------------------ planes producer
    // The whole warp copies a block's planes and their scales with cp.async (generic
    // proxy: it reads what other CTAs stored after the counter's acquire without a
    // global proxy fence), then one shared-memory proxy fence hands them to the MMA.
    // Only the block's rows of the planes are copied: the MMA's columns for the other
    // rows read stale shared memory and their results are never stored.
    {
      int cur_blk = -1, nblk = 0;
      bool ok = true;
      for (int x = x_beg; x < x_end && ok;) {
        const Seg sg = seg_at(P, x, x_end);
        x += sg.kb1 - sg.kb0;
        const int b = sg.u / kG2Slices;
        if (b == cur_blk) continue;
        // the MMAs on the previous block's planes have completed
        if (nblk > 0 && !mbar_wait(planes_empty, (uint32_t)(nblk - 1) & 1u, sAbort, kWaitBudgetNs)) {
          if (lane == 0) fail(kStatusTimeoutProducer);
          break;
        }
        // GEMM1 published all 32 slices of the block's rows (every lane acquires)
        if (!wait_counter(&a.blk_ready[b], kG1Slices, sAbort, kWaitBudgetNs)) {
          ok = false;
          if (lane == 0) fail(kStatusTimeoutProducer);
          break;
        }
        const int4 blk = dbg_block(a.blocks[b], BN, a.e_local, a.pcap, a.status);
        const int r0 = blk.y, nr = min(blk.z, BN);
        // planes: [16 K-blocks][2 planes][nr rows][8 chunks of 16 B] into 128B-swizzled tiles
        const int n_plane_chunks = kIBlocks * 2 * nr * 8;
        for (int i = lane; i < n_plane_chunks; i += 32) {
          const int ch = i & 7, rest = i >> 3;
          const int t = rest % nr, pk = rest / nr;
          const int kb = pk >> 1, pl = pk & 1;
          const uint8_t* src = a.planes + ((size_t)pl * a.pcap + r0 + t) * kInter + kb * kBlk + ch * 16;
          cp_async_16(smem_u32(sPlanes + kb * kPlaneKBytes + pl * BN * 128 + sw128_offset(t, ch)), src, 16u);
        }
        // scales: [2 planes][32 chunks][16 rows] fp32, four rows per copy
        for (int i = lane; i < 2 * kChunks * (BN / 4); i += 32) {
          const int q4 = i & 3, pc = i >> 2;
          cp_async_16(smem_u32(sm + kP2PScale + (pc * BN + 4 * q4) * 4), a.plane_scale + (size_t)pc * a.pcap + r0 + 4 * q4,
                      16u);
        }
        cp_async_commit();
        cp_async_wait_all();
        fence_proxy_async_smem();  // generic-proxy shared-memory writes -> the MMA's reads
        __syncwarp();
        if (lane == 0) mbar_arrive(planes_full);
        ++nblk;
        cur_blk = b;
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = umma_idesc(0u, 128, kCols2);  // e4m3 x e4m3
      Ring ring(SR);
      uint32_t c = 0;  // K-blocks so far (slot uses)
      int cur_blk = -1, nblk = 0;
      bool ok = true;
      bool any = false;
      for (int x = x_beg, ug = 0; x < x_end && ok; ++ug) {
        const Seg sg = seg_at(P, x, x_end);
        x += sg.kb1 - sg.kb0;
        const int b = sg.u / kG2Slices;
        if (b != cur_blk) {
          if (!mbar_wait(planes_full, (uint32_t)nblk & 1u, sAbort, kWaitBudgetNs)) {
            ok = false;
            fail(kStatusTimeoutMma);
            break;
          }
          ++nblk;
          cur_blk = b;
        }
        for (int kb = sg.kb0; kb < sg.kb1 && ok; ++kb) {
          if (!mbar_wait(&raw_full[ring.slot], ring.phase, sAbort, kWaitBudgetNs)) {
            ok = false;
            fail(kStatusTimeoutMma);
            break;
          }
          const uint32_t slot = c % kSlots2;
          if (!mbar_wait(&tempty[slot], ((c / kSlots2) & 1u) ^ 1u, sAbort, kWaitBudgetNs)) {
            ok = false;
            fail(kStatusTimeoutMma);
            break;
          }
          tc_fence_after();
          const uint64_t adesc = umma_desc_sw128(smem_u32(sRaw + ring.slot * kRawBytes));
          const uint64_t bdesc = umma_desc_sw128(smem_u32(sPlanes + kb * kPlaneKBytes));
          // two 64-K chunks, each into its own half of the slot (promoted with its own plane scales)
#pragma unroll
          for (int ch = 0; ch < 2; ++ch) {
            const uint32_t d = tmem_base + (slot * 2 + ch) * kCols2;
            mma_f8f6f4(d, adesc + 4 * ch, bdesc + 4 * ch, idesc, 0u);
            mma_f8f6f4(d, adesc + 4 * ch + 2, bdesc + 4 * ch + 2, idesc, 1u);
          }
          tc_commit(&tfull[slot]);
          any = true;
          ring.next();
          ++c;
        }
        if (!ok) break;
        // another block follows in this CTA's range: release the planes once these MMAs complete
        if (x < x_end && seg_at(P, x, x_end).u / kG2Slices != b) tc_commit(planes_empty);
      }
      if (any) {
        tc_commit(drain);
        mbar_wait_drain(drain, 0, kWaitBudgetNs);
      }
    }
    __syncwarp();
  } else if (warp >= 4) {
    // ------------------------------------------------------------ promotion
    // All 16 warps take every chunk: warp w reads TMEM lanes 32 (w % 4) .. +31 (its
    // 32 W2 rows) and columns of token rows 4 tg .. 4 tg + 3, tg = (w - 4) / 4, of
    // both planes; each thread accumulates its W2 row for those four tokens.
    const int q4 = warp & 3;           // TMEM lane quarter
    const int tg = (warp - 4) >> 2;    // token rows 4 tg .. 4 tg + 3
    const int hrow = q4 * 32 + lane;   // W2 row of the tile == TMEM lane
    const uint32_t lane_base = (uint32_t)(q4 * 32) << 16;
    uint32_t c = 0;    // K-blocks so far, in the MMA's order
    int rstage = 0;    // the raw W2 stage K-block c was read from
    bool ok = true;
    for (int x = x_beg; x < x_end && ok;) {
      const Seg sg = seg_at(P, x, x_end);
      x += sg.kb1 - sg.kb0;
      const int nk = sg.kb1 - sg.kb0;
      const int u = sg.u;
      const int4 blk = dbg_block(a.blocks[u / kG2Slices], BN, a.e_local, a.pcap, a.status);
      const int h = u % kG2Slices;
      const int e = blk.x, r0 = blk.y, nrows = blk.z;
      const float lane_scale = __ldg(a.w2_scale + ((size_t)e * kHBlocks + h) * kIBlocks + (lane & (kIBlocks - 1)));
      float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
      for (int kb = sg.kb0; kb < sg.kb1; ++kb) {
        const float ws = __shfl_sync(0xffffffffu, lane_scale, kb);
        float d[2][2][4];  // [chunk][plane][token]
        const uint32_t slot = c % kSlots2;
        if (!mbar_wait(&tfull[slot], (c / kSlots2) & 1u, sAbort, kWaitBudgetNs)) {
          ok = false;
          if (lane == 0) fail(kStatusTimeoutEpilogue);
          break;
        }
        tc_fence_after();
#pragma unroll
        for (int ch = 0; ch < 2; ++ch)
#pragma unroll
          for (int pl = 0; pl < 2; ++pl)
            tmem_ld4(tmem_base + lane_base + (slot * 2 + ch) * kCols2 + pl * BN + 4 * tg, d[ch][pl]);
        tmem_wait_ld();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&tempty[slot]);
        // the slot's MMAs are complete, so the raw W2 stage they read is free (one thread signals)
        if (threadIdx.x == 128) mbar_arrive(&raw_empty[rstage]);
        rstage = rstage + 1 == kRawStages ? 0 : rstage + 1;
        ++c;
#pragma unroll
        for (int ch = 0; ch < 2; ++ch) {
          const int chunk = 2 * kb + ch;
#pragma unroll
          for (int pl = 0; pl < 2; ++pl) {
            // this plane's scales of the chunk for token rows 4 tg .. 4 tg + 3
            const float4 sv = *reinterpret_cast<const float4*>(sPScale + (pl * kChunks + chunk) * BN + 4 * tg);
            const float sj[4] = {sv.x, sv.y, sv.z, sv.w};
#pragma unroll
            for (int j = 0; j < 4; ++j) acc[j] = fmaf(d[ch][pl][j], ws * sj[j], acc[j]);
          }
        }
      }
      if (!ok) break;
      (void)nk;
      const int sp = blockIdx.x - P.first_owner(u);  // segment index = plane of pair rows
      __half* dst = a.pair_out + (size_t)sp * a.plane_elems + (size_t)r0 * kHidden + h * 128 + hrow;
      bool sat = false;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int t = 4 * tg + j;
        if (t < nrows) dst[(size_t)t * kHidden] = to_half_sat(acc[j] * __ldg(a.row_weight + r0 + t), sat);
      }
      if (sat) atomicOr(a.status, kStatusSaturated);
    }
  }
}

// ============================================================== combine phase
// After every CTA has written its pair rows (one arrival each on a grid counter
// that the permute kernel zeroed): out[t, 8c .. 8c+7] for every token t and
// column group c, spread over all threads of the grid.  The token's pair rows are
// summed over planes, then slots, in fixed order (deterministic), in fp32.
__device__ __forceinline__ void combine_phase(const DecodeArgs& a, int nb, volatile int* sAbort) {
  const Partition P2 = gemm2_partition(nb, a.streamk != 0);
  constexpr int kGroupsPerRow = kHidden / 8;
  const int tasks = a.T * kGroupsPerRow;
  // consecutive tasks go to different CTAs, so a small T still uses many SMs
  const int first = threadIdx.x * gridDim.x + blockIdx.x;
  // A task's slot rows and plane counts depend only on the permutation, so the
  // first task's are fetched while the grid arrival completes.
  int rows[kTopK], np[kTopK];
  auto prep = [&](int task) {
    const int t = task / kGroupsPerRow, h = (task % kGroupsPerRow) * 8 / 128;
    const int4* rows4 = reinterpret_cast<const int4*>(a.token_rows + (size_t)t * kTopK);
    const int4 ra = __ldg(rows4), rb = __ldg(rows4 + 1);
    rows[0] = ra.x; rows[1] = ra.y; rows[2] = ra.z; rows[3] = ra.w;
    rows[4] = rb.x; rows[5] = rb.y; rows[6] = rb.z; rows[7] = rb.w;
#pragma unroll
    for (int k = 0; k < kTopK; ++k) rows[k] = dbg_row(rows[k], a.pcap, a.status);
    // planes of each slot's pair row: the GEMM2 segments of its unit (block = row / 16, slice h)
#pragma unroll
    for (int k = 0; k < kTopK; ++k) np[k] = rows[k] >= 0 ? P2.nseg((rows[k] / BN) * kG2Slices + h) : 0;
  };
  // this CTA's pair rows (ordered before by the CTA barrier) are visible grid-wide
  // once the release-add lands
  if (threadIdx.x == 0) red_release_gpu_add(a.grid_sync, 1);
  // the first task's slot rows load while the other CTAs arrive
  if (first < tasks) prep(first);
  if (threadIdx.x == 0) {
    if (!wait_counter(a.grid_sync, (int)gridDim.x + a.grid_extra, sAbort, a.grid_wait_ns)) {
      *sAbort = 1;
      atomicOr(a.status, kStatusTimeoutEpilogue);
    }
  }
  __syncthreads();
  if (*sAbort) return;
  for (int task = first; task < tasks; task += gridDim.x * kThreads) {
    if (task != first) prep(task);
    const int t = task / kGroupsPerRow;
    const size_t col = (size_t)(task % kGroupsPerRow) * 8;
    float acc[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) acc[i] = 0.0f;
    for (int pl = 0; pl < 2; ++pl) {  // planes, then slots: fixed order
      // the plane's (up to 8) rows are loaded together: one L2 round trip per plane
      uint4 v[kTopK];
#pragma unroll
      for (int k = 0; k < kTopK; ++k)
        v[k] = pl < np[k] ? __ldcg(reinterpret_cast<const uint4*>(a.pair_out + (size_t)pl * a.plane_elems +
                                                                  (size_t)rows[k] * kHidden + col))
                          : make_uint4(0u, 0u, 0u, 0u);
#pragma unroll
      for (int k = 0; k < kTopK; ++k) {
        if (pl < np[k]) {
          const uint32_t w[4] = {v[k].x, v[k].y, v[k].z, v[k].w};
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&w[i]));
            acc[2 * i] += f.x;
            acc[2 * i + 1] += f.y;
          }
        }
      }
    }
    if (a.f32_out) {
      float4* o = reinterpret_cast<float4*>(reinterpret_cast<float*>(a.out) + (size_t)t * kHidden + col);
      o[0] = make_float4(acc[0], acc[1], acc[2], acc[3]);
      o[1] = make_float4(acc[4], acc[5], acc[6], acc[7]);
    } else {
      uint4 o;
      uint32_t* ow = reinterpret_cast<uint32_t*>(&o);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const __nv_bfloat162 bv = __floats2bfloat162_rn(acc[2 * i], acc[2 * i + 1]);
        ow[i] = *reinterpret_cast<const uint32_t*>(&bv);
      }
      *reinterpret_cast<uint4*>(reinterpret_cast<__nv_bfloat16*>(a.out) + (size_t)t * kHidden + col) = o;
    }
  }
}

__global__ void __launch_bounds__(kThreads, 1) decode_kernel(const __grid_constant__ DecodeArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars1 = reinterpret_cast<uint64_t*>(sm + kOffBar);
  uint64_t* bars2 = bars1 + kNumBars1;
  uint32_t* sTmem = reinterpret_cast<uint32_t*>(sm + kOffMisc);
  volatile int* sAbort = reinterpret_cast<volatile int*>(sm + kOffMisc + 4);
  volatile int* sLast = reinterpret_cast<volatile int*>(sm + kOffMisc + 8);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    // phase 1: full/empty [8], tfull/tempty [32], drain
    for (int s = 0; s < kStages1; ++s) {
      mbar_init(&bars1[s], 2);               // producer expect_tx arrive + cp.async completion arrive
      mbar_init(&bars1[kStages1 + s], 1);    // tcgen05.commit
    }
    for (int b = 0; b < kBufs1; ++b) {
      mbar_init(&bars1[2 * kStages1 + b], 1);           // tcgen05.commit
      mbar_init(&bars1[2 * kStages1 + kBufs1 + b], 4);  // one arrive per warp of the owning set
    }
    mbar_init(&bars1[2 * kStages1 + 2 * kBufs1], 1);
    // phase 2: raw full/empty, planes full/empty, tfull/tempty, drain
    uint64_t* b2 = bars2;
    for (int s = 0; s < kRawStages; ++s) {
      mbar_init(&b2[s], 1);                // producer's expect_tx arrive
      mbar_init(&b2[kRawStages + s], 1);   // one promotion thread, after the slot's commit
    }
    b2 += 2 * kRawStages;
    mbar_init(&b2[0], 1);  // the block's planes written (one arrive)
    mbar_init(&b2[1], 1);  // MMA done with them (tcgen05.commit)
    b2 += 2;
    for (int b = 0; b < kSlots2; ++b) {
      mbar_init(&b2[b], 1);             // tcgen05.commit
      mbar_init(&b2[kSlots2 + b], 16);  // one arrive per promotion warp
    }
    mbar_init(&b2[2 * kSlots2], 1);
    *sAbort = 0;
    fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&a.tm_w1);
    tma_prefetch_desc(&a.tm_w2);
  }
  if (warp == 1) {
    tmem_alloc(sTmem, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  pdl_wait();
  pdl_trigger();
  fence_proxy_async_global();
  const uint32_t tmem_base = *sTmem;
  const int nb = *a.n_blocks;

  if (nb == 0) {
    // no local (token, expert) pair: the output is all zeros
    const size_t n16 = (size_t)a.T * kHidden * (a.f32_out ? 4 : 2) / 16;
    uint4* o = reinterpret_cast<uint4*>(a.out);
    for (size_t i = (size_t)blockIdx.x * kThreads + threadIdx.x; i < n16; i += (size_t)gridDim.x * kThreads)
      o[i] = make_uint4(0u, 0u, 0u, 0u);
  } else {
    gemm1_phase(a, sm, bars1, tmem_base, nb, sAbort, sLast);
    // The shared region changes role: order this CTA's generic-proxy accesses of
    // phase 1 before the TMA writes of phase 2, and phase 1's TMEM reads before
    // phase 2's MMAs.
    fence_proxy_async_smem();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (!*sAbort) gemm2_phase(a, sm, bars2, tmem_base, nb, sAbort);
    __syncthreads();  // this CTA's pair rows are all written
    combine_phase(a, nb, sAbort);
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, kTmemCols);
  }
  // The decode kernel is the last of the call: a status bit set by any kernel of
  // the call (this CTA's included, ordered by the barrier above) reaches the sink.
  if (threadIdx.x == 0) forward_status_to_sink(a.status, a.sink);
}

}  // namespace

// How the decode kernel was last launched (fbmoe_decode_launch_mode).
static std::atomic<int> g_decode_mode{0};

int decode_launch_mode() { return g_decode_mode.load(std::memory_order_relaxed); }

cudaError_t launch_decode(const CUtensorMap* tm_w1, const CUtensorMap* tm_w2,
                          const uint8_t* hidden, const float* hidden_scale, int T, const float* w1_scale,
                          const float* w2_scale, const Layout& L, uint8_t* ws, void* out, bool f32_out, int num_sms,
                          uint32_t* sink, bool w1_packed, cudaStream_t stream) {
  static DeviceFlags attr_set;
  if (cudaError_t err = set_max_dynamic_smem(decode_kernel, kSmemBytes, attr_set); err != cudaSuccess) return err;
  DecodeArgs a;
  a.tm_w1 = *tm_w1;
  a.tm_w2 = *tm_w2;
  a.hidden = hidden;
  a.hidden_scale = hidden_scale;
  a.w1_scale = w1_scale;
  a.w2_scale = w2_scale;
  a.n_blocks = reinterpret_cast<const int32_t*>(ws + L.n_blocks);
  a.blocks = reinterpret_cast<const int4*>(ws + L.blocks);
  a.row_token = reinterpret_cast<const int32_t*>(ws + L.row_token);
  a.row_weight = reinterpret_cast<const float*>(ws + L.row_weight);
  a.token_rows = reinterpret_cast<const int32_t*>(ws + L.token_rows);
  a.streamk = L.split_items > 0 ? 1 : 0;
  a.split_count = reinterpret_cast<int32_t*>(ws + L.split_count);
  a.split_part = reinterpret_cast<float*>(ws + L.split_part);
  a.blk_ready = reinterpret_cast<int32_t*>(ws + L.blk_ready);
  a.grid_sync = reinterpret_cast<int32_t*>(ws + L.grid_sync);
  a.planes = ws + L.inter;  // the f16 intermediate's region holds the two fp8 planes
  a.plane_scale = reinterpret_cast<float*>(ws + L.plane_scale);
  a.pair_out = reinterpret_cast<__half*>(ws + L.pair_out);
  a.out = out;
  a.status = reinterpret_cast<uint32_t*>(ws + L.status);
  a.sink = sink;
  a.plane_elems = (size_t)L.pcap * kHidden;
  a.T = T;
  a.pcap = L.pcap;
  a.e_local = L.e_local;
  a.w1_packed = w1_packed ? 1 : 0;
  a.f32_out = f32_out ? 1 : 0;
  const bool expire = test_expire_grid_wait();
  a.grid_extra = expire ? 1 : 0;
  a.grid_wait_ns = expire ? kTestGridWaitNs : kWaitBudgetNs;
  // Every CTA waits at the grid arrival for all the others, so the whole grid
  // must be resident at once: one CTA per SM, and the occupancy query confirms
  // that one fits.  The default launch is a plain programmatic one (its CTAs start
  // while the router still runs; measured 1-3.5 us per call faster than a
  // cooperative launch).  With FBMOE_DECODE_COOPERATIVE=1 the kernel is launched
  // cooperatively, so that the launch itself guarantees co-residency even when
  // other work holds SMs: with programmatic serialization if the driver accepts
  // both, else without it.  The arrival wait is bounded either way.
  int occ = 0;
  cudaError_t e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, decode_kernel, kThreads, kSmemBytes);
  if (e != cudaSuccess) return e;
  if (occ < 1) return cudaErrorInvalidConfiguration;
  const int grid = num_sms > 0 ? num_sms : 1;
  static const bool coop = [] {
    const char* v = std::getenv("FBMOE_DECODE_COOPERATIVE");
    return v != nullptr && v[0] == '1';
  }();
  if (coop) {
    const int mode = g_decode_mode.load(std::memory_order_relaxed);
    if (mode == 0 || mode == 1) {
      e = launch_coop(decode_kernel, dim3(grid), dim3(kThreads), kSmemBytes, stream, true, a);
      if (e == cudaSuccess) {
        g_decode_mode.store(1, std::memory_order_relaxed);
        return e;
      }
      if (mode == 1) return e;
      (void)cudaGetLastError();  // a refused launch configuration is not a sticky error
    }
    e = launch_coop(decode_kernel, dim3(grid), dim3(kThreads), kSmemBytes, stream, false, a);
    if (e == cudaSuccess) g_decode_mode.store(2, std::memory_order_relaxed);
    return e;
  }
  g_decode_mode.store(3, std::memory_order_relaxed);
  return launch_pdl(decode_kernel, dim3(grid), dim3(kThreads), kSmemBytes, stream, a);
}

}  // namespace fbmoe
