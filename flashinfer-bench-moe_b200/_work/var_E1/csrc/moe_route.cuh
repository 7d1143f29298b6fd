// moe_route.cuh -- device code of the DeepSeek-V3 no-aux router: route_token()
// routes one token with one warp, so any kernel can embed the router (the
// router kernel in moe_route.cu is its only caller today).  The algorithm and
// its exactness argument are described in moe_route.cu.
#pragma once
#include <float.h>
#include <math.h>

#include "fbmoe_common.cuh"

namespace fbmoe {
namespace route_dev {

// ---- torch.topk(sorted=False) CPU selection, replayed on (v, ix) arrays ----
__device__ __forceinline__ bool goes_before(float a, float b) { return (isnan(a) && !isnan(b)) || (a > b); }

__device__ __forceinline__ void swap_at(float* v, int* ix, int a, int b) {
  float tv = v[a];
  v[a] = v[b];
  v[b] = tv;
  int ti = ix[a];
  ix[a] = ix[b];
  ix[b] = ti;
}

__device__ inline void heap_push_dev(float* v, int* ix, int hole, int top, float val, int vi) {
  int parent = (hole - 1) / 2;
  while (hole > top && goes_before(v[parent], val)) {
    v[hole] = v[parent];
    ix[hole] = ix[parent];
    hole = parent;
    parent = (hole - 1) / 2;
  }
  v[hole] = val;
  ix[hole] = vi;
}

__device__ inline void heap_adjust_dev(float* v, int* ix, int hole, int len, float val, int vi) {
  const int top = hole;
  int child = hole;
  while (child < (len - 1) / 2) {
    child = 2 * (child + 1);
    if (goes_before(v[child], v[child - 1])) child--;
    v[hole] = v[child];
    ix[hole] = ix[child];
    hole = child;
  }
  if ((len & 1) == 0 && child == (len - 2) / 2) {
    child = 2 * (child + 1);
    v[hole] = v[child - 1];
    ix[hole] = ix[child - 1];
    hole = child - 1;
  }
  heap_push_dev(v, ix, hole, top, val, vi);
}

__device__ inline void heap_select_dev(float* v, int* ix, int mid, int n) {
  if (mid >= 2) {
    for (int parent = (mid - 2) / 2;; parent--) {
      heap_adjust_dev(v, ix, parent, mid, v[parent], ix[parent]);
      if (parent == 0) break;
    }
  }
  for (int i = mid; i < n; i++) {
    if (goes_before(v[i], v[0])) {
      float val = v[i];
      int vi = ix[i];
      v[i] = v[0];
      ix[i] = ix[0];
      heap_adjust_dev(v, ix, 0, mid, val, vi);
    }
  }
}

__device__ inline void insertion_sort_dev(float* v, int* ix, int n) {
  for (int i = 1; i < n; i++) {
    float val = v[i];
    int vi = ix[i];
    if (goes_before(val, v[0])) {
      for (int j = i; j > 0; j--) {
        v[j] = v[j - 1];
        ix[j] = ix[j - 1];
      }
      v[0] = val;
      ix[0] = vi;
    } else {
      int j = i;
      while (goes_before(val, v[j - 1])) {
        v[j] = v[j - 1];
        ix[j] = ix[j - 1];
        j--;
      }
      v[j] = val;
      ix[j] = vi;
    }
  }
}

// After the call, v/ix[0..nth] hold the nth+1 front-most elements exactly as
// std::nth_element leaves them.
__device__ inline void nth_select_dev(float* v, int* ix, int n, int nth) {
  if (n == 0 || nth == n) return;
  int first = 0, last = n;
  int lg = 0;
  for (int m = n; m > 1; m >>= 1) lg++;
  int depth = 2 * lg;
  while (last - first > 3) {
    if (depth == 0) {
      heap_select_dev(v + first, ix + first, nth + 1 - first, last - first);
      swap_at(v, ix, first, nth);
      return;
    }
    depth--;
    const int a = first + 1, b = first + (last - first) / 2, c = last - 1;
    int m;
    if (goes_before(v[a], v[b])) {
      if (goes_before(v[b], v[c])) m = b;
      else if (goes_before(v[a], v[c])) m = c;
      else m = a;
    } else if (goes_before(v[a], v[c])) m = a;
    else if (goes_before(v[b], v[c])) m = c;
    else m = b;
    swap_at(v, ix, first, m);
    int lo = first + 1, hi = last;
    for (;;) {
      while (goes_before(v[lo], v[first])) lo++;
      hi--;
      while (goes_before(v[first], v[hi])) hi--;
      if (!(lo < hi)) break;
      swap_at(v, ix, lo, hi);
      lo++;
    }
    if (lo <= nth) first = lo;
    else last = lo;
  }
  insertion_sort_dev(v + first, ix + first, last - first);
}

__device__ __forceinline__ float sigmoid_exact(float x) {
  const float e = (float)exp(-(double)x);
  return __fdiv_rn(1.0f, __fadd_rn(1.0f, e));
}

// Bias of this lane's 8 experts (bf16 -> fp32 is exact).
__device__ __forceinline__ void load_bias8(const __nv_bfloat16* __restrict__ bias, float (&bs)[8]) {
  const int lane = threadIdx.x & 31;
  const uint4 braw = *reinterpret_cast<const uint4*>(bias + lane * 8);
  const uint32_t w[4] = {braw.x, braw.y, braw.z, braw.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    bs[2 * i] = __uint_as_float(w[i] << 16);
    bs[2 * i + 1] = __uint_as_float(w[i] & 0xFFFF0000u);
  }
}

// This lane's 8 logits of token t (experts 8 * lane .. 8 * lane + 7).
__device__ __forceinline__ void load_logits8(const float* __restrict__ logits, int t, float (&x)[8]) {
  const int lane = threadIdx.x & 31;
  const float4* lp = reinterpret_cast<const float4*>(logits + (size_t)t * kExperts + lane * 8);
  const float4 xa = __ldg(lp), xb = __ldg(lp + 1);
  x[0] = xa.x; x[1] = xa.y; x[2] = xa.z; x[3] = xa.w;
  x[4] = xb.x; x[5] = xb.y; x[6] = xb.z; x[7] = xb.w;
}

// The calling warp routes token t from its logits x (load_logits8): topk_idx/topk_w
// [t*8 .. t*8+7].  wv, wi, ws: this warp's scratch of 256 entries each; ssel: its scratch of 8.
__device__ __forceinline__ void route_token(const float (&x)[8], int t, const float (&bs)[8], float scale,
                                            int32_t* __restrict__ topk_idx, float* __restrict__ topk_w, float* wv,
                                            int* wi, float* ws, int* ssel) {
  const int lane = threadIdx.x & 31;
  float s[8], sb[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    s[i] = sigmoid_exact(x[i]);
    sb[i] = __fadd_rn(s[i], bs[i]);
  }
  *reinterpret_cast<float4*>(ws + lane * 8) = make_float4(s[0], s[1], s[2], s[3]);
  *reinterpret_cast<float4*>(ws + lane * 8 + 4) = make_float4(s[4], s[5], s[6], s[7]);

  // ---- group score: sum of the two largest (as a multiset: tie-independent)
  float m1 = -INFINITY, m2 = -INFINITY;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    if (sb[i] > m1) {
      m2 = m1;
      m1 = sb[i];
    } else if (sb[i] > m2) {
      m2 = sb[i];
    }
  }
#pragma unroll
  for (int d = 1; d <= 2; d <<= 1) {
    const float o1 = __shfl_xor_sync(0xffffffffu, m1, d);
    const float o2 = __shfl_xor_sync(0xffffffffu, m2, d);
    const float n1 = fmaxf(m1, o1);
    const float n2 = fmaxf(fminf(m1, o1), fmaxf(m2, o2));
    m1 = n1;
    m2 = n2;
  }
  const float gscore = __fadd_rn(m1, m2);
  float gs[kGroups];
#pragma unroll
  for (int g = 0; g < kGroups; ++g) gs[g] = __shfl_sync(0xffffffffu, gscore, g * 4);

  // ---- keep 4 of 8 groups.  Sorted copy decides whether the boundary is tied.
  float srt[kGroups];
#pragma unroll
  for (int g = 0; g < kGroups; ++g) srt[g] = gs[g];
#pragma unroll
  for (int a = 0; a < kGroups; ++a)
#pragma unroll
    for (int b = 0; b < kGroups - 1 - a; ++b) {
      const float hi = fmaxf(srt[b], srt[b + 1]), lo = fminf(srt[b], srt[b + 1]);
      srt[b] = hi;
      srt[b + 1] = lo;
    }
  uint32_t keep = 0;
  if (srt[kTopKGroups - 1] != srt[kTopKGroups]) {
#pragma unroll
    for (int g = 0; g < kGroups; ++g) keep |= (gs[g] >= srt[kTopKGroups - 1]) ? (1u << g) : 0u;
  } else {
    if (lane == 0) {
#pragma unroll
      for (int g = 0; g < kGroups; ++g) {
        wv[g] = gs[g];
        wi[g] = g;
      }
      nth_select_dev(wv, wi, kGroups, kTopKGroups - 1);
      uint32_t k = 0;
      for (int j = 0; j < kTopKGroups; ++j) k |= 1u << wi[j];
      wi[0] = (int)k;
    }
    __syncwarp();
    keep = (uint32_t)wi[0];
    __syncwarp();
  }

  // ---- top-8 experts of the kept groups (masked entries = finfo(fp32).min)
  const bool mine = (keep >> (lane >> 2)) & 1u;
  float mv[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) mv[i] = mine ? sb[i] : -FLT_MAX;

  int sel[kTopK];
  float selv[kTopK];
  float v9 = -INFINITY;
  uint32_t taken = 0;
#pragma unroll
  for (int r = 0; r <= kTopK; ++r) {
    float bv = -INFINITY;
    int bi = 0x7fffffff;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      if (!((taken >> i) & 1u) && mv[i] > bv) {
        bv = mv[i];
        bi = lane * 8 + i;
      }
    }
    // Warp arg-max with the same order (largest value; among equal values the
    // smallest index): one redux.max over an order-preserving key of the value,
    // then the lowest lane holding the maximum (a lane's experts are 8 * lane + i,
    // and its local scan kept the smallest i).  -0 is folded into +0, as in the
    // float comparison.
    {
      uint32_t ub = __float_as_uint(bv);
      if (ub == 0x80000000u) ub = 0u;
      const uint32_t key = (ub & 0x80000000u) ? ~ub : (ub | 0x80000000u);
      const uint32_t kmax = __reduce_max_sync(0xffffffffu, key);
      const int win = __ffs(__ballot_sync(0xffffffffu, key == kmax)) - 1;
      bv = __shfl_sync(0xffffffffu, bv, win);
      bi = __shfl_sync(0xffffffffu, bi, win);
    }
    if (r < kTopK) {
      sel[r] = bi;
      selv[r] = bv;
      if ((bi >> 3) == lane) taken |= 1u << (bi & 7);
    } else {
      v9 = bv;
    }
  }

  if (v9 == selv[kTopK - 1]) {
    // Tied boundary: replay torch's selection over all 256 (masked) entries.
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      wv[lane * 8 + i] = mv[i];
      wi[lane * 8 + i] = lane * 8 + i;
    }
    __syncwarp();
    if (lane == 0) {
      nth_select_dev(wv, wi, kExperts, kTopK - 1);
      // canonical order of the chosen set
      int ci[kTopK];
      float cv[kTopK];
      for (int j = 0; j < kTopK; ++j) {
        ci[j] = wi[j];
        cv[j] = wv[j];
      }
      for (int a = 1; a < kTopK; ++a)
        for (int b = a; b > 0; --b) {
          if (cv[b] > cv[b - 1] || (cv[b] == cv[b - 1] && ci[b] < ci[b - 1])) {
            const float tv = cv[b];
            cv[b] = cv[b - 1];
            cv[b - 1] = tv;
            const int ti = ci[b];
            ci[b] = ci[b - 1];
            ci[b - 1] = ti;
          } else {
            break;
          }
        }
      for (int j = 0; j < kTopK; ++j) ssel[j] = ci[j];
    }
    __syncwarp();
#pragma unroll
    for (int j = 0; j < kTopK; ++j) sel[j] = ssel[j];
    __syncwarp();
  }

  // ---- weights: s / (sum over the set in ascending id + 1e-20) * scale
  int asc[kTopK];
#pragma unroll
  for (int j = 0; j < kTopK; ++j) asc[j] = sel[j];
#pragma unroll
  for (int a = 0; a < kTopK; ++a)
#pragma unroll
    for (int b = 0; b < kTopK - 1 - a; ++b) {
      const int lo = min(asc[b], asc[b + 1]), hi = max(asc[b], asc[b + 1]);
      asc[b] = lo;
      asc[b + 1] = hi;
    }
  __syncwarp();
  float sum = 0.0f;
#pragma unroll
  for (int j = 0; j < kTopK; ++j) sum = __fadd_rn(sum, ws[asc[j]]);
  sum = __fadd_rn(sum, 1e-20f);
  if (lane < kTopK) {
    int my = sel[0];
#pragma unroll
    for (int j = 1; j < kTopK; ++j) my = (lane == j) ? sel[j] : my;
    topk_idx[(size_t)t * kTopK + lane] = my;
    topk_w[(size_t)t * kTopK + lane] = __fmul_rn(__fdiv_rn(ws[my], sum), scale);
  }
  __syncwarp();
}

}  // namespace route_dev
}  // namespace fbmoe
