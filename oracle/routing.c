/*
 * oracle/routing.c -- TEST INFRASTRUCTURE ONLY (the parity checker, never the product).
 *
 * CPU restatement of the DeepSeek-V3 no-aux router that the reference operator
 * computes in PyTorch (solution/triton/main.py:2522-2553 of weichengz0616/flashinfer-bench-moe):
 *
 *   s            = 1 / (1 + exp(-logits))                       main.py:2526
 *   s_with_bias  = s + bias                                     main.py:2527
 *   group score  = sum of the top-2 of each group of 32         main.py:2530-2534
 *   keep groups  = topk(group scores, 4, sorted=False)          main.py:2537
 *   experts      = topk(masked s_with_bias, 8, sorted=False)    main.py:2542-2546
 *   weights      = s[e] / (sum_e s[e] + 1e-20) * scale          main.py:2549-2553
 *
 * Tie semantics.  torch.topk(sorted=False) on a CPU tensor selects with
 * std::nth_element over (value, index) pairs ordered by "a.value > b.value"
 * (NaN first), so which of several equal values is kept is decided by the
 * introselect permutation, not by index.  topk_nth() below restates that
 * selection (GNU libstdc++ introselect: median-of-three pivot moved to the
 * front, unguarded Hoare partition, heap-select fallback when the depth limit
 * 2*floor(log2 n) runs out, insertion sort for <= 3 elements).  Its output
 * (order included) is checked against torch.topk itself and against
 * std::nth_element (oracle/nth_check.cc) by the CPU tests.
 *
 * Arithmetic.  exp() is evaluated in double and rounded once to float, i.e. the
 * correctly rounded fp32 exp; the add and the division are IEEE fp32.  torch's
 * own CPU exp is within 1 ulp of this value, so the two can differ in the last
 * bit of s; the CPU tests measure how often that changes a selection.
 * The expert weights are summed in ascending expert order.
 *
 * The selected experts are emitted in a canonical order (descending
 * s_with_bias, ascending index among equals); the operator's result depends only
 * on the selected set.
 */
#include <math.h>
#include <stdint.h>
#include <string.h>

typedef struct {
    float v;
    int32_t i;
} pair_t;

/* "a goes before b" for a largest-first selection: torch's comparator. */
static inline int before(const pair_t *a, const pair_t *b) {
    return (isnan(a->v) && !isnan(b->v)) || (a->v > b->v);
}

static inline void swap_pairs(pair_t *a, pair_t *b) {
    pair_t t = *a;
    *a = *b;
    *b = t;
}

/* Sift `val` up from `hole` towards `top` (binary max-heap on `before`). */
static void heap_push(pair_t *base, long hole, long top, pair_t val) {
    long parent = (hole - 1) / 2;
    while (hole > top && before(&base[parent], &val)) {
        base[hole] = base[parent];
        hole = parent;
        parent = (hole - 1) / 2;
    }
    base[hole] = val;
}

/* Move the larger child up until a leaf is reached, then push `val` back. */
static void heap_adjust(pair_t *base, long hole, long len, pair_t val) {
    const long top = hole;
    long child = hole;
    while (child < (len - 1) / 2) {
        child = 2 * (child + 1);
        if (before(&base[child], &base[child - 1])) child--;
        base[hole] = base[child];
        hole = child;
    }
    if ((len & 1) == 0 && child == (len - 2) / 2) {
        child = 2 * (child + 1);
        base[hole] = base[child - 1];
        hole = child - 1;
    }
    heap_push(base, hole, top, val);
}

static void heap_build(pair_t *base, long len) {
    if (len < 2) return;
    for (long parent = (len - 2) / 2;; parent--) {
        heap_adjust(base, parent, len, base[parent]);
        if (parent == 0) return;
    }
}

/* Keep the `mid` front-most elements of [0, n) under `before` in base[0, mid). */
static void heap_select(pair_t *base, long mid, long n) {
    heap_build(base, mid);
    for (long i = mid; i < n; i++) {
        if (before(&base[i], &base[0])) {
            pair_t val = base[i];
            base[i] = base[0];
            heap_adjust(base, 0, mid, val);
        }
    }
}

static void insertion_sort(pair_t *base, long n) {
    for (long i = 1; i < n; i++) {
        pair_t val = base[i];
        if (before(&val, &base[0])) {
            memmove(&base[1], &base[0], (size_t)i * sizeof(pair_t));
            base[0] = val;
        } else {
            long j = i;
            while (before(&val, &base[j - 1])) {
                base[j] = base[j - 1];
                j--;
            }
            base[j] = val;
        }
    }
}

static long floor_log2(long n) {
    long k = 0;
    while (n > 1) {
        n >>= 1;
        k++;
    }
    return k;
}

/* Partially order base[0, n) so that base[nth] holds the element a full sort
 * would put there and nothing after it goes before anything ahead of it. */
static void nth_element_pairs(pair_t *base, long n, long nth) {
    if (n == 0 || nth == n) return;
    long first = 0, last = n;
    long depth = 2 * floor_log2(n);
    while (last - first > 3) {
        if (depth == 0) {
            heap_select(base + first, nth + 1 - first, last - first);
            swap_pairs(&base[first], &base[nth]);
            return;
        }
        depth--;
        /* median of (first+1, mid, last-1) is swapped into `first` */
        long a = first + 1, b = first + (last - first) / 2, c = last - 1, m;
        if (before(&base[a], &base[b])) {
            if (before(&base[b], &base[c])) m = b;
            else if (before(&base[a], &base[c])) m = c;
            else m = a;
        } else if (before(&base[a], &base[c])) m = a;
        else if (before(&base[b], &base[c])) m = c;
        else m = b;
        swap_pairs(&base[first], &base[m]);
        /* unguarded partition of [first+1, last) around base[first] */
        long lo = first + 1, hi = last;
        for (;;) {
            while (before(&base[lo], &base[first])) lo++;
            hi--;
            while (before(&base[first], &base[hi])) hi--;
            if (!(lo < hi)) break;
            swap_pairs(&base[lo], &base[hi]);
            lo++;
        }
        if (lo <= nth) first = lo;
        else last = lo;
    }
    insertion_sort(base + first, last - first);
}

/* torch.topk(values[0:n], k, largest=True, sorted=False).indices, order included. */
void topk_nth(const float *values, int n, int k, int32_t *out_idx) {
    pair_t buf[1024];
    pair_t *p = buf;
    if (n > 1024 || k < 1 || k > n) return;
    for (int i = 0; i < n; i++) {
        p[i].v = values[i];
        p[i].i = i;
    }
    nth_element_pairs(p, n, k - 1);
    for (int i = 0; i < k; i++) out_idx[i] = p[i].i;
}

/* Full permutation left by the selection (perm[j] = original index at j). */
void nth_perm(const float *values, int n, int nth, int32_t *perm) {
    pair_t buf[4096];
    if (n > 4096 || nth < 0 || nth > n) return;
    for (int i = 0; i < n; i++) {
        buf[i].v = values[i];
        buf[i].i = i;
    }
    nth_element_pairs(buf, n, nth);
    for (int i = 0; i < n; i++) perm[i] = buf[i].i;
}

/* fp32 sigmoid with a correctly rounded exp, as the router kernel computes it. */
static inline float sigmoid_cr(float x) {
    float e = (float)exp(-(double)x);
    float d = 1.0f + e;
    return 1.0f / d;
}

enum { N_EXPERTS = 256, N_GROUPS = 8, GROUP_SIZE = 32, TOPK_GROUPS = 4, TOPK = 8 };

/*
 * Route T tokens.  logits: fp32 [T, 256] row-major.  bias: fp32 [256] (the
 * bf16 bias widened exactly).  Outputs: topk_idx int32 [T, 8] (global expert
 * ids, canonical order), topk_w fp32 [T, 8] (weight of the same expert),
 * s_bias fp32 [T, 256] (s + bias, may be NULL), tie_flag int32 [T] (may be
 * NULL): bit0 = group selection had a boundary tie, bit1 = expert selection
 * had a boundary tie.
 */
void route_tokens(const float *logits, const float *bias, int T, float scale,
                  int32_t *topk_idx, float *topk_w, float *s_bias, int32_t *tie_flag) {
    for (int t = 0; t < T; t++) {
        const float *x = logits + (size_t)t * N_EXPERTS;
        float s[N_EXPERTS], sb[N_EXPERTS];
        for (int e = 0; e < N_EXPERTS; e++) {
            s[e] = sigmoid_cr(x[e]);
            sb[e] = s[e] + bias[e];
            if (s_bias) s_bias[(size_t)t * N_EXPERTS + e] = sb[e];
        }
        /* group score: sum of the two largest (tie-independent) */
        float gscore[N_GROUPS];
        for (int g = 0; g < N_GROUPS; g++) {
            int32_t two[2];
            topk_nth(sb + g * GROUP_SIZE, GROUP_SIZE, 2, two);
            gscore[g] = sb[g * GROUP_SIZE + two[0]] + sb[g * GROUP_SIZE + two[1]];
        }
        int32_t gsel[TOPK_GROUPS];
        topk_nth(gscore, N_GROUPS, TOPK_GROUPS, gsel);
        int keep[N_GROUPS] = {0};
        for (int j = 0; j < TOPK_GROUPS; j++) keep[gsel[j]] = 1;
        float pruned[N_EXPERTS];
        for (int e = 0; e < N_EXPERTS; e++)
            pruned[e] = keep[e / GROUP_SIZE] ? sb[e] : -3.40282346638528859812e+38f;
        int32_t esel[TOPK];
        topk_nth(pruned, N_EXPERTS, TOPK, esel);

        if (tie_flag) {
            /* boundary tie: the k-th and (k+1)-th largest values are equal */
            float g[N_GROUPS];
            memcpy(g, gscore, sizeof g);
            for (int a = 1; a < N_GROUPS; a++)
                for (int b = a; b > 0 && g[b] > g[b - 1]; b--) {
                    float tmp = g[b]; g[b] = g[b - 1]; g[b - 1] = tmp;
                }
            int flag = (g[TOPK_GROUPS - 1] == g[TOPK_GROUPS]) ? 1 : 0;
            float kth = INFINITY;
            for (int j = 0; j < TOPK; j++) kth = fminf(kth, pruned[esel[j]]);
            for (int e = 0; e < N_EXPERTS; e++) {
                int inside = 0;
                for (int j = 0; j < TOPK; j++) inside |= (esel[j] == e);
                if (!inside && pruned[e] == kth) flag |= 2;
            }
            tie_flag[t] = flag;
        }

        /* canonical order: descending s_with_bias, ascending index among equals */
        for (int a = 1; a < TOPK; a++)
            for (int b = a; b > 0; b--) {
                float vb = sb[esel[b]], va = sb[esel[b - 1]];
                if (vb > va || (vb == va && esel[b] < esel[b - 1])) {
                    int32_t tmp = esel[b]; esel[b] = esel[b - 1]; esel[b - 1] = tmp;
                } else break;
            }
        /* weights: s / (sum of s over the selected set, ascending expert id) */
        int32_t asc[TOPK];
        memcpy(asc, esel, sizeof asc);
        for (int a = 1; a < TOPK; a++)
            for (int b = a; b > 0 && asc[b] < asc[b - 1]; b--) {
                int32_t tmp = asc[b]; asc[b] = asc[b - 1]; asc[b - 1] = tmp;
            }
        float sum = 0.0f;
        for (int j = 0; j < TOPK; j++) sum += s[asc[j]];
        sum = sum + 1e-20f;
        for (int j = 0; j < TOPK; j++) {
            topk_idx[(size_t)t * TOPK + j] = esel[j];
            topk_w[(size_t)t * TOPK + j] = (s[esel[j]] / sum) * scale;
        }
    }
}
