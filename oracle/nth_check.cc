// oracle/nth_check.cc -- TEST INFRASTRUCTURE ONLY.
// Pins oracle/routing.c's nth_perm() against the C++ standard library's own
// std::nth_element (the selection torch.topk(sorted=False) runs on CPU) on
// random, tie-heavy and pivot-adversarial inputs.  Prints the mismatch count
// and exits non-zero on any mismatch.
#include <algorithm>
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <random>
#include <utility>
#include <vector>

extern "C" void nth_perm(const float *values, int n, int nth, int32_t *perm);

static bool run_case(const std::vector<float> &v, int nth) {
  const int n = (int)v.size();
  std::vector<std::pair<float, int>> q(n);
  for (int i = 0; i < n; i++) q[i] = {v[i], i};
  std::nth_element(q.begin(), q.begin() + nth, q.end(),
                   [](const std::pair<float, int> &a, const std::pair<float, int> &b) {
                     return (std::isnan(a.first) && !std::isnan(b.first)) || (a.first > b.first);
                   });
  std::vector<int32_t> perm(n);
  nth_perm(v.data(), n, nth, perm.data());
  for (int i = 0; i < n; i++)
    if (perm[i] != q[i].second) return false;
  return true;
}

int main(int argc, char **argv) {
  long cases = argc > 1 ? atol(argv[1]) : 200000;
  std::mt19937_64 rng(12345);
  long bad = 0, done = 0;
  const int sizes[] = {4, 5, 7, 8, 9, 16, 31, 32, 33, 64, 100, 128, 255, 256, 257, 1000};
  for (long c = 0; c < cases; c++) {
    int n = sizes[rng() % (sizeof(sizes) / sizeof(sizes[0]))];
    int nth = (int)(rng() % n);
    int kind = (int)(rng() % 5);
    std::vector<float> v(n);
    int nuniq = 1 + (int)(rng() % 6);
    for (int i = 0; i < n; i++) {
      switch (kind) {
        case 0: v[i] = (float)(rng() % 1000003) / 7.0f; break;           // mostly distinct
        case 1: v[i] = (float)(rng() % nuniq); break;                     // heavy ties
        case 2: v[i] = (float)(i % nuniq); break;                         // periodic ties
        case 3: v[i] = (float)((i * 7919) % n); break;                    // permutation
        default: v[i] = (rng() % 11 == 0) ? NAN : (float)(rng() % 9); break;  // NaNs + ties
      }
    }
    bad += !run_case(v, nth);
    done++;
  }
  // Pivot-adversarial inputs: organ-pipe and sawtooth patterns over many sizes.
  for (int n = 4; n <= 1024; n++) {
    std::vector<float> v(n);
    for (int i = 0; i < n; i++) v[i] = (float)std::min(i, n - 1 - i);
    for (int nth : {0, n / 2, n - 1, std::min(7, n - 1)}) { bad += !run_case(v, nth); done++; }
    for (int i = 0; i < n; i++) v[i] = (float)((i & 1) ? i : n - i);
    for (int nth : {0, n / 2, n - 1, std::min(7, n - 1)}) { bad += !run_case(v, nth); done++; }
  }
  // Median-of-three killer (Musser): forces the heap-select fallback.
  for (int n = 8; n <= 1024; n += 8) {
    std::vector<float> v(n);
    int k = n / 2;
    for (int i = 1; i <= k; i++) {
      if (i % 2 == 1) { v[i - 1] = (float)i; v[i] = (float)(k + i); }
      v[k + i - 1] = (float)(2 * i);
    }
    for (int nth : {0, n / 2, n - 1, std::min(7, n - 1)}) { bad += !run_case(v, nth); done++; }
  }
  printf("nth_check cases=%ld mismatches=%ld\n", done, bad);
  return bad ? 1 : 0;
}
