// topk_heap.cuh — per-thread bounded top-k heaps in shared memory.
//
// One thread owns one query row.  Its heap holds the k best (score, index)
// pairs seen so far as a binary heap whose root is the WORST kept pair, so the
// root score is the admission threshold.  Entries of all threads are
// interleaved ([pos][thread], stride = threads) so that threads touching the
// same heap position hit distinct shared-memory banks.
//
// Order ("better"): higher score first; among equal scores the LOWER index
// first — the tie rule of jax.lax.top_k that the reference relies on
// (src/kernels/tiled_topk.py:176, src/model/retrieval.py:301).
#pragma once

#include <cstdint>
#include <climits>

namespace dwa {

constexpr int32_t kSentinelIdx = INT32_MAX;

// true when (as, ai) ranks strictly below (bs, bi)
__device__ __forceinline__ bool topk_worse(float as, int32_t ai, float bs, int32_t bi) {
  return as < bs || (as == bs && ai > bi);
}

struct SmemHeap {
  float* s;      // scores,  element (pos, thread) at s[pos * stride + thread]
  int32_t* i;    // indices, same layout
  int stride;    // number of threads sharing the arrays
  int k;         // heap size (entries per thread)

  __device__ __forceinline__ float& S(int pos, int t) const { return s[pos * stride + t]; }
  __device__ __forceinline__ int32_t& I(int pos, int t) const { return i[pos * stride + t]; }

  __device__ __forceinline__ void init(int t) const {
    for (int p = 0; p < k; ++p) {
      S(p, t) = -INFINITY;
      I(p, t) = kSentinelIdx;
    }
  }

  // Replace the root (worst entry) by (ns, ni), which must rank above it, and
  // restore the heap order by sifting down.
  __device__ __forceinline__ void replace_root(int t, float ns, int32_t ni) const {
    int p = 0;
    while (true) {
      int c = 2 * p + 1;
      if (c >= k) break;
      float cs = S(c, t);
      int32_t ci = I(c, t);
      if (c + 1 < k) {
        const float c2s = S(c + 1, t);
        const int32_t c2i = I(c + 1, t);
        if (topk_worse(c2s, c2i, cs, ci)) {
          c = c + 1;
          cs = c2s;
          ci = c2i;
        }
      }
      if (!topk_worse(cs, ci, ns, ni)) break;
      S(p, t) = cs;
      I(p, t) = ci;
      p = c;
    }
    S(p, t) = ns;
    I(p, t) = ni;
  }

  // Sift entry at position p down within heap prefix [0, n).
  __device__ __forceinline__ void sift_down(int t, int p, int n) const {
    const float ns = S(p, t);
    const int32_t ni = I(p, t);
    while (true) {
      int c = 2 * p + 1;
      if (c >= n) break;
      float cs = S(c, t);
      int32_t ci = I(c, t);
      if (c + 1 < n) {
        const float c2s = S(c + 1, t);
        const int32_t c2i = I(c + 1, t);
        if (topk_worse(c2s, c2i, cs, ci)) {
          c = c + 1;
          cs = c2s;
          ci = c2i;
        }
      }
      if (!topk_worse(cs, ci, ns, ni)) break;
      S(p, t) = cs;
      I(p, t) = ci;
      p = c;
    }
    S(p, t) = ns;
    I(p, t) = ni;
  }

  // In-place heapsort: afterwards position 0 holds the best entry and
  // position k-1 the worst.
  __device__ __forceinline__ void sort_best_first(int t) const {
    for (int end = k - 1; end > 0; --end) {
      const float rs = S(0, t);
      const int32_t ri = I(0, t);
      S(0, t) = S(end, t);
      I(0, t) = I(end, t);
      S(end, t) = rs;
      I(end, t) = ri;
      sift_down(t, 0, end);
    }
  }
};

}  // namespace dwa
