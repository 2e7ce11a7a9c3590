// topk_heap.cuh — per-thread bounded top-k heaps in shared memory.
//
// One thread owns one query row.  Its heap holds the k best (score, index)
// pairs seen so far as a binary heap whose root is the WORST kept pair, so the
// root score is the admission threshold.  An entry is 8 bytes (score bits,
// index), read and written with one 64-bit shared-memory access.  Entries of
// all threads are interleaved ([pos][thread], stride = threads): at any heap
// position the 32 lanes of a warp touch 32 consecutive entries (two
// wavefronts).  Because the stride is a multiple of 32 entries, a lane's bank
// pair depends only on its lane index, so lanes at different positions within
// a half-warp never conflict; lanes 16 apart share a bank pair, and a sift in
// which lanes have diverged can take an extra wavefront for them.
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
  uint32_t base;  // shared-memory address of entry (0, 0)
  int stride;     // number of threads sharing the array
  int k;          // heap size (entries per thread)

  __device__ __forceinline__ uint32_t addr(int pos, int t) const {
    return base + static_cast<uint32_t>(pos * stride + t) * 8u;
  }
  __device__ __forceinline__ void load(int pos, int t, float& s, int32_t& i) const {
    uint32_t a, b;
    asm volatile("ld.shared.v2.u32 {%0, %1}, [%2];" : "=r"(a), "=r"(b) : "r"(addr(pos, t)));
    s = __uint_as_float(a);
    i = static_cast<int32_t>(b);
  }
  __device__ __forceinline__ void store(int pos, int t, float s, int32_t i) const {
    asm volatile("st.shared.v2.u32 [%0], {%1, %2};" ::"r"(addr(pos, t)), "r"(__float_as_uint(s)),
                 "r"(static_cast<uint32_t>(i))
                 : "memory");
  }
  __device__ __forceinline__ float score(int pos, int t) const {
    float s;
    int32_t i;
    load(pos, t, s, i);
    return s;
  }

  __device__ __forceinline__ void init(int t) const {
    for (int p = 0; p < k; ++p) store(p, t, -INFINITY, kSentinelIdx);
  }

  // Sift (ns, ni) down from position p within the heap prefix [0, n).
  __device__ __forceinline__ void sift_from(int t, int p, int n, float ns, int32_t ni) const {
    while (true) {
      int c = 2 * p + 1;
      if (c >= n) break;
      float cs, c2s;
      int32_t ci, c2i;
      load(c, t, cs, ci);
      if (c + 1 < n) {
        load(c + 1, t, c2s, c2i);
        if (topk_worse(c2s, c2i, cs, ci)) {
          c = c + 1;
          cs = c2s;
          ci = c2i;
        }
      }
      if (!topk_worse(cs, ci, ns, ni)) break;
      store(p, t, cs, ci);
      p = c;
    }
    store(p, t, ns, ni);
  }

  // Replace the root (worst entry) by (ns, ni), which must rank above it.
  __device__ __forceinline__ void replace_root(int t, float ns, int32_t ni) const {
    sift_from(t, 0, k, ns, ni);
  }

  // In-place heapsort: afterwards position 0 holds the best entry and
  // position k-1 the worst.
  __device__ __forceinline__ void sort_best_first(int t) const {
    for (int end = k - 1; end > 0; --end) {
      float rs, es;
      int32_t ri, ei;
      load(0, t, rs, ri);
      load(end, t, es, ei);
      store(end, t, rs, ri);
      sift_from(t, 0, end, es, ei);
    }
  }
};

}  // namespace dwa
