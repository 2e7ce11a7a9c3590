// merge_topk.cu — k-way merge of sorted per-split / per-shard top-k lists.
//
// Two callers:
//  * dwa_score_topk: merges the key-range splits of the fused kernel (raw
//    scores s, each list sorted best first), evaluates
//    v(s) = [sigmoid(lambda (s - tau))] * exp(s / T) on the k survivors
//    (tiled_topk.py:172-175) and adds the shard's global index offset
//    (retrieval.py:292-293).
//  * dwa_merge_topk: the cross-shard merge after the all-gather, i.e. the
//    transpose/reshape + top_k + take of _chip_topk (retrieval.py:299-302).
//    Flattening [P, M, k] chip-major and taking top_k with lower position first
//    among ties equals ordering by (v desc, global index asc), because shard p's
//    global indices all precede shard p+1's and each list is already sorted.
//
// One warp per query row, the row's lists staged in shared memory; lane l
// holds the heads of lists l, l+32, l+64, l+96 (up to kMaxSplits lists);
// every output step is a warp arg-max over the lane heads followed by an
// advance of the winning list.  Lists must be sorted best first (score
// descending, lower index first among equal scores).
#include <cuda_runtime.h>

#include <cmath>

#include "dwa_internal.h"
#include "score_params.cuh"
#include "sm100_ptx.cuh"
#include "topk_heap.cuh"

namespace dwa {

namespace {

constexpr int kWarps = 8;           // most rows per block
constexpr int kMaxStagedEntries = 2048;  // n_lists x k_in staged per row (16 KB)

constexpr int kMaxPeers = 16;       // peer lists of the NVLink exchange

struct MergeArgs {
  const float* cv;
  const int32_t* ci;
  // peer mode: list l is peer[l] + row * stride_row, (score bits, index) pairs
  const int32_t* peer[kMaxPeers];
  const int32_t* flags;  // this GPU's flag words, one per peer: >= wait_step when ready
  int wait_step;
  uint64_t wait_ns;      // limit of the wait for the peers' flags
  int* status;
  int64_t stride_list, stride_pos, stride_row;
  int64_t M;
  int64_t idx_offset;
  int n_lists, k_in, k;
  int transform, use_sigmoid;
  float lambda_sharp, tau, T;
  const float* params;  // device {lambda_sharp, tau, T} overriding the values above, or null
  float* out_v;
  int32_t* out_i;
};

__device__ __forceinline__ float fused_score(float s, int use_sigmoid, float lambda_sharp, float tau,
                                             float T) {
  const float e = expf(s / T);
  if (!use_sigmoid) return e;
  const float g = 1.0f / (1.0f + expf(-(lambda_sharp * (s - tau))));
  return g * e;
}

__device__ __forceinline__ int32_t ld_acquire_sys(const int32_t* p) {
  int32_t v;
  asm volatile("ld.acquire.sys.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Keys whose unsigned order is the merge order: a float-order image of the
// score (-0.0 tied with +0.0, as in the float comparison) and the reversed
// index (lower index first among equal scores).
__device__ __forceinline__ uint32_t score_key(float s) {
  uint32_t su = __float_as_uint(s);
  if (su == 0x80000000u) su = 0u;
  return (su & 0x80000000u) ? ~su : (su | 0x80000000u);
}
__device__ __forceinline__ uint32_t index_key(int32_t i) {
  return 0x7FFFFFFFu - static_cast<uint32_t>(i);  // i >= 0 or the sentinel
}

// One warp per query row.  The row's lists are first staged in this warp's
// shared memory (entry p of list l as a (score bits, index) pair at l k_in +
// p), so no global-memory latency sits on the merge's critical path.  Lane l
// owns lists l, l + 32, ... (KSLOTS of them) and keeps their heads and its
// best head in registers.  Each output step is a warp arg-best over the lane
// bests (two hardware max-reductions and a ballot); only the winning lane
// then advances its list and recomputes its best, so a step costs a few
// warp-wide instructions whatever the number of lists.
template <bool kPeer, int KSLOTS>
__global__ void __launch_bounds__(kWarps * 32) merge_sorted_kernel(const MergeArgs a) {
  __shared__ float st_s[kWarps][DWA_MERGE_MAX_K];
  __shared__ int32_t st_i[kWarps][DWA_MERGE_MAX_K];
  extern __shared__ uint4 stage_raw[];
  const int w = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int wpb = blockDim.x >> 5;
  const int64_t row = static_cast<int64_t>(blockIdx.x) * wpb + w;
  if (row >= a.M) return;  // warp-uniform; only warp-level synchronisation below
  ScoreParams sp{a.lambda_sharp, a.tau, a.T};
  if (a.transform) {
    sp = load_score_params(a.params, a.lambda_sharp, a.tau, a.T);
    if (!score_params_ok(sp, a.use_sigmoid)) {
      // device-held scalars the selection cannot honour: no top-k is defined
      if (lane == 0) record_status(a.status, kStatusDeviceCheck);
      for (int j = lane; j < a.k; j += 32) {
        a.out_v[row * a.k + j] = NAN;
        a.out_i[row * a.k + j] = -1;
      }
      return;
    }
  }
  const int n_lists = a.n_lists, k_in = a.k_in;
  int2* stage = reinterpret_cast<int2*>(stage_raw) + static_cast<size_t>(w) * n_lists * k_in;
  if constexpr (kPeer) {
    // Wait (bounded) until every peer has published this step's lists.
    bool ready = true;
    if (lane < n_lists) {
      const uint64_t t0 = globaltimer_ns();
      while (ld_acquire_sys(a.flags + lane) < a.wait_step) {
        if (globaltimer_ns() - t0 > a.wait_ns) {
          ready = false;
          break;
        }
      }
    }
    if (!__all_sync(0xffffffffu, ready)) {
      if (lane == 0) atomicCAS(a.status, 0, kStatusTimeout);
      for (int j = lane; j < a.k; j += 32) {
        a.out_v[row * a.k + j] = -INFINITY;
        a.out_i[row * a.k + j] = -1;
      }
      return;
    }
    // This row's P lists (k (score, index) pairs each, 8k bytes contiguous
    // per list) with 16-byte loads all in flight together, so NVLink latency
    // is paid once per row.  Plain (coherent) loads after the acquire.
    const int words = k_in >> 1;  // 16-byte words per list row (k even)
    uint4* dst = reinterpret_cast<uint4*>(stage);
    for (int t = lane; t < n_lists * words; t += 32) {
      const int l = t / words, c = t - l * words;
      dst[t] = *reinterpret_cast<const uint4*>(a.peer[l] + row * a.stride_row + 4 * c);
    }
  } else {
    // four entries per lane in flight per round
    const int total = n_lists * k_in;
    for (int t0 = 0; t0 < total; t0 += 128) {
      float sv[4];
      int32_t iv[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int t = t0 + 32 * u + lane;
        if (t < total) {
          const int l = t / k_in, p = t - l * k_in;
          const int64_t off = l * a.stride_list + row * a.stride_row + p * a.stride_pos;
          sv[u] = __ldg(a.cv + off);
          iv[u] = __ldg(a.ci + off);
        }
      }
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int t = t0 + 32 * u + lane;
        if (t < total) stage[t] = make_int2(__float_as_int(sv[u]), iv[u]);
      }
    }
  }
  __syncwarp();

  int pos[KSLOTS] = {};
  float hs[KSLOTS];
  int32_t hi[KSLOTS];
  auto load_head = [&](int u) {
    const int l = lane + 32 * u;
    if (l < n_lists && pos[u] < k_in) {
      const int2 e = stage[l * k_in + pos[u]];
      hs[u] = __int_as_float(e.x);
      hi[u] = e.y;
    } else {
      hs[u] = -INFINITY;
      hi[u] = kSentinelIdx;
    }
  };
  float bs;
  int32_t bi;
  int bu;
  uint32_t skey, ikey;
  auto pick_best = [&]() {
    bs = hs[0];
    bi = hi[0];
    bu = 0;
#pragma unroll
    for (int u = 1; u < KSLOTS; ++u)
      if (topk_worse(bs, bi, hs[u], hi[u])) {
        bs = hs[u];
        bi = hi[u];
        bu = u;
      }
    skey = score_key(bs);
    ikey = index_key(bi);
  };
#pragma unroll
  for (int u = 0; u < KSLOTS; ++u) {
    pos[u] = 0;
    load_head(u);
  }
  pick_best();

  for (int j = 0; j < a.k; ++j) {
    const uint32_t smax = __reduce_max_sync(0xffffffffu, skey);
    const uint32_t imax = __reduce_max_sync(0xffffffffu, skey == smax ? ikey : 0u);
    const uint32_t win = __ballot_sync(0xffffffffu, skey == smax && ikey == imax);
    if (lane == __ffs(win) - 1) {
      st_s[w][j] = bs;
      st_i[w][j] = bi;
#pragma unroll
      for (int u = 0; u < KSLOTS; ++u)
        if (u == bu) {
          ++pos[u];
          load_head(u);
        }
      pick_best();
    }
  }
  __syncwarp();

  if (a.transform) {
    for (int j = lane; j < a.k; j += 32)
      st_s[w][j] = fused_score(st_s[w][j], a.use_sigmoid, sp.lambda_sharp, sp.tau, sp.T);
    __syncwarp();
    // v is non-decreasing in s, so the list is ordered by v already; entries
    // whose v became equal must still be ordered by lower index first.
    if (lane == 0) {
      for (int p = 1; p < a.k; ++p) {
        const float vs = st_s[w][p];
        const int32_t vi = st_i[w][p];
        int q = p - 1;
        while (q >= 0 && topk_worse(st_s[w][q], st_i[w][q], vs, vi)) {
          st_s[w][q + 1] = st_s[w][q];
          st_i[w][q + 1] = st_i[w][q];
          --q;
        }
        st_s[w][q + 1] = vs;
        st_i[w][q + 1] = vi;
      }
    }
    __syncwarp();
  }

  float* ov = a.out_v + row * a.k;
  int32_t* oi = a.out_i + row * a.k;
  for (int j = lane; j < a.k; j += 32) {
    const int32_t ix = st_i[w][j];
    ov[j] = st_s[w][j];
    oi[j] = ix == kSentinelIdx ? -1 : static_cast<int32_t>(ix + a.idx_offset);
  }
}

// Lists too long to stage (n_lists k_in > kMaxStagedEntries): each lane keeps
// a cursor with the next kCache entries of each of its lists in registers
// and reloads them from global memory as the list advances.
constexpr int kSlots = kMaxSplits / 32;  // lists per lane
constexpr int kCache = 4;                // entries cached per list

template <typename V>
__device__ __forceinline__ V pick4(const V (&c)[kCache], int j) {
  const V lo = (j & 1) ? c[1] : c[0];
  const V hi = (j & 1) ? c[3] : c[2];
  return (j & 2) ? hi : lo;
}

struct ListCursor {
  float s[kCache];
  int32_t i[kCache];
  int base;  // position of s[0] in the list
  int off;   // current head = entry `off` of the cache
};

__device__ __forceinline__ void load_block(ListCursor& L, const float* vp, const int32_t* ip,
                                           int64_t stride_pos, int k_in) {
#pragma unroll
  for (int e = 0; e < kCache; ++e) {
    const int p = L.base + e;
    const bool in = p < k_in;
    L.s[e] = in ? __ldg(vp + p * stride_pos) : -INFINITY;
    L.i[e] = in ? __ldg(ip + p * stride_pos) : kSentinelIdx;
  }
}

__global__ void __launch_bounds__(kWarps * 32) merge_cursor_kernel(const MergeArgs a) {
  __shared__ float st_s[kWarps][DWA_MERGE_MAX_K];
  __shared__ int32_t st_i[kWarps][DWA_MERGE_MAX_K];
  const int w = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int64_t row = static_cast<int64_t>(blockIdx.x) * kWarps + w;
  if (row >= a.M) return;  // warp-uniform; only warp-level synchronisation below
  ScoreParams sp{a.lambda_sharp, a.tau, a.T};
  if (a.transform) {
    sp = load_score_params(a.params, a.lambda_sharp, a.tau, a.T);
    if (!score_params_ok(sp, a.use_sigmoid)) {
      // device-held scalars the selection cannot honour: no top-k is defined
      if (lane == 0) record_status(a.status, kStatusDeviceCheck);
      for (int j = lane; j < a.k; j += 32) {
        a.out_v[row * a.k + j] = NAN;
        a.out_i[row * a.k + j] = -1;
      }
      return;
    }
  }
  ListCursor cur[kSlots];
  const float* vbase[kSlots];
  const int32_t* ibase[kSlots];
#pragma unroll
  for (int u = 0; u < kSlots; ++u) {
    const int l = lane + 32 * u;
    cur[u].base = 0;
    cur[u].off = 0;
    if (l < a.n_lists) {
      vbase[u] = a.cv + l * a.stride_list + row * a.stride_row;
      ibase[u] = a.ci + l * a.stride_list + row * a.stride_row;
      load_block(cur[u], vbase[u], ibase[u], a.stride_pos, a.k_in);
    } else {
      vbase[u] = nullptr;
      ibase[u] = nullptr;
#pragma unroll
      for (int e = 0; e < kCache; ++e) {
        cur[u].s[e] = -INFINITY;
        cur[u].i[e] = kSentinelIdx;
      }
    }
  }

  for (int j = 0; j < a.k; ++j) {
    // best head of this lane's lists
    float bs = -INFINITY;
    int32_t bi = kSentinelIdx;
    int bu = 0;
#pragma unroll
    for (int u = 0; u < kSlots; ++u) {
      const float hs = pick4(cur[u].s, cur[u].off);
      const int32_t hi = pick4(cur[u].i, cur[u].off);
      if (topk_worse(bs, bi, hs, hi)) {
        bs = hs;
        bi = hi;
        bu = u;
      }
    }
    // Warp arg-best with two hardware max-reductions: first over an unsigned
    // image of the score that preserves float order, then over the reversed
    // index among the lanes holding that score (lower index wins ties).
    uint32_t su = __float_as_uint(bs);
    if (su == 0x80000000u) su = 0u;  // -0.0 ties with +0.0, as in the float comparison
    const uint32_t skey = (su & 0x80000000u) ? ~su : (su | 0x80000000u);
    const uint32_t ikey = 0x7FFFFFFFu - static_cast<uint32_t>(bi);  // bi >= 0 or the sentinel
    const uint32_t smax = __reduce_max_sync(0xffffffffu, skey);
    const uint32_t imax = __reduce_max_sync(0xffffffffu, skey == smax ? ikey : 0u);
    const uint32_t win = __ballot_sync(0xffffffffu, skey == smax && ikey == imax);
    const int wl = __ffs(win) - 1;
    const float ws = __shfl_sync(0xffffffffu, bs, wl);
    const int32_t wi = __shfl_sync(0xffffffffu, bi, wl);
    if (lane == 0) {
      st_s[w][j] = ws;
      st_i[w][j] = wi;
    }
    if (lane == wl) {
#pragma unroll
      for (int u = 0; u < kSlots; ++u) {
        if (u == bu) {
          if (++cur[u].off == kCache) {
            cur[u].off = 0;
            cur[u].base += kCache;
            if (vbase[u] != nullptr) {
              load_block(cur[u], vbase[u], ibase[u], a.stride_pos, a.k_in);
            }
          }
        }
      }
    }
  }
  __syncwarp();

  if (a.transform) {
    for (int j = lane; j < a.k; j += 32)
      st_s[w][j] = fused_score(st_s[w][j], a.use_sigmoid, sp.lambda_sharp, sp.tau, sp.T);
    __syncwarp();
    // v is non-decreasing in s, so the list is ordered by v already; entries
    // whose v became equal must still be ordered by lower index first.
    if (lane == 0) {
      for (int p = 1; p < a.k; ++p) {
        const float vs = st_s[w][p];
        const int32_t vi = st_i[w][p];
        int q = p - 1;
        while (q >= 0 && topk_worse(st_s[w][q], st_i[w][q], vs, vi)) {
          st_s[w][q + 1] = st_s[w][q];
          st_i[w][q + 1] = st_i[w][q];
          --q;
        }
        st_s[w][q + 1] = vs;
        st_i[w][q + 1] = vi;
      }
    }
    __syncwarp();
  }

  float* ov = a.out_v + row * a.k;
  int32_t* oi = a.out_i + row * a.k;
  for (int j = lane; j < a.k; j += 32) {
    const int32_t ix = st_i[w][j];
    ov[j] = st_s[w][j];
    oi[j] = ix == kSentinelIdx ? -1 : static_cast<int32_t>(ix + a.idx_offset);
  }
}

// Rows per block for the staged kernel: up to kWarps, within kStageBudget
// bytes of staged lists per block, so that three blocks fit on an SM.
constexpr int64_t kStageBudget = 64 * 1024;

int merge_warps_per_block(int n_lists, int k_in) {
  const int64_t per_warp = static_cast<int64_t>(n_lists) * k_in * 8;
  const int64_t w = kStageBudget / per_warp;
  return static_cast<int>(w < 1 ? 1 : w > kWarps ? kWarps : w);
}

template <bool kPeer, int KSLOTS>
cudaError_t launch_merge_kernel(const MergeArgs& a, cudaStream_t stream) {
  const int wpb = merge_warps_per_block(a.n_lists, a.k_in);
  const size_t smem = static_cast<size_t>(wpb) * a.n_lists * a.k_in * 8;
  if (smem > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(merge_sorted_kernel<kPeer, KSLOTS>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(smem));
    if (e != cudaSuccess) return e;
  }
  const int64_t blocks = (a.M + wpb - 1) / wpb;
  merge_sorted_kernel<kPeer, KSLOTS>
      <<<static_cast<unsigned>(blocks), wpb * 32, smem, stream>>>(a);
  return cudaGetLastError();
}

}  // namespace

cudaError_t launch_merge_topk(const float* cand_vals, const int32_t* cand_idx, int n_lists,
                              int k_in, int64_t stride_list, int64_t stride_pos,
                              int64_t stride_row, int64_t M, int k, int transform,
                              float lambda_sharp, float tau, float T, int use_sigmoid,
                              int64_t idx_offset, float* out_vals, int32_t* out_idx,
                              cudaStream_t stream, const float* params, int* status) {
  if (M <= 0) return cudaSuccess;
  if (n_lists < 1 || n_lists > kMaxSplits || k < 1 || k > DWA_MERGE_MAX_K)
    return cudaErrorInvalidValue;
  MergeArgs a{};
  a.cv = cand_vals;
  a.ci = cand_idx;
  a.stride_list = stride_list;
  a.stride_pos = stride_pos;
  a.stride_row = stride_row;
  a.M = M;
  a.idx_offset = idx_offset;
  a.n_lists = n_lists;
  a.k_in = k_in;
  a.k = k;
  a.transform = transform;
  a.use_sigmoid = use_sigmoid;
  a.lambda_sharp = lambda_sharp;
  a.tau = tau;
  a.T = T;
  a.params = params;
  a.status = status;
  a.out_v = out_vals;
  a.out_i = out_idx;
  if (static_cast<int64_t>(n_lists) * k_in > kMaxStagedEntries) {
    const int64_t blocks = (M + kWarps - 1) / kWarps;
    merge_cursor_kernel<<<static_cast<unsigned>(blocks), kWarps * 32, 0, stream>>>(a);
    return cudaGetLastError();
  }
  if (n_lists <= 32) return launch_merge_kernel<false, 1>(a, stream);
  if (n_lists <= 64) return launch_merge_kernel<false, 2>(a, stream);
  return launch_merge_kernel<false, 4>(a, stream);
}

namespace {
__device__ __forceinline__ void st_release_sys(int32_t* p, int32_t v) {
  asm volatile("st.release.sys.global.b32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

struct SignalArgs {
  int32_t* flag_base[kMaxPeers];
  int n, my_rank, value;
};

// One thread: everything this GPU's earlier kernels on the stream wrote is made
// visible system-wide, then flag[my_rank] = value on every peer (release).
__global__ void peer_signal_kernel(const SignalArgs a) {
  __threadfence_system();
  for (int p = 0; p < a.n; ++p) st_release_sys(a.flag_base[p] + a.my_rank, a.value);
}
}  // namespace

int max_peers() { return kMaxPeers; }

cudaError_t launch_peer_signal(int32_t* const* flag_bases, int n, int my_rank, int value,
                               cudaStream_t stream) {
  if (n < 1 || n > kMaxPeers || my_rank < 0 || my_rank >= n) return cudaErrorInvalidValue;
  SignalArgs a{};
  for (int p = 0; p < n; ++p) a.flag_base[p] = flag_bases[p];
  a.n = n;
  a.my_rank = my_rank;
  a.value = value;
  peer_signal_kernel<<<1, 1, 0, stream>>>(a);
  return cudaGetLastError();
}

cudaError_t launch_merge_topk_peers(const int32_t* const* packed, int n, int64_t M, int k,
                                    const int32_t* flags, int step, uint64_t wait_ns,
                                    float* out_vals, int32_t* out_idx, int* status,
                                    cudaStream_t stream) {
  if (M <= 0) return cudaSuccess;
  if (n < 1 || n > kMaxPeers || k < 1 || k > DWA_MERGE_MAX_K) return cudaErrorInvalidValue;
  MergeArgs a{};
  for (int p = 0; p < n; ++p) a.peer[p] = packed[p];
  a.flags = flags;
  a.wait_step = step;
  a.wait_ns = wait_ns;
  a.status = status;
  a.stride_list = 0;
  a.stride_pos = 2;
  a.stride_row = 2 * static_cast<int64_t>(k);
  a.M = M;
  a.idx_offset = 0;
  a.n_lists = n;
  a.k_in = k;
  a.k = k;
  a.transform = 0;
  a.out_v = out_vals;
  a.out_i = out_idx;
  if (k % 2 != 0) return cudaErrorInvalidValue;  // 16-byte staging words
  static_assert(kMaxPeers <= 32, "one list per lane");
  return launch_merge_kernel<true, 1>(a, stream);
}

}  // namespace dwa
