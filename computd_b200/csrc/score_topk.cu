// score_topk.cu — fused query x pool-key score GEMM with a streaming top-k
// epilogue, for sm_100a (B200).
//
// Replaces the executed score + top-k of the reference,
// tiled_topk_fallback (src/kernels/tiled_topk.py:160-176):
//     sims = jnp.dot(queries, keys.T); score = gate(sims) * exp(sims / T);
//     lax.top_k(score, k_max)
// which materialises the whole [M, N] score matrix before a sort-based top-k.
// Here each [256 x 256] score tile lives only in tensor memory (TMEM); the
// epilogue keeps the k best (score, index) per query row in registers (a
// sorted list, k <= 64; for k > 64 the best 64 in registers and the rest in
// a shared-memory heap), so the full score matrix never reaches HBM.
//
// Launch unit = a CTA pair (cluster of 2 on neighbouring SMs) running
// tcgen05.mma.cta_group::2: one 256 x 256 x 16 MMA covers 256 query rows (128
// per CTA) against 256 keys (128 staged per CTA), so each SM stages only half
// of the key tile and half of the pair's query rows per k-block.
// Each CTA = 6 warps, warp-specialised:
//   warp 0     TMA producer: its 128 query rows x 64 and its 128 keys x 64
//              (bf16, 128-byte swizzle) per k-block into a STAGES-deep ring;
//              the byte counts complete on the leader CTA's "full" barrier
//   warp 1     TMEM allocator (both CTAs) + UMMA issuer (leader CTA only):
//              fp32 accumulators double-buffered in TMEM (2 x 256 columns)
//   warps 2-5  epilogue: warp w reads TMEM lanes 32*(w%4).. with tcgen05.ld;
//              thread = one query row; the list's k-th entry = admission
//              threshold; candidates are buffered per lane and inserted in
//              warp-wide passes (k <= 32: warps 2-9, two warpgroups each
//              scanning half of every tile's columns)
//
// Work unit = (pair query tile, contiguous range of key tiles).  Units are
// ordered split-major so the pairs resident at one time sweep the same few
// key ranges: each key tile is fetched from HBM about once and re-served
// from L2 to every query tile.  When the queries are too large for L2 the
// units go in groups of a few query tiles x all splits instead, so that the
// resident query tiles stay in L2 as well.  Each unit leaves one sorted partial top-k list
// per row in the workspace; merge_topk.cu merges the splits, applies the
// gate/exp and adds the global index offset.
#include <cuda.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <atomic>
#include <cmath>
#include <mutex>

#include "dwa_internal.h"
#include "score_params.cuh"
#include "sm100_ptx.cuh"
#include "topk_heap.cuh"

namespace dwa {

namespace {

// 2 non-epilogue warps (TMA, MMA) + NWG epilogue warpgroups of 4 warps.
constexpr int threads_for(int nwg) { return 64 + 128 * nwg; }
constexpr int kMaxDynSmem = 232448;  // 227 KB opt-in limit on sm_100
constexpr int kPairRows = 2 * kTileM;      // 256 query rows per CTA pair
constexpr int64_t kSplitListMinWork = int64_t(1) << 20;  // key tiles x d per unit, see plan_score_topk
constexpr int kKeysPerCta = kTileN / 2;    // 128 keys of each 256-key tile per CTA

template <int KCAP, int NWG>
struct TopkCfg {
  static constexpr int kStageA = kTileM * kTileK * 2;       // 16 KB: this CTA's query rows
  static constexpr int kStageB = kKeysPerCta * kTileK * 2;  // 16 KB: this CTA's half of the keys
  static constexpr int kStageBytes = kStageA + kStageB;
  // k <= 64 keeps its lists in registers; the two-level list (KCAP 128) keeps
  // ranks 65..128 in a shared-memory heap per row per warpgroup, the whole-heap
  // variant (KCAP 129) all 128
  static constexpr int kHeapBytes = KCAP == 129   ? 128 * kTileM * 8 * NWG
                                    : KCAP > 64 ? (KCAP - 64) * kTileM * 8 * NWG
                                                : 0;
  static constexpr int kBarBytes = 256;
  static constexpr int kStagesFit = (kMaxDynSmem - 1024 - kHeapBytes - kBarBytes) / kStageBytes;
  static constexpr int kStages = kStagesFit > 7 ? 7 : kStagesFit;
  static constexpr int kSmemBytes = 1024 + kStages * kStageBytes + kHeapBytes + kBarBytes;
  static_assert(kStages >= 2, "pipeline needs at least two stages");
  static_assert(kSmemBytes <= kMaxDynSmem, "shared memory budget exceeded");
};

// v[j] for a runtime j without indexing the register array dynamically (which
// would spill it to local memory): a 5-level select tree, 31 selects.
__device__ __forceinline__ float pick32(const float (&v)[32], int j) {
  float a[16], b[8], c[4], d[2];
#pragma unroll
  for (int i = 0; i < 16; ++i) a[i] = (j & 1) ? v[2 * i + 1] : v[2 * i];
#pragma unroll
  for (int i = 0; i < 8; ++i) b[i] = (j & 2) ? a[2 * i + 1] : a[2 * i];
#pragma unroll
  for (int i = 0; i < 4; ++i) c[i] = (j & 4) ? b[2 * i + 1] : b[2 * i];
#pragma unroll
  for (int i = 0; i < 2; ++i) d[i] = (j & 8) ? c[2 * i + 1] : c[2 * i];
  return (j & 16) ? d[1] : d[0];
}

// Per-row top-k of one unit held in registers, sorted best first, for
// k <= KCAP <= 64.  Slots [0, KCAP - k) are pinned at +inf so the admission
// threshold is always the static slot KCAP - 1.  Insertion is a branch-free
// network: every slot takes its own value, the new entry or its upper
// neighbour's old value, so all slots update in parallel from old values and
// nothing touches memory (a shared-memory heap competes with the tensor core
// for shared-memory bandwidth and measured ~900 cycles per insert).
template <int KCAP>
struct RegTopK {
  float s[KCAP];
  int32_t i[KCAP];
  __device__ __forceinline__ void init(int k) {
#pragma unroll
    for (int p = 0; p < KCAP; ++p) {
      s[p] = p < KCAP - k ? INFINITY : -INFINITY;
      i[p] = kSentinelIdx;
    }
  }
  __device__ __forceinline__ float worst() const { return s[KCAP - 1]; }
  // (x, xi) must rank above the worst entry; inside a unit indices only
  // grow, so "above" is a strict score comparison and equal scores keep the
  // older (lower) index first.
  __device__ __forceinline__ void insert(float x, int32_t xi) {
    bool hi = true;
#pragma unroll
    for (int p = KCAP - 1; p >= 1; --p) {
      const bool lo = x > s[p - 1];
      const float ns = lo ? s[p - 1] : (hi ? x : s[p]);
      const int32_t ni = lo ? i[p - 1] : (hi ? xi : i[p]);
      s[p] = ns;
      i[p] = ni;
      hi = lo;
    }
    if (hi) {
      s[0] = x;
      i[0] = xi;
    }
  }
  __device__ __forceinline__ void write_out(float* vs, int32_t* is, int k) const {
#pragma unroll
    for (int p = 0; p < KCAP; ++p)
      if (p >= KCAP - k) {
        vs[p - (KCAP - k)] = s[p];
        is[p - (KCAP - k)] = i[p];
      }
  }
};

// Per-row top-k for 64 < k <= 128 (KCAP = 128), in two levels: the best 64
// in a register list (RegTopK<64>, the k <= 64 machinery) and ranks 65..k in a
// min-heap of k - 64 entries in shared memory, whose root (the k-th best) is
// the admission threshold.  Everything in the register list ranks above
// everything in the heap: an entry enters the heap either because it does
// not beat the list's 64th entry, or because a better entry pushed it out of
// the list.  Keeping the best half in registers halves the shared memory the
// lists take (64 KB per CTA instead of 128 KB), which buys the operand ring
// two more stages.
struct SplitTopK {
  RegTopK<64> upper;
  SmemHeap lower;  // k - 64 entries per row
  int row;
  __device__ __forceinline__ void init(int) {
    upper.init(64);
    lower.init(row);
  }
  __device__ __forceinline__ float worst() const { return lower.score(0, row); }
  // (x, xi) must rank above the heap root (the caller's admission cut).
  __device__ __forceinline__ void insert(float x, int32_t xi) {
    if (x > upper.worst()) {
      // x joins the register list; its old 64th entry drops to rank 65
      const float es = upper.s[63];
      const int32_t ei = upper.i[63];
      upper.insert(x, xi);
      float rs;
      int32_t ri;
      lower.load(0, row, rs, ri);
      if (topk_worse(rs, ri, es, ei)) lower.replace_root(row, es, ei);
    } else {
      lower.replace_root(row, x, xi);
    }
  }
  __device__ __forceinline__ void write_out(float* vs, int32_t* is, int k) const {
    upper.write_out(vs, is, 64);
    lower.sort_best_first(row);
    for (int p = 0; p < k - 64; ++p) {
      float hs;
      int32_t hi;
      lower.load(p, row, hs, hi);
      vs[64 + p] = hs;
      is[64 + p] = hi;
    }
  }
};

// Per-row top-k for 64 < k <= 128 wholly in a shared-memory heap (128 KB per
// CTA, three ring stages).  Each insert is one sift-down, cheaper than the
// two-level list's register network plus heap step, so it wins when a unit's
// key range is short and its lists spend much of it filling up.
struct HeapTopK {
  SmemHeap heap;
  int row;
  __device__ __forceinline__ void init(int) { heap.init(row); }
  __device__ __forceinline__ float worst() const { return heap.score(0, row); }
  __device__ __forceinline__ void insert(float x, int32_t xi) { heap.replace_root(row, x, xi); }
  __device__ __forceinline__ void write_out(float* vs, int32_t* is, int k) const {
    heap.sort_best_first(row);
    for (int p = 0; p < k; ++p) {
      float hs;
      int32_t hi;
      heap.load(p, row, hs, hi);
      vs[p] = hs;
      is[p] = hi;
    }
  }
};

// KCAP values: 16, 32, 64 (register lists), 128 (two-level list) and
// kCapHeap128 (k in (64, 128] in a whole shared-memory heap).
constexpr int kCapHeap128 = 129;

template <int KCAP>
struct TopKFor {
  using type = RegTopK<KCAP>;
};
template <>
struct TopKFor<128> {
  using type = SplitTopK;
};
template <>
struct TopKFor<kCapHeap128> {
  using type = HeapTopK;
};

// Shared admission bounds, kBoundSlots int32 per query row (one 64-byte line):
//   [0]      P = 1: the best k-th score of any list of the row
//   [1, 3)   P = 2: slot c holds the best (k/2)-th score of the lists l = c mod 2
//   [3, 7)   P = 4: slot c holds the best (k/4)-th score of the lists l = c mod 4
//   [7, 15)  P = 8: slot c holds the best (k/8)-th score of the lists l = c mod 8
// Lists of distinct classes cover disjoint key sets, so for each P the P
// class maxima name P disjoint lists holding k/P scores each that are >= the
// smallest of them: min over the P slots is a lower bound of the row's k-th
// best.  The bound taken is the largest of the four.
constexpr int kBoundSlots = 16;

// Order-preserving map float -> int32 (signed integer order = float order),
// so atomicMax on the image maximises the float.
__device__ __forceinline__ int32_t ordered_int(float f) {
  const int32_t i = __float_as_int(f);
  return i >= 0 ? i : (i ^ 0x7FFFFFFF);
}
__device__ __forceinline__ float ordered_float(int32_t i) {
  return __int_as_float(i >= 0 ? i : (i ^ 0x7FFFFFFF));
}
// Largest float strictly below x: "s >= x" <=> "s > float_below(x)"; -inf stays -inf.
__device__ __forceinline__ float float_below(float x) {
  if (x == -INFINITY) return -INFINITY;
  if (x == 0.0f) return -1.40129846e-45f;
  const int32_t i = __float_as_int(x);
  return __int_as_float(x > 0.0f ? i - 1 : i + 1);
}

struct TopkKernelArgs {
  int64_t N;         // keys in this shard
  int64_t n_kt;      // 256-key tiles
  int64_t m_pad;     // padded query rows (row count of the partial lists)
  int num_kb;        // 64-wide k-blocks along d
  int k;             // kept per row
  int n_qt;          // 256-row pair query tiles
  int n_split;       // key-range splits
  int group;         // query tiles per unit group, 0 = split-major over all query tiles
  int32_t* row_bound;  // [m_pad][kBoundSlots] shared admission bounds per query row (ordered_int images)
  float* ws_vals;    // [n_split * NWG][m_pad][k] raw scores, sorted best first
  int32_t* ws_idx;   // [n_split * NWG][m_pad][k] local key indices
  int* status;       // device status word
  // Per-sequence mean of the fused scores (the kernel's AUX variant only):
  // aux[g * ld_aux + n] += v(s[m, n]) / group_rows for the rows m of group
  // g = m / group_rows, every key n of the shard.
  int64_t M;           // real query rows (rows beyond are padding)
  float* aux;
  int64_t ld_aux;
  int64_t group_rows;
  const float* params;  // device {lambda_sharp, tau, T} or null (then the host values)
  float lambda_sharp, tau, T;
  int use_sigmoid;
};

// Column sums of one 32-column chunk over the warp's 32 rows, in place: each
// halving step keeps half of the values and adds the partner lane's copy of
// them, so after five steps lane l holds the sum over all lanes of value l.
__device__ __forceinline__ float warp_column_sum32(float (&f)[32], int lane) {
#pragma unroll
  for (int step = 0; step < 5; ++step) {
    const int o = 16 >> step;
    const int H = 16 >> step;
    const bool up = (lane & o) != 0;
#pragma unroll
    for (int i = 0; i < H; ++i) {
      const float send = up ? f[i] : f[i + H];
      const float keep = up ? f[i + H] : f[i];
      f[i] = keep + __shfl_xor_sync(0xffffffffu, send, o);
    }
  }
  return f[0];
}

template <int KCAP, int NWG, bool AUX>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(threads_for(NWG), 1)
    score_topk_kernel(const __grid_constant__ CUtensorMap tmap_q,
                      const __grid_constant__ CUtensorMap tmap_k, const TopkKernelArgs a) {
  using C = TopkCfg<KCAP, NWG>;
  constexpr int S = C::kStages;

  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  const uint32_t base = (raw_addr + 1023u) & ~1023u;
  uint8_t* smem = smem_raw + (base - raw_addr);

  const uint32_t sA0 = base;               // stage s query rows at sA0 + s * kStageBytes
  const uint32_t sB0 = base + C::kStageA;  // stage s keys       at sB0 + s * kStageBytes
  // heaps: warpgroup g's 8-byte entries at heap0 + g * KCAP * 128 * 8
  const uint32_t heap0 = base + S * C::kStageBytes;
  uint8_t* bar_area = smem + S * C::kStageBytes + C::kHeapBytes;
  const uint32_t bar0 = smem_u32(bar_area);
  auto full_bar = [&](int s) { return bar0 + 8u * s; };             // leader: TMA bytes, both CTAs
  auto empty_bar = [&](int s) { return bar0 + 8u * (S + s); };      // each: stage free again
  auto tfull_bar = [&](int acc) { return bar0 + 8u * (2 * S + acc); };       // each: acc ready
  auto tempty_bar = [&](int acc) { return bar0 + 8u * (2 * S + 2 + acc); };  // leader: all epilogue warps
  const uint32_t drain_bar = bar0 + 8u * (2 * S + 4);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bar_area + 8 * (2 * S + 5));
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  int* n_issued = reinterpret_cast<int*>(tmem_slot + 2);
  int* n_consumed = reinterpret_cast<int*>(tmem_slot + 3);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t cta = cluster_cta_rank();  // 0 = leader (issues the MMAs), 1 = peer
  const bool leader = cta == 0;

  const int pair = blockIdx.x >> 1;
  int qt, split;
  if (a.group > 0) {
    // groups of `group` query tiles, each group split-major over all splits
    const int per_group = a.group * a.n_split;
    const int g = pair / per_group;
    const int r = pair - g * per_group;
    const int q0 = g * a.group;
    const int gsize = min(a.group, a.n_qt - q0);
    split = r / gsize;
    qt = q0 + (r - split * gsize);
  } else {
    qt = pair % a.n_qt;
    split = pair / a.n_qt;
  }
  const int64_t kt_begin = static_cast<int64_t>(split) * a.n_kt / a.n_split;
  const int64_t kt_end = static_cast<int64_t>(split + 1) * a.n_kt / a.n_split;
  const int n_tiles = static_cast<int>(kt_end - kt_begin);
  const int32_t row0 = qt * kPairRows + static_cast<int32_t>(cta) * kTileM;  // this CTA's rows

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(full_bar(s), 1);
      mbar_init(empty_bar(s), 1);
    }
    for (int acc = 0; acc < 2; ++acc) {
      mbar_init(tfull_bar(acc), 1);
      mbar_init(tempty_bar(acc), 2 * 4 * NWG);  // every epilogue warp of both CTAs
    }
    mbar_init(drain_bar, 1);
    *abort_flag = 0;
    *n_issued = 0;
    *n_consumed = 0;
    fence_mbar_init();
    tma_prefetch_desc(&tmap_q);
    tma_prefetch_desc(&tmap_k);
  }
  if (warp == 1) {
    tmem_alloc_pair(smem_u32(tmem_slot), 2 * kTileN);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  cluster_sync();  // barriers of both CTAs initialised, TMEM allocated in both
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      const uint64_t pol_q = l2_policy_evict_last();
      const uint64_t pol_k = l2_policy_evict_normal();
      int it = 0;
      bool ok = true;
      for (int t = 0; t < n_tiles && ok; ++t) {
        const int32_t krow =
            static_cast<int32_t>((kt_begin + t) * kTileN) + static_cast<int32_t>(cta) * kKeysPerCta;
        for (int kb = 0; kb < a.num_kb; ++kb, ++it) {
          const int s = it % S;
          const uint32_t r = static_cast<uint32_t>(it / S);
          if (!mbar_wait(empty_bar(s), (r & 1u) ^ 1u, a.status, abort_flag)) {
            ok = false;
            break;
          }
          // The leader expects the bytes of both CTAs on its own barrier.
          if (leader) mbar_arrive_expect_tx(full_bar(s), 2 * C::kStageBytes);
          const uint32_t lead_full = map_to_cta(full_bar(s), 0);
          tma_load_2d_pair(sA0 + s * C::kStageBytes, &tmap_q, lead_full, kb * kTileK, row0, pol_q);
          tma_load_2d_pair(sB0 + s * C::kStageBytes, &tmap_k, lead_full, kb * kTileK, krow, pol_k);
        }
      }
      *n_issued = it;
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ UMMA issuer
    if (leader && lane == 0) {
      constexpr uint32_t idesc = umma_idesc_bf16_f32(kPairRows, kTileN);
      int it = 0;
      bool ok = true;
      for (int t = 0; t < n_tiles && ok; ++t) {
        const int acc = t & 1;
        const uint32_t use = static_cast<uint32_t>(t >> 1);
        if (!mbar_wait_cluster(tempty_bar(acc), (use & 1u) ^ 1u, a.status, abort_flag)) break;
        tc_fence_after();
        const uint32_t tmem_d = tmem_base + static_cast<uint32_t>(acc * kTileN);
        for (int kb = 0; kb < a.num_kb; ++kb, ++it) {
          const int s = it % S;
          const uint32_t r = static_cast<uint32_t>(it / S);
          if (!mbar_wait_cluster(full_bar(s), r & 1u, a.status, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t ad = sw128_kmajor_desc(sA0 + s * C::kStageBytes);
          const uint64_t bd = sw128_kmajor_desc(sB0 + s * C::kStageBytes);
#pragma unroll
          for (int kk = 0; kk < kTileK / 16; ++kk) {
            // +32 bytes along K inside the swizzled 128-byte row = +2 in the address field
            umma_bf16_ss_pair(tmem_d, ad + 2u * kk, bd + 2u * kk, idesc, (kb | kk) != 0 ? 1u : 0u);
          }
          umma_commit_pair_all(empty_bar(s), 0x3);  // frees stage s in both CTAs
        }
        if (ok) umma_commit_pair_all(tfull_bar(acc), 0x3);
      }
      *n_consumed = it;
      // Every MMA must finish (it reads both CTAs' shared memory and writes
      // both TMEMs) before either CTA releases them.
      umma_commit_pair_local(drain_bar);
      mbar_wait(drain_bar, 0u, a.status, nullptr);
    }
  } else {
    // ------------------------------------------------------------ epilogue
    // Admission: a score enters this unit's list when it beats the list's k-th entry
    // (theta_loc; strict, since indices only grow inside a unit) AND is not
    // below the row's shared bound.  The bound is the best k-th score any unit
    // of the same query row has published; the union's k-th best is at least
    // that, so lower scores can never reach the final top-k.  Scores equal to
    // the bound stay admissible (they may win an index tie).
    // With two warpgroups, warpgroup g scans columns [128 g, 128 g + 128) of
    // every tile (keys tile * 256 + 128 g + j, so each list still sees its
    // keys in increasing order).  Both scan the same accumulator at once and
    // release it together, so a tile costs max(MMA, epilogue / 2).  (Taking
    // alternate tiles instead costs (MMA + epilogue) / 2: with two TMEM
    // buffers the MMA of tile t + 2 waits for tile t's release, so the second
    // warpgroup would only overlap the MMA, never the other warpgroup.)
    const int g = (warp - 2) >> 2;     // epilogue warpgroup
    constexpr int kColsPerWg = kTileN / NWG;
    const int ew = warp & 3;           // TMEM lane quarter this warp may access
    const int row = ew * 32 + lane;    // query row within this CTA's 128
    typename TopKFor<KCAP>::type topk;
    if constexpr (KCAP == kCapHeap128) {
      topk.heap = SmemHeap{heap0 + static_cast<uint32_t>(g * 128 * kTileM * 8), kTileM, a.k};
      topk.row = row;
    } else if constexpr (KCAP > 64) {
      topk.lower = SmemHeap{heap0 + static_cast<uint32_t>(g * (KCAP - 64) * kTileM * 8), kTileM,
                            a.k - 64};
      topk.row = row;
    }
    topk.init(a.k);
    int32_t* bound_ptr = a.row_bound + static_cast<int64_t>(row0 + row) * kBoundSlots;
    const int list_id = split * NWG + g;  // disjoint key set of this list
    // quantile slots are static list positions when the list is exactly full-width
    const bool quantiles = KCAP <= 64 && a.k == KCAP;
    float theta_loc = -INFINITY;       // worst kept score of this unit
    float bound = ordered_float(__ldcg(bound_ptr));
    float cut = fmaxf(theta_loc, float_below(bound));  // admit iff score > cut
    // Deferred insertion.  Past the first tiles of a unit a row meets a
    // candidate only every few tiles, and an immediate insert makes all 32
    // lanes of the warp wait for the one lane that has it.  Instead each lane
    // appends its candidates to a kDefer-entry buffer (a register shift: slot
    // 0 newest, slot n_def - 1 oldest) and the warp drains the buffers only
    // when one of them would overflow, so one insert pass serves every lane
    // with an entry waiting.  Draining re-checks each entry against the cut
    // and inserts a lane's entries in column order (buffer oldest first, then
    // the current chunk), so the list is the one immediate insertion builds.
    constexpr int kDefer = 4;
    float def_s[kDefer];
    int32_t def_i[kDefer];
    int n_def = 0;
    // Insert every buffered entry, then every candidate of mask m over v.
    // One loop (one copy of the insertion network); lanes run their own
    // iteration counts.
    auto drain = [&](uint32_t m, const float (&v)[32], int32_t col0) {
      while (n_def > 0 || m != 0u) {
        float x;
        int32_t xi;
        if (n_def > 0) {
          const int q = n_def - 1;  // oldest entry: a 2-level select, no dynamic indexing
          const float s01 = (q & 1) ? def_s[1] : def_s[0];
          const float s23 = (q & 1) ? def_s[3] : def_s[2];
          const int32_t i01 = (q & 1) ? def_i[1] : def_i[0];
          const int32_t i23 = (q & 1) ? def_i[3] : def_i[2];
          x = (q & 2) ? s23 : s01;
          xi = (q & 2) ? i23 : i01;
          --n_def;
        } else {
          const int j = __ffs(m) - 1;
          m &= m - 1u;
          x = pick32(v, j);
          xi = col0 + j;
        }
        if (x > cut) {
          topk.insert(x, xi);
          theta_loc = topk.worst();
          cut = fmaxf(theta_loc, float_below(bound));
        }
      }
    };
    static_assert(kDefer == 4, "drain() selects among exactly four buffered entries");
    // Scan 32 scores of this row (columns col0 .. col0 + min(rem, 32) - 1).
    auto scan_chunk = [&](const uint32_t (&r)[32], int rem, int32_t col0) {
      float v[32];
#pragma unroll
      for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r[j]);
      // Warp-wide prefilter: skip the chunk when no lane has a score above its cut.
      float mx[16];
#pragma unroll
      for (int i = 0; i < 16; ++i) mx[i] = fmaxf(v[2 * i], v[2 * i + 1]);
#pragma unroll
      for (int w2 = 8; w2 > 0; w2 >>= 1)
#pragma unroll
        for (int i = 0; i < w2; ++i) mx[i] = fmaxf(mx[i], mx[i + w2]);
      const bool maybe = rem < 32 || mx[0] > cut;
      if (!__any_sync(0xffffffffu, maybe)) return;
      // candidate bit mask, combined as a tree (short dependency chains)
      uint32_t b[16];
#pragma unroll
      for (int i = 0; i < 16; ++i)
        b[i] = (v[2 * i] > cut ? 1u : 0u) | (v[2 * i + 1] > cut ? 2u : 0u);
#pragma unroll
      for (int w2 = 8, sh = 2; w2 > 0; w2 >>= 1, sh <<= 1)
#pragma unroll
        for (int i = 0; i < w2; ++i) b[i] = b[2 * i] | (b[2 * i + 1] << sh);
      uint32_t m = b[0];
      if (rem < 32) m &= (1u << rem) - 1u;
      const int nc = __popc(m);
      if (__any_sync(0xffffffffu, n_def + nc > kDefer)) {
        drain(m, v, col0);
        return;
      }
      while (m) {
        const int j = __ffs(m) - 1;
        m &= m - 1u;
        const float s = pick32(v, j);
        if (s > cut) {
#pragma unroll
          for (int q = kDefer - 1; q >= 1; --q) {
            def_s[q] = def_s[q - 1];
            def_i[q] = def_i[q - 1];
          }
          def_s[0] = s;
          def_i[0] = col0 + j;
          ++n_def;
        }
      }
    };
    // AUX: the fused score of every (row, key) of the chunk, summed over the
    // rows of the row's group (sequence) and added into aux.  Runs after the
    // chunk's scan and overwrites the chunk's registers with v(s).
    //   v(s) = 2^(s c_exp)                                   (exp(s / T))
    //        * 1 / (1 + 2^(s c_g1 + c_g0))                   (the gate, when on)
    // with c_exp = log2(e) / T, c_g1 = -lambda log2(e), c_g0 = lambda tau log2(e):
    // per score one FMA-pipe and one special-function instruction without the
    // gate, four and three with it; the 1 / group_rows scale goes on the column
    // sums, and the TMEM loads overlap the work as in the plain scan.  (The
    // reciprocal as Newton steps on the FMA pipe instead measured slower: the
    // epilogue is issue-bound, not bound by the special-function unit.)
    const int64_t grow = static_cast<int64_t>(row0) + row;
    const int64_t my_group = AUX && grow < a.M ? grow / a.group_rows : -1;
    ScoreParams sp{a.lambda_sharp, a.tau, a.T};
    if constexpr (AUX) sp = load_score_params(a.params, a.lambda_sharp, a.tau, a.T);
    const float c_exp = kLog2e / sp.T;
    const float c_g1 = -sp.lambda_sharp * kLog2e;
    const float c_g0 = sp.lambda_sharp * sp.tau * kLog2e;
    const float aux_scale = AUX ? 1.0f / static_cast<float>(a.group_rows) : 0.0f;
    const int64_t g0 = __shfl_sync(0xffffffffu, my_group, 0);
    // rows increase with the lane: lane 0 invalid means the whole warp is padding
    const bool aux_uniform = __all_sync(0xffffffffu, my_group == g0 || my_group < 0);
    const bool aux_all_rows = __all_sync(0xffffffffu, my_group >= 0);
    auto aux_chunk = [&](uint32_t (&r)[32], int rem, int32_t col0) {
      if (g0 < 0) return;
      if (a.use_sigmoid) {
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          const float sc = __uint_as_float(r[j]);
          const float gate = rcp_approx(1.0f + ex2_approx(fmaf(sc, c_g1, c_g0)));
          r[j] = __float_as_uint(ex2_approx(sc * c_exp) * gate);
        }
      } else {
#pragma unroll
        for (int j = 0; j < 32; ++j) r[j] = __float_as_uint(ex2_approx(__uint_as_float(r[j]) * c_exp));
      }
      if (rem < 32 || !aux_all_rows) {
#pragma unroll
        for (int j = 0; j < 32; ++j)
          if (my_group < 0 || j >= rem) r[j] = 0u;
      }
      float f[32];
#pragma unroll
      for (int j = 0; j < 32; ++j) f[j] = __uint_as_float(r[j]);
      if (aux_uniform) {
        const float colsum = warp_column_sum32(f, lane);
        if (lane < rem) atomicAdd(a.aux + g0 * a.ld_aux + col0 + lane, colsum * aux_scale);
      } else if (my_group >= 0) {
        // rows of two groups in this warp: every lane adds its own values
#pragma unroll
        for (int j = 0; j < 32; ++j)
          if (j < rem) atomicAdd(a.aux + my_group * a.ld_aux + col0 + j, f[j] * aux_scale);
      }
    };
    const uint32_t lead_tempty0 = map_to_cta(tempty_bar(0), 0);
    const uint32_t lead_tempty1 = map_to_cta(tempty_bar(1), 0);
    for (int t = 0; t < n_tiles; ++t) {
      const int acc = t & 1;
      const uint32_t use = static_cast<uint32_t>(t >> 1);
      // warp-uniform outcome: the votes below need all 32 lanes on the same path
      const bool got = mbar_wait(tfull_bar(acc), use & 1u, a.status, abort_flag);
      if (!__all_sync(0xffffffffu, got)) break;
      tc_fence_after();
      // The row's shared bounds as published so far, read before the scan so
      // the latency hides behind it.  With two warpgroups the 16 registers
      // are not there (10 warps share four 16K-register sub-partitions: at
      // most 168 per thread), so they are read after the scan.
      int4 sb0, sb1, sb2, sb3;
      if constexpr (NWG == 1) {
        sb0 = ld_relaxed_gpu_v4(bound_ptr);
        sb1 = ld_relaxed_gpu_v4(bound_ptr + 4);
        sb2 = ld_relaxed_gpu_v4(bound_ptr + 8);
        sb3 = ld_relaxed_gpu_v4(bound_ptr + 12);
      }
      const int64_t n0 = (kt_begin + t) * kTileN;
      const int valid = static_cast<int>(min(static_cast<int64_t>(kTileN), a.N - n0));
      // this warpgroup's columns [cb, ce) of the tile (empty on a short last tile)
      const int cb = g * kColsPerWg;
      const int ce = min(valid, cb + kColsPerWg);
      const uint32_t taddr =
          tmem_base + (static_cast<uint32_t>(ew * 32) << 16) + static_cast<uint32_t>(acc * kTileN);
      // Chunks of 32 columns.  Two register sets in flight (the TMEM load of
      // the next chunk overlaps the scan and aux sums of the current one)
      // wherever the list leaves the registers for them.
      constexpr bool kOverlap = !AUX || KCAP == 16 || KCAP == kCapHeap128 || NWG == 1 && KCAP <= 32;
      if (!kOverlap) {
        for (int c = cb; c < ce; c += 32) {
          uint32_t r[32];
          tmem_ld_32x32b_x32_async(taddr + c, r);
          tmem_wait_ld_pin(r);
          scan_chunk(r, ce - c, static_cast<int32_t>(n0 + c));
          if constexpr (AUX) aux_chunk(r, ce - c, static_cast<int32_t>(n0 + c));
        }
      } else if (cb < ce) {
        uint32_t ra[32], rb[32];
        tmem_ld_32x32b_x32_async(taddr + cb, ra);
        tmem_wait_ld_pin(ra);
        for (int c = cb; c < ce; c += 64) {
          const bool has_b = c + 32 < ce;   // warp-uniform
          if (has_b) tmem_ld_32x32b_x32_async(taddr + c + 32, rb);
          scan_chunk(ra, ce - c, static_cast<int32_t>(n0 + c));
          if constexpr (AUX) aux_chunk(ra, ce - c, static_cast<int32_t>(n0 + c));
          if (has_b) {
            tmem_wait_ld_pin(rb);
            const bool has_next = c + 64 < ce;
            if (has_next) tmem_ld_32x32b_x32_async(taddr + c + 64, ra);
            scan_chunk(rb, ce - c - 32, static_cast<int32_t>(n0 + c + 32));
            if constexpr (AUX) aux_chunk(rb, ce - c - 32, static_cast<int32_t>(n0 + c + 32));
            if (has_next) tmem_wait_ld_pin(ra);
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(acc ? lead_tempty1 : lead_tempty0);
      // Publish this list's k-th best and its (k/P)-th bests (no round trip)
      // and take up the best bound read at the start of the tile.
      if (theta_loc > -INFINITY) red_max_gpu(bound_ptr, ordered_int(theta_loc));
      if constexpr (KCAP <= 64) {
        if (quantiles) {
          const float q2 = topk.s[KCAP / 2 - 1], q4 = topk.s[KCAP / 4 - 1], q8 = topk.s[KCAP / 8 - 1];
          if (q2 > -INFINITY) red_max_gpu(bound_ptr + 1 + (list_id & 1), ordered_int(q2));
          if (q4 > -INFINITY) red_max_gpu(bound_ptr + 3 + (list_id & 3), ordered_int(q4));
          if (q8 > -INFINITY) red_max_gpu(bound_ptr + 7 + (list_id & 7), ordered_int(q8));
        }
      }
      if constexpr (NWG != 1) {
        sb0 = ld_relaxed_gpu_v4(bound_ptr);
        sb1 = ld_relaxed_gpu_v4(bound_ptr + 4);
        sb2 = ld_relaxed_gpu_v4(bound_ptr + 8);
        sb3 = ld_relaxed_gpu_v4(bound_ptr + 12);
      }
      {
        int32_t bi = sb0.x;
        bi = max(bi, min(sb0.y, sb0.z));
        bi = max(bi, min(min(sb0.w, sb1.x), min(sb1.y, sb1.z)));
        bi = max(bi, min(min(min(sb1.w, sb2.x), min(sb2.y, sb2.z)),
                         min(min(sb2.w, sb3.x), min(sb3.y, sb3.z))));
        bound = fmaxf(bound, ordered_float(bi));
      }
      cut = fmaxf(theta_loc, float_below(bound));
    }
    {
      float none[32];
#pragma unroll
      for (int j = 0; j < 32; ++j) none[j] = -INFINITY;
      drain(0u, none, 0);
    }
    // Flush this unit's list for the row, best first: [split * NWG + g][row][pos].
    const int64_t o = (static_cast<int64_t>(split * NWG + g) * a.m_pad + row0 + row) * a.k;
    topk.write_out(a.ws_vals + o, a.ws_idx + o, a.k);
  }

  tc_fence_before();
  __syncthreads();
  if (leader && threadIdx.x == 0) {
    // Loads issued but never consumed (only after an abort) must land before exit.
    for (int i = *n_consumed; i < *n_issued; ++i)
      mbar_wait_cluster(full_bar(i % S), static_cast<uint32_t>(i / S) & 1u, a.status, nullptr);
  }
  tc_fence_before();
  cluster_sync();  // the leader's MMAs are done; the peer may release its memory
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, 2 * kTileN);
  }
}

__global__ void fill_i32_kernel(int32_t* p, int64_t n, int32_t v) {
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i < n) p[i] = v;
}

// ---------------------------------------------------------------- host side
template <int KCAP, int NWG, bool AUX>
cudaError_t configure_once() {
  static std::atomic<uint64_t> done_mask{0};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  const uint64_t bit = 1ull << (dev & 63);
  if (done_mask.load(std::memory_order_acquire) & bit) return cudaSuccess;
  e = cudaFuncSetAttribute(score_topk_kernel<KCAP, NWG, AUX>,
                           cudaFuncAttributeMaxDynamicSharedMemorySize,
                           TopkCfg<KCAP, NWG>::kSmemBytes);
  if (e == cudaSuccess) done_mask.fetch_or(bit, std::memory_order_acq_rel);
  return e;
}

template <int KCAP, int NWG, bool AUX>
cudaError_t launch_variant(const ScoreTopkPlan& p, const CUtensorMap& mq, const CUtensorMap& mk,
                           const TopkKernelArgs& args, cudaStream_t stream) {
  cudaError_t e = configure_once<KCAP, NWG, AUX>();
  if (e != cudaSuccess) return e;
  const unsigned grid = 2u * static_cast<unsigned>(p.n_qt) * static_cast<unsigned>(p.n_split);
  score_topk_kernel<KCAP, NWG, AUX>
      <<<grid, threads_for(NWG), TopkCfg<KCAP, NWG>::kSmemBytes, stream>>>(mq, mk, args);
  return cudaGetLastError();
}

}  // namespace

// Shared with key_projection.cu (declared in dwa_internal.h).
PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
  static std::once_flag once;
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault,
                                         &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

bool make_bf16_tile_map(CUtensorMap* map, const void* ptr, uint64_t inner, uint64_t rows,
                        uint64_t ld_elems, uint32_t box_inner, uint32_t box_rows) {
  auto encode = tensor_map_encoder();
  if (!encode) return false;
  cuuint64_t dims[2] = {inner, rows};
  cuuint64_t strides[1] = {ld_elems * 2};
  cuuint32_t box[2] = {box_inner, box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = encode(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(ptr), dims,
                      strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                      CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                      CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

cudaError_t launch_plan(const ScoreTopkPlan& p, const CUtensorMap& mq, const CUtensorMap& mk,
                        const TopkKernelArgs& args, cudaStream_t stream);

int device_sm_count() {
  static std::atomic<int> cache[64] = {};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 148;
  int v = cache[dev & 63].load(std::memory_order_relaxed);
  if (v > 0) return v;
  if (cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || v <= 0)
    v = 148;
  cache[dev & 63].store(v, std::memory_order_relaxed);
  return v;
}

bool plan_score_topk(int64_t M, int64_t N, int d, int k, int num_sms, ScoreTopkPlan* plan) {
  if (M <= 0 || N <= 0 || d <= 0 || k <= 0 || num_sms <= 1) return false;
  ScoreTopkPlan p;
  p.M = M;
  p.N = N;
  p.d = d;
  p.k = k;
  p.kcap = k <= 16 ? 16 : k <= 32 ? 32 : k <= 64 ? 64 : k <= 128 ? 128 : 0;
  if (p.kcap == 0) return false;
  const int64_t n_qt = (M + kPairRows - 1) / kPairRows;
  if (n_qt > (1 << 24)) return false;
  p.n_qt = static_cast<int>(n_qt);
  p.n_kt = (N + kTileN - 1) / kTileN;
  p.num_kb = (d + kTileK - 1) / kTileK;
  p.m_pad = n_qt * kPairRows;
  // Two epilogue warpgroups (one list each, half of every tile's columns) for k <= 32,
  // where the register lists leave room for 10 warps; k >= 64 keeps one.
  p.nwg = p.kcap <= 32 ? 2 : 1;
  // Choose the number of key-range splits: minimise the modelled makespan
  // waves * (tiles per unit + per-unit overhead), one CTA pair per two SMs.
  // Per-unit overhead in tile-times: pipeline fill/drain, the heap warm-up at
  // the start of every unit (the first tiles insert most candidates), the
  // sorted flush and one more list for the split merge.
  const double unit_overhead_tiles = 8.0;
  const int64_t pairs = num_sms / 2;
  int best_s = 1;
  double best_cost = 1e300;
  const int64_t s_max = std::min<int64_t>(p.n_kt, kMaxSplits / p.nwg);
  for (int64_t s = 1; s <= s_max; ++s) {
    const int64_t units = n_qt * s;
    if (2 * units > (1ll << 31) - 1) break;
    const int64_t waves = (units + pairs - 1) / pairs;
    const int64_t tiles_per_unit = (p.n_kt + s - 1) / s;
    const double cost =
        static_cast<double>(waves) * (static_cast<double>(tiles_per_unit) + unit_overhead_tiles);
    if (cost < best_cost * (1.0 - 1e-9)) {
      best_cost = cost;
      best_s = static_cast<int>(s);
    }
  }
  p.n_split = best_s;
  // Unit order.  Split-major over all query tiles keeps the resident pairs on
  // a few key ranges, so each key tile is read from HBM about once; that
  // needs the whole query set to stay in L2.  Once the queries exceed half
  // of L2, every key tile would re-read its pair's query tile from HBM, so
  // units go in groups of G query tiles x all splits (G * n_split about the
  // resident pair count): G query tiles stay in L2 and each key tile is
  // read once per group.
  // k in (64, 128]: the two-level list (five ring stages) when a unit's MMA
  // work (key tiles x d) is long next to filling its lists; the whole-heap
  // list (three stages, cheaper inserts) otherwise.  Measured, same indices:
  // 16384 x 2,097,152 x 4096 (546-tile units) 241.5 vs 270.0 ms,
  // 16384 x 262,144 x 4096 (128-tile units) 35.5 vs 35.4 ms,
  // 8192 x 131,072 x 1024 (57-tile units) 5.71 vs 4.57 ms.
  if (p.kcap == 128 &&
      (p.n_kt + p.n_split - 1) / p.n_split * static_cast<int64_t>(d) < kSplitListMinWork)
    p.kcap = 129;
  const int64_t query_bytes = p.m_pad * static_cast<int64_t>(p.num_kb) * kTileK * 2;
  p.group = 0;
  if (query_bytes > (64ll << 20)) {
    const int64_t g = std::max<int64_t>(1, pairs / p.n_split);
    if (g < n_qt) p.group = static_cast<int>(g);
  }
  p.ws_bytes = kStatusBytes + static_cast<size_t>(p.m_pad) * kBoundSlots * 4u +
               static_cast<size_t>(p.n_split) * p.nwg * static_cast<size_t>(k) *
                   static_cast<size_t>(p.m_pad) * 8u;
  *plan = p;
  return true;
}

cudaError_t launch_score_topk(const ScoreTopkPlan& p, const void* q, int64_t ldq, const void* keys,
                              int64_t ldk, float lambda_sharp, float tau, float T, int use_sigmoid,
                              int64_t idx_offset, float* out_vals, int32_t* out_idx, void* ws,
                              cudaStream_t stream, const char** err_detail, const float* params,
                              const SeqMeanOut* seq_mean) {
  CUtensorMap mq, mk;
  if (!make_bf16_tile_map(&mq, q, static_cast<uint64_t>(p.d), static_cast<uint64_t>(p.M),
                          static_cast<uint64_t>(ldq), kTileK, kTileM) ||
      !make_bf16_tile_map(&mk, keys, static_cast<uint64_t>(p.d), static_cast<uint64_t>(p.N),
                          static_cast<uint64_t>(ldk), kTileK, kKeysPerCta)) {
    if (err_detail) *err_detail = "cuTensorMapEncodeTiled failed for the query or key tensor";
    return cudaErrorInvalidValue;
  }
  uint8_t* wsb = static_cast<uint8_t*>(ws);
  TopkKernelArgs args;
  args.N = p.N;
  args.n_kt = p.n_kt;
  args.m_pad = p.m_pad;
  args.num_kb = p.num_kb;
  args.k = p.k;
  args.n_qt = p.n_qt;
  args.n_split = p.n_split;
  args.group = p.group;
  args.status = reinterpret_cast<int*>(wsb);
  const size_t list_elems = static_cast<size_t>(p.n_split) * p.nwg * p.k * p.m_pad;
  const size_t bound_bytes = static_cast<size_t>(p.m_pad) * kBoundSlots * 4u;
  args.row_bound = reinterpret_cast<int32_t*>(wsb + kStatusBytes);
  args.ws_vals = reinterpret_cast<float*>(wsb + kStatusBytes + bound_bytes);
  args.ws_idx = reinterpret_cast<int32_t*>(wsb + kStatusBytes + bound_bytes + list_elems * 4);
  args.M = p.M;
  args.aux = nullptr;
  args.ld_aux = 0;
  args.group_rows = 1;
  args.params = params;
  args.lambda_sharp = lambda_sharp;
  args.tau = tau;
  args.T = T;
  args.use_sigmoid = use_sigmoid;
  if (seq_mean != nullptr) {
    args.aux = seq_mean->out;
    args.ld_aux = seq_mean->ld;
    args.group_rows = seq_mean->group_rows;
    // the kernel adds into it: start from zero (stream-ordered)
    const int64_t groups = p.M / seq_mean->group_rows;
    cudaError_t ez = cudaMemset2DAsync(seq_mean->out, static_cast<size_t>(seq_mean->ld) * 4, 0,
                                       static_cast<size_t>(p.N) * 4, static_cast<size_t>(groups),
                                       stream);
    if (ez != cudaSuccess) return ez;
  }

  cudaError_t e = cudaMemsetAsync(ws, 0, sizeof(int), stream);
  if (e != cudaSuccess) return e;
  // The ordered image of -inf: "no bound yet" (every score is admissible).
  constexpr int32_t kImageNegInf = static_cast<int32_t>(0xFF800000u ^ 0x7FFFFFFFu);
  const int64_t n_bounds = p.m_pad * kBoundSlots;
  fill_i32_kernel<<<static_cast<unsigned>((n_bounds + 255) / 256), 256, 0, stream>>>(
      args.row_bound, n_bounds, kImageNegInf);
  e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  e = launch_plan(p, mq, mk, args, stream);
  if (e != cudaSuccess) return e;
  return launch_merge_topk(args.ws_vals, args.ws_idx, p.n_split * p.nwg, p.k,
                           static_cast<int64_t>(p.k) * p.m_pad, 1, p.k, p.M, p.k,
                           /*transform=*/1, lambda_sharp, tau, T, use_sigmoid, idx_offset, out_vals,
                           out_idx, stream, params, args.status);
}

cudaError_t launch_plan(const ScoreTopkPlan& p, const CUtensorMap& mq, const CUtensorMap& mk,
                        const TopkKernelArgs& args, cudaStream_t stream) {
  const bool aux = args.aux != nullptr;
  switch (p.kcap * 8 + p.nwg * 2 + (aux ? 1 : 0)) {
    case 16 * 8 + 4: return launch_variant<16, 2, false>(p, mq, mk, args, stream);
    case 32 * 8 + 4: return launch_variant<32, 2, false>(p, mq, mk, args, stream);
    case 64 * 8 + 2: return launch_variant<64, 1, false>(p, mq, mk, args, stream);
    case 128 * 8 + 2: return launch_variant<128, 1, false>(p, mq, mk, args, stream);
    case 129 * 8 + 2: return launch_variant<129, 1, false>(p, mq, mk, args, stream);
    case 16 * 8 + 5: return launch_variant<16, 2, true>(p, mq, mk, args, stream);
    case 32 * 8 + 5: return launch_variant<32, 2, true>(p, mq, mk, args, stream);
    case 64 * 8 + 3: return launch_variant<64, 1, true>(p, mq, mk, args, stream);
    case 128 * 8 + 3: return launch_variant<128, 1, true>(p, mq, mk, args, stream);
    case 129 * 8 + 3: return launch_variant<129, 1, true>(p, mq, mk, args, stream);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace dwa
