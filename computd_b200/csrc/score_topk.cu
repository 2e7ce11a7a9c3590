// score_topk.cu — fused query x pool-key score GEMM with a streaming top-k
// epilogue, for sm_100a (B200).
//
// Replaces the executed score + top-k of the reference,
// tiled_topk_fallback (src/kernels/tiled_topk.py:160-176):
//     sims = jnp.dot(queries, keys.T); score = gate(sims) * exp(sims / T);
//     lax.top_k(score, k_max)
// which materialises the whole [M, N] score matrix before a sort-based top-k.
// Here the [128 x 256] score tile lives only in tensor memory (TMEM); the
// epilogue keeps the k best (score, index) per query row in a shared-memory
// heap and the full score matrix never reaches HBM.
//
// CTA = 6 warps, warp-specialised:
//   warp 0     TMA producer: bf16 query tile [128 x 64] and key tile [256 x 64]
//              per k-block, 128-byte swizzled, into a STAGES-deep ring
//   warp 1     TMEM allocator + UMMA issuer: tcgen05.mma.cta_group::1.kind::f16
//              128x256x16, fp32 accumulators double-buffered in TMEM (2 x 256 cols)
//   warps 2-5  epilogue: warp w reads TMEM lanes 32*(w%4).. with tcgen05.ld;
//              thread = one query row, register threshold = heap root, warp-wide
//              OR of the "beats threshold" masks skips clean 32-column chunks
//
// Work unit = (query tile, contiguous range of key tiles).  Units are ordered
// split-major so the CTAs resident at one time sweep the same few key ranges:
// every key tile is fetched from HBM about once and re-served from L2 to all
// query tiles.  Each unit leaves one partial top-k list per row in the
// workspace; merge_topk.cu merges the splits, sorts, applies the gate/exp and
// adds the global index offset.
#include <cuda.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <atomic>
#include <cmath>
#include <mutex>

#include "dwa_internal.h"
#include "sm100_ptx.cuh"
#include "topk_heap.cuh"

namespace dwa {

namespace {

constexpr int kThreads = 192;
constexpr int kMaxDynSmem = 232448;  // 227 KB opt-in limit on sm_100

template <int KCAP>
struct TopkCfg {
  static constexpr int kStageA = kTileM * kTileK * 2;  // 16 KB query tile
  static constexpr int kStageB = kTileN * kTileK * 2;  // 32 KB key tile
  static constexpr int kStageBytes = kStageA + kStageB;
  static constexpr int kHeapBytes = KCAP * kTileM * 8;
  static constexpr int kBarBytes = 256;
  static constexpr int kStagesFit = (kMaxDynSmem - 1024 - kHeapBytes - kBarBytes) / kStageBytes;
  static constexpr int kStages = kStagesFit > 4 ? 4 : kStagesFit;
  static constexpr int kSmemBytes = 1024 + kStages * kStageBytes + kHeapBytes + kBarBytes;
  static_assert(kStages >= 2, "pipeline needs at least two stages");
  static_assert(kSmemBytes <= kMaxDynSmem, "shared memory budget exceeded");
};

struct TopkKernelArgs {
  int64_t N;         // keys in this shard
  int64_t n_kt;      // key tiles
  int64_t m_pad;     // padded query rows (row stride of the partial lists)
  int num_kb;        // 64-wide k-blocks along d
  int k;             // kept per row
  int n_qt;          // query tiles
  int n_split;       // key-range splits
  float* ws_vals;    // [n_split][k][m_pad] raw scores
  int32_t* ws_idx;   // [n_split][k][m_pad] local key indices
  int* status;       // device status word
};

template <int KCAP>
__global__ void __launch_bounds__(kThreads, 1)
    score_topk_kernel(const __grid_constant__ CUtensorMap tmap_q,
                      const __grid_constant__ CUtensorMap tmap_k, const TopkKernelArgs a) {
  using C = TopkCfg<KCAP>;
  constexpr int S = C::kStages;

  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  const uint32_t base = (raw_addr + 1023u) & ~1023u;
  uint8_t* smem = smem_raw + (base - raw_addr);

  const uint32_t sA0 = base;               // stage s query tile at sA0 + s * kStageBytes
  const uint32_t sB0 = base + C::kStageA;  // stage s key tile   at sB0 + s * kStageBytes
  float* heap_s = reinterpret_cast<float*>(smem + S * C::kStageBytes);
  int32_t* heap_i = reinterpret_cast<int32_t*>(smem + S * C::kStageBytes + KCAP * kTileM * 4);
  uint8_t* bar_area = smem + S * C::kStageBytes + C::kHeapBytes;
  const uint32_t bar0 = smem_u32(bar_area);
  auto full_bar = [&](int s) { return bar0 + 8u * s; };
  auto empty_bar = [&](int s) { return bar0 + 8u * (S + s); };
  auto tfull_bar = [&](int acc) { return bar0 + 8u * (2 * S + acc); };
  auto tempty_bar = [&](int acc) { return bar0 + 8u * (2 * S + 2 + acc); };
  const uint32_t drain_bar = bar0 + 8u * (2 * S + 4);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bar_area + 8 * (2 * S + 5));
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  int* n_issued = reinterpret_cast<int*>(tmem_slot + 2);
  int* n_consumed = reinterpret_cast<int*>(tmem_slot + 3);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  const int unit = blockIdx.x;
  const int qt = unit % a.n_qt;
  const int split = unit / a.n_qt;
  const int64_t kt_begin = static_cast<int64_t>(split) * a.n_kt / a.n_split;
  const int64_t kt_end = static_cast<int64_t>(split + 1) * a.n_kt / a.n_split;
  const int n_tiles = static_cast<int>(kt_end - kt_begin);

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(full_bar(s), 1);
      mbar_init(empty_bar(s), 1);
    }
    for (int acc = 0; acc < 2; ++acc) {
      mbar_init(tfull_bar(acc), 1);
      mbar_init(tempty_bar(acc), 4);
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
    tmem_alloc(smem_u32(tmem_slot), 2 * kTileN);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
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
        const int32_t krow = static_cast<int32_t>((kt_begin + t) * kTileN);
        for (int kb = 0; kb < a.num_kb; ++kb, ++it) {
          const int s = it % S;
          const uint32_t r = static_cast<uint32_t>(it / S);
          if (!mbar_wait(empty_bar(s), (r & 1u) ^ 1u, a.status, abort_flag)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(full_bar(s), C::kStageBytes);
          tma_load_2d(sA0 + s * C::kStageBytes, &tmap_q, full_bar(s), kb * kTileK, qt * kTileM,
                      pol_q);
          tma_load_2d(sB0 + s * C::kStageBytes, &tmap_k, full_bar(s), kb * kTileK, krow, pol_k);
        }
      }
      *n_issued = it;
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ UMMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = umma_idesc_bf16_f32(kTileM, kTileN);
      int it = 0;
      bool ok = true;
      for (int t = 0; t < n_tiles && ok; ++t) {
        const int acc = t & 1;
        const uint32_t use = static_cast<uint32_t>(t >> 1);
        if (!mbar_wait(tempty_bar(acc), (use & 1u) ^ 1u, a.status, abort_flag)) break;
        tc_fence_after();
        const uint32_t tmem_d = tmem_base + static_cast<uint32_t>(acc * kTileN);
        for (int kb = 0; kb < a.num_kb; ++kb, ++it) {
          const int s = it % S;
          const uint32_t r = static_cast<uint32_t>(it / S);
          if (!mbar_wait(full_bar(s), r & 1u, a.status, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t ad = sw128_kmajor_desc(sA0 + s * C::kStageBytes);
          const uint64_t bd = sw128_kmajor_desc(sB0 + s * C::kStageBytes);
#pragma unroll
          for (int kk = 0; kk < kTileK / 16; ++kk) {
            // +32 bytes along K inside the swizzled 128-byte row = +2 in the address field
            umma_bf16_ss(tmem_d, ad + 2u * kk, bd + 2u * kk, idesc, (kb | kk) != 0 ? 1u : 0u);
          }
          umma_commit(empty_bar(s));
        }
        if (ok) umma_commit(tfull_bar(acc));
      }
      *n_consumed = it;
      // All MMAs this thread issued must finish before TMEM is released.
      umma_commit(drain_bar);
      mbar_wait(drain_bar, 0u, a.status, nullptr);
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int ew = warp & 3;           // TMEM lane quarter this warp may access
    const int row = ew * 32 + lane;    // query row within the tile
    const SmemHeap heap{heap_s, heap_i, kTileM, a.k};
    heap.init(row);
    float theta = -INFINITY;           // score of the heap root (worst kept)
    for (int t = 0; t < n_tiles; ++t) {
      const int acc = t & 1;
      const uint32_t use = static_cast<uint32_t>(t >> 1);
      if (!mbar_wait(tfull_bar(acc), use & 1u, a.status, abort_flag)) break;
      tc_fence_after();
      const int64_t n0 = (kt_begin + t) * kTileN;
      const int valid = static_cast<int>(min(static_cast<int64_t>(kTileN), a.N - n0));
      const uint32_t taddr =
          tmem_base + (static_cast<uint32_t>(ew * 32) << 16) + static_cast<uint32_t>(acc * kTileN);
      for (int c = 0; c < valid; c += 32) {
        float v[32];
        tmem_ld_32x32b_x32_sync(taddr + c, v);
        uint32_t m = 0;
#pragma unroll
        for (int j = 0; j < 32; ++j) m |= (v[j] > theta ? 1u : 0u) << j;
        const int rem = valid - c;
        if (rem < 32) m &= (1u << rem) - 1u;
        uint32_t wm = __reduce_or_sync(0xffffffffu, m);
        while (wm) {
          const int j = __ffs(wm) - 1;
          wm &= wm - 1u;
          // Re-read column j for all 32 rows (warp-collective) rather than
          // index the register array dynamically.
          const float s = tmem_ld_32x32b_x1_sync(taddr + c + j);
          if (((m >> j) & 1u) && s > theta) {
            heap.replace_root(row, s, static_cast<int32_t>(n0 + c + j));
            theta = heap.S(0, row);
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(tempty_bar(acc));
    }
    // Flush this unit's partial list: [split][pos][row], coalesced across rows.
    const int64_t col = static_cast<int64_t>(qt) * kTileM + row;
    for (int p = 0; p < a.k; ++p) {
      const int64_t o = (static_cast<int64_t>(split) * a.k + p) * a.m_pad + col;
      a.ws_vals[o] = heap.S(p, row);
      a.ws_idx[o] = heap.I(p, row);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (threadIdx.x == 0) {
    // Loads issued but never consumed (only after an abort) must land before exit.
    for (int i = *n_consumed; i < *n_issued; ++i)
      mbar_wait(full_bar(i % S), static_cast<uint32_t>(i / S) & 1u, a.status, nullptr);
  }
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, 2 * kTileN);
  }
}

// ---------------------------------------------------------------- host side
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

template <int KCAP>
cudaError_t configure_once() {
  static std::atomic<uint64_t> done_mask{0};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  const uint64_t bit = 1ull << (dev & 63);
  if (done_mask.load(std::memory_order_acquire) & bit) return cudaSuccess;
  e = cudaFuncSetAttribute(score_topk_kernel<KCAP>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           TopkCfg<KCAP>::kSmemBytes);
  if (e == cudaSuccess) done_mask.fetch_or(bit, std::memory_order_acq_rel);
  return e;
}

template <int KCAP>
cudaError_t launch_variant(const ScoreTopkPlan& p, const CUtensorMap& mq, const CUtensorMap& mk,
                           const TopkKernelArgs& args, cudaStream_t stream) {
  cudaError_t e = configure_once<KCAP>();
  if (e != cudaSuccess) return e;
  const unsigned grid = static_cast<unsigned>(p.n_qt) * static_cast<unsigned>(p.n_split);
  score_topk_kernel<KCAP><<<grid, kThreads, TopkCfg<KCAP>::kSmemBytes, stream>>>(mq, mk, args);
  return cudaGetLastError();
}

}  // namespace

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
  if (M <= 0 || N <= 0 || d <= 0 || k <= 0 || num_sms <= 0) return false;
  ScoreTopkPlan p;
  p.M = M;
  p.N = N;
  p.d = d;
  p.k = k;
  p.kcap = k <= 16 ? 16 : k <= 32 ? 32 : k <= 64 ? 64 : k <= 128 ? 128 : 0;
  if (p.kcap == 0) return false;
  const int64_t n_qt = (M + kTileM - 1) / kTileM;
  if (n_qt > (1 << 24)) return false;
  p.n_qt = static_cast<int>(n_qt);
  p.n_kt = (N + kTileN - 1) / kTileN;
  p.num_kb = (d + kTileK - 1) / kTileK;
  p.m_pad = n_qt * kTileM;
  // Choose the number of key-range splits: minimise the modelled makespan
  // waves * (tiles per unit + per-unit overhead), one CTA per SM.
  const double unit_overhead_tiles = 1.5;
  int best_s = 1;
  double best_cost = 1e300;
  const int64_t s_max = std::min<int64_t>(p.n_kt, 4096);
  for (int64_t s = 1; s <= s_max; ++s) {
    const int64_t units = n_qt * s;
    if (units > (1ll << 31) - 1) break;
    const int64_t waves = (units + num_sms - 1) / num_sms;
    const int64_t tiles_per_unit = (p.n_kt + s - 1) / s;
    const double cost =
        static_cast<double>(waves) * (static_cast<double>(tiles_per_unit) + unit_overhead_tiles);
    if (cost < best_cost * (1.0 - 1e-9)) {
      best_cost = cost;
      best_s = static_cast<int>(s);
    }
  }
  p.n_split = best_s;
  p.ws_bytes = kStatusBytes + static_cast<size_t>(p.n_split) * static_cast<size_t>(k) *
                                  static_cast<size_t>(p.m_pad) * 8u;
  *plan = p;
  return true;
}

cudaError_t launch_score_topk(const ScoreTopkPlan& p, const void* q, int64_t ldq, const void* keys,
                              int64_t ldk, float lambda_sharp, float tau, float T, int use_sigmoid,
                              int64_t idx_offset, float* out_vals, int32_t* out_idx, void* ws,
                              cudaStream_t stream, const char** err_detail) {
  CUtensorMap mq, mk;
  if (!make_bf16_tile_map(&mq, q, static_cast<uint64_t>(p.d), static_cast<uint64_t>(p.M),
                          static_cast<uint64_t>(ldq), kTileK, kTileM) ||
      !make_bf16_tile_map(&mk, keys, static_cast<uint64_t>(p.d), static_cast<uint64_t>(p.N),
                          static_cast<uint64_t>(ldk), kTileK, kTileN)) {
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
  args.status = reinterpret_cast<int*>(wsb);
  const size_t list_elems = static_cast<size_t>(p.n_split) * p.k * p.m_pad;
  args.ws_vals = reinterpret_cast<float*>(wsb + kStatusBytes);
  args.ws_idx = reinterpret_cast<int32_t*>(wsb + kStatusBytes + list_elems * 4);

  cudaError_t e = cudaMemsetAsync(ws, 0, sizeof(int), stream);
  if (e != cudaSuccess) return e;
  switch (p.kcap) {
    case 16: e = launch_variant<16>(p, mq, mk, args, stream); break;
    case 32: e = launch_variant<32>(p, mq, mk, args, stream); break;
    case 64: e = launch_variant<64>(p, mq, mk, args, stream); break;
    case 128: e = launch_variant<128>(p, mq, mk, args, stream); break;
    default: return cudaErrorInvalidValue;
  }
  if (e != cudaSuccess) return e;
  return launch_merge_topk(args.ws_vals, args.ws_idx, p.n_split, p.k,
                           static_cast<int64_t>(p.k) * p.m_pad, p.m_pad, 1, p.M, p.k,
                           /*transform=*/1, lambda_sharp, tau, T, use_sigmoid, idx_offset, out_vals,
                           out_idx, stream);
}

}  // namespace dwa
