// key_projection.cu — pool keys of the DWA retrieval: projection, per-aspect
// L2 normalisation and aspect collapse in one tcgen05 GEMM, for sm_100a (B200).
//
// Reference: MultiAspectRetrieval.pallas_hybrid_forward
// (src/model/retrieval.py:241-242, 253, 261):
//     keys_s = einsum('skd,nd->snk', W_K, vectors)           (S, N, d_k)
//     keys_s = keys_s / (norm(keys_s, axis=-1) + 1e-8)
//     keys_w = einsum('s,snk->nk', softmax(aspect_logits), keys_s)
// The reference materialises the (S, N, d_k) projection.  Here the pool rows
// [N, D] times W_K viewed as [S * d_k, D] run as one GEMM on the tensor cores
// (a CTA pair, tcgen05.mma.cta_group::2, 256 rows x 256 projection columns
// per accumulator, fp32 in TMEM); the epilogue normalises each d_k-wide aspect
// segment of a row and adds w_s times it into a d_k-register accumulator, so
// the collapse happens in registers and only keys_w [N, d_k] (bf16) is
// written.
//
// Warp roles per CTA (as in the score kernel): warp 0 TMA producer, warp 1
// TMEM allocation + MMA issue (leader CTA), warps 2-5 epilogue (one pool row
// per thread).  A pair owns 256 pool rows and walks all ceil(S d_k / 256)
// projection tiles; pool-row tiles are re-read from L2 for each projection
// tile.  All waits are bounded (2 s) and report DWA_ERR_TIMEOUT through the
// optional status word.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <cmath>

#include "dwa_internal.h"
#include "sm100_ptx.cuh"

namespace dwa {

namespace {

constexpr int kKpThreads = 192;
constexpr int kKpPairRows = 2 * kTileM;   // 256 pool rows per CTA pair
constexpr int kKpColsPerCta = kTileN / 2; // 128 projection columns staged per CTA
constexpr int kKpStageA = kTileM * kTileK * 2;
constexpr int kKpStageB = kKpColsPerCta * kTileK * 2;
constexpr int kKpStageBytes = kKpStageA + kKpStageB;
constexpr int kKpMaxSmem = 232448;
constexpr int kKpStages = std::min(7, (kKpMaxSmem - 1024 - 256) / kKpStageBytes);
constexpr int kKpSmemBytes = 1024 + kKpStages * kKpStageBytes + 256;

struct KeyProjArgs {
  int64_t N;
  int num_kb;   // 64-wide blocks along D
  int n_nt;     // 256-column projection tiles
  int S;
  const float* w;  // [S] aspect weights
  __nv_bfloat16* out;
  int64_t ldo;
  int* status;  // may be null
};

// PACK = false: keys_w[n] = sum_s w_s k_s / (|k_s| + 1e-8)  (the collapse of
//               pallas_hybrid_forward, retrieval.py:261), out [N, DK].
// PACK = true:  out[n, s DK : (s + 1) DK] = sqrt(w_s) k_s / (|k_s| + 1e-8), the
//               per-aspect keys side by side, out [N, S DK].  Then
//               <[sqrt(w_s) q_s]_s, [sqrt(w_s) k_s]_s> = sum_s w_s <q_s, k_s>,
//               the score of hybrid_forward (retrieval.py:154-165), is one dot
//               product of length S DK.
template <int DK, bool PACK>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kKpThreads, 1)
    key_project_kernel(const __grid_constant__ CUtensorMap tmap_v,
                       const __grid_constant__ CUtensorMap tmap_w, const KeyProjArgs a) {
  constexpr int S = kKpStages;
  constexpr int kSegs = kTileN / DK;  // aspect segments per projection tile
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  const uint32_t base = (raw_addr + 1023u) & ~1023u;
  uint8_t* smem = smem_raw + (base - raw_addr);
  const uint32_t sA0 = base;
  const uint32_t sB0 = base + kKpStageA;
  uint8_t* bar_area = smem + S * kKpStageBytes;
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
  const uint32_t cta = cluster_cta_rank();
  const bool leader = cta == 0;
  const int pair = blockIdx.x >> 1;
  const int32_t row0 = pair * kKpPairRows + static_cast<int32_t>(cta) * kTileM;

  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(full_bar(s), 1);
      mbar_init(empty_bar(s), 1);
    }
    for (int acc = 0; acc < 2; ++acc) {
      mbar_init(tfull_bar(acc), 1);
      mbar_init(tempty_bar(acc), 8);
    }
    mbar_init(drain_bar, 1);
    *abort_flag = 0;
    *n_issued = 0;
    *n_consumed = 0;
    fence_mbar_init();
    tma_prefetch_desc(&tmap_v);
    tma_prefetch_desc(&tmap_w);
  }
  if (warp == 1) {
    tmem_alloc_pair(smem_u32(tmem_slot), 2 * kTileN);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  cluster_sync();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      const uint64_t pol_v = l2_policy_evict_last();
      const uint64_t pol_w = l2_policy_evict_normal();
      int it = 0;
      bool ok = true;
      for (int t = 0; t < a.n_nt && ok; ++t) {
        const int32_t wrow = t * kTileN + static_cast<int32_t>(cta) * kKpColsPerCta;
        for (int kb = 0; kb < a.num_kb; ++kb, ++it) {
          const int s = it % S;
          const uint32_t r = static_cast<uint32_t>(it / S);
          if (!mbar_wait(empty_bar(s), (r & 1u) ^ 1u, a.status, abort_flag)) {
            ok = false;
            break;
          }
          if (leader) mbar_arrive_expect_tx(full_bar(s), 2 * kKpStageBytes);
          const uint32_t lead_full = map_to_cta(full_bar(s), 0);
          tma_load_2d_pair(sA0 + s * kKpStageBytes, &tmap_v, lead_full, kb * kTileK, row0, pol_v);
          tma_load_2d_pair(sB0 + s * kKpStageBytes, &tmap_w, lead_full, kb * kTileK, wrow, pol_w);
        }
      }
      *n_issued = it;
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ UMMA issuer
    if (leader && lane == 0) {
      constexpr uint32_t idesc = umma_idesc_bf16_f32(kKpPairRows, kTileN);
      int it = 0;
      bool ok = true;
      for (int t = 0; t < a.n_nt && ok; ++t) {
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
          const uint64_t ad = sw128_kmajor_desc(sA0 + s * kKpStageBytes);
          const uint64_t bd = sw128_kmajor_desc(sB0 + s * kKpStageBytes);
#pragma unroll
          for (int kk = 0; kk < kTileK / 16; ++kk)
            umma_bf16_ss_pair(tmem_d, ad + 2u * kk, bd + 2u * kk, idesc, (kb | kk) != 0 ? 1u : 0u);
          umma_commit_pair_all(empty_bar(s), 0x3);
        }
        if (ok) umma_commit_pair_all(tfull_bar(acc), 0x3);
      }
      *n_consumed = it;
      umma_commit_pair_local(drain_bar);
      mbar_wait(drain_bar, 0u, a.status, nullptr);
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int ew = warp & 3;          // TMEM lane quarter
    const int row = ew * 32 + lane;   // pool row within this CTA's 128
    float acc_out[PACK ? 1 : DK];
#pragma unroll
    for (int c = 0; c < (PACK ? 1 : DK); ++c) acc_out[c] = 0.f;
    const int64_t grow = static_cast<int64_t>(row0) + row;
    const uint32_t lead_tempty0 = map_to_cta(tempty_bar(0), 0);
    const uint32_t lead_tempty1 = map_to_cta(tempty_bar(1), 0);
    bool ok = true;
    for (int t = 0; t < a.n_nt; ++t) {
      const int acc = t & 1;
      const uint32_t use = static_cast<uint32_t>(t >> 1);
      const bool got = mbar_wait(tfull_bar(acc), use & 1u, a.status, abort_flag);
      if (!__all_sync(0xffffffffu, got)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const uint32_t taddr =
          tmem_base + (static_cast<uint32_t>(ew * 32) << 16) + static_cast<uint32_t>(acc * kTileN);
#pragma unroll
      for (int sg = 0; sg < kSegs; ++sg) {
        const int s_idx = t * kSegs + sg;  // aspect of this segment (padding beyond S)
        if (s_idx < a.S) {
          // pass 1: squared norm of the row's segment
          float ss = 0.f;
#pragma unroll
          for (int c = 0; c < DK / 32; ++c) {
            float v[32];
            tmem_ld_32x32b_x32_sync(taddr + sg * DK + 32 * c, v);
#pragma unroll
            for (int j = 0; j < 32; ++j) ss = fmaf(v[j], v[j], ss);
          }
          if constexpr (PACK) {
            // pass 2: sqrt(w_s) * segment / (norm + 1e-8), stored as segment s of the row
            const float scale = sqrtf(__ldg(a.w + s_idx)) / (sqrtf(ss) + 1e-8f);
#pragma unroll
            for (int c = 0; c < DK / 32; ++c) {
              float v[32];
              tmem_ld_32x32b_x32_sync(taddr + sg * DK + 32 * c, v);
              if (grow < a.N) {
                uint4* dst = reinterpret_cast<uint4*>(a.out + grow * a.ldo +
                                                      static_cast<int64_t>(s_idx) * DK + 32 * c);
#pragma unroll
                for (int q8 = 0; q8 < 4; ++q8) {
                  uint4 wv;
                  uint32_t* wp = reinterpret_cast<uint32_t*>(&wv);
#pragma unroll
                  for (int q = 0; q < 4; ++q) {
                    const __nv_bfloat162 h2 = __floats2bfloat162_rn(
                        scale * v[8 * q8 + 2 * q], scale * v[8 * q8 + 2 * q + 1]);
                    wp[q] = *reinterpret_cast<const uint32_t*>(&h2);
                  }
                  dst[q8] = wv;
                }
              }
            }
          } else {
            const float scale = __ldg(a.w + s_idx) / (sqrtf(ss) + 1e-8f);
            // pass 2: w_s * segment / (norm + 1e-8) into the collapsed key
#pragma unroll
            for (int c = 0; c < DK / 32; ++c) {
              float v[32];
              tmem_ld_32x32b_x32_sync(taddr + sg * DK + 32 * c, v);
#pragma unroll
              for (int j = 0; j < 32; ++j)
                acc_out[32 * c + j] = fmaf(scale, v[j], acc_out[32 * c + j]);
            }
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(acc ? lead_tempty1 : lead_tempty0);
    }
    if (!PACK && ok && grow < a.N) {
      uint4* dst = reinterpret_cast<uint4*>(a.out + grow * a.ldo);
#pragma unroll
      for (int c = 0; c < DK / 8; ++c) {
        uint4 wv;
        uint32_t* wp = reinterpret_cast<uint32_t*>(&wv);
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const __nv_bfloat162 h2 = __floats2bfloat162_rn(acc_out[8 * c + 2 * q], acc_out[8 * c + 2 * q + 1]);
          wp[q] = *reinterpret_cast<const uint32_t*>(&h2);
        }
        dst[c] = wv;
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (leader && threadIdx.x == 0) {
    for (int i = *n_consumed; i < *n_issued; ++i)
      mbar_wait_cluster(full_bar(i % S), static_cast<uint32_t>(i / S) & 1u, a.status, nullptr);
  }
  tc_fence_before();
  cluster_sync();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, 2 * kTileN);
  }
}

template <int DK, bool PACK>
cudaError_t launch_dk(const CUtensorMap& mv, const CUtensorMap& mw, const KeyProjArgs& args,
                      unsigned grid, cudaStream_t stream) {
  static std::atomic<uint64_t> done{0};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  const uint64_t bit = 1ull << (dev & 63);
  if (!(done.load(std::memory_order_acquire) & bit)) {
    e = cudaFuncSetAttribute(key_project_kernel<DK, PACK>,
                             cudaFuncAttributeMaxDynamicSharedMemorySize, kKpSmemBytes);
    if (e != cudaSuccess) return e;
    done.fetch_or(bit, std::memory_order_acq_rel);
  }
  key_project_kernel<DK, PACK><<<grid, kKpThreads, kKpSmemBytes, stream>>>(mv, mw, args);
  return cudaGetLastError();
}

}  // namespace

cudaError_t launch_project_keys(const void* vectors, int64_t N, int64_t ldv, int D, const void* w_k,
                                int64_t ldw, int S, int d_k, const float* aspect_w, void* keys_out,
                                int64_t ldo, int* status, cudaStream_t stream, bool packed) {
  if (N <= 0) return cudaSuccess;
  CUtensorMap mv, mw;
  const uint64_t wrows = static_cast<uint64_t>(S) * d_k;
  if (!make_bf16_tile_map(&mv, vectors, static_cast<uint64_t>(D), static_cast<uint64_t>(N),
                          static_cast<uint64_t>(ldv), kTileK, kTileM) ||
      !make_bf16_tile_map(&mw, w_k, static_cast<uint64_t>(D), wrows, static_cast<uint64_t>(ldw),
                          kTileK, kKpColsPerCta))
    return cudaErrorInvalidValue;
  KeyProjArgs args;
  args.N = N;
  args.num_kb = (D + kTileK - 1) / kTileK;
  args.n_nt = static_cast<int>((wrows + kTileN - 1) / kTileN);
  args.S = S;
  args.w = aspect_w;
  args.out = static_cast<__nv_bfloat16*>(keys_out);
  args.ldo = ldo;
  args.status = status;
  const unsigned grid = 2u * static_cast<unsigned>((N + kKpPairRows - 1) / kKpPairRows);
  switch (d_k * 2 + (packed ? 1 : 0)) {
    case 64: return launch_dk<32, false>(mv, mw, args, grid, stream);
    case 128: return launch_dk<64, false>(mv, mw, args, grid, stream);
    case 256: return launch_dk<128, false>(mv, mw, args, grid, stream);
    case 65: return launch_dk<32, true>(mv, mw, args, grid, stream);
    case 129: return launch_dk<64, true>(mv, mw, args, grid, stream);
    case 257: return launch_dk<128, true>(mv, mw, args, grid, stream);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace dwa
