// seq_scores.cu — the sequence-mean auxiliary scores of the retrieval.
//
// pallas_hybrid_forward (src/model/retrieval.py:332-341) returns, besides the
// per-position top-k, one score row per sequence for its auxiliary losses:
//     sims_seq[b, n]      = <q_mean_w[b], keys_w[n]>            (336)
//     alpha_raw_seq[b, n] = sigmoid(lambda (sims - tau)) * exp(sims / T)
//                           or exp(sims / T)                    (338-341)
// for the B sequence-mean queries (B = batch, a handful of rows) against every
// key of the shard.  With B this small the product is a skinny
// [B, d] x [d, N] whose cost is reading the key shard once from HBM.  Two
// kernels:
//  * seq_scores_mma_kernel (B <= 10 and the split query operand fits in
//    shared memory): tcgen05 with TMA-streamed key tiles, the fp32 queries as
//    three exact bf16 parts, fp32 accumulation; it runs at HBM speed;
//  * seq_scores_kernel otherwise, on the CUDA cores: each warp streams KR key
//    rows at a time with 16-byte loads (the next chunk's loads are in flight
//    while the current chunk's FMAs run), the QB queries of a pass sit in
//    shared memory in fp32 (the reference computes this product in fp32), and
//    the KR x QB dot products of a warp are summed across its lanes with one
//    transpose-reduction; B > QB takes several passes over the keys.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdint>

#include "dwa_internal.h"
#include "score_params.cuh"
#include "sm100_ptx.cuh"

namespace dwa {

namespace {

constexpr int kSeqWarps = 8;    // warps per block
constexpr int kSeqRows = 8;     // key rows per warp per step
constexpr int kSmemLimit = 200 * 1024;

struct SeqArgs {
  const float* q;
  int64_t B, ldq;
  const uint16_t* keys;
  int64_t N, ldk;
  int d;
  const float* params;
  int use_sigmoid;
  float* sims;
  int64_t lds;
  float* fused;
  int64_t ldf;
  int* status;
};

__device__ __forceinline__ uint4 ld_stream16(const void* p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

__device__ __forceinline__ float bf16_lo(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float bf16_hi(uint32_t w) { return __uint_as_float(w & 0xFFFF0000u); }

// Shared-memory query layout: element 8c + 4h + e of query row i lives at
// float4 index (2 i + h) * (d / 8) + c, so lane l's float4 loads for chunk c
// are consecutive across the warp (no bank conflicts).
template <int QB>
__global__ void __launch_bounds__(kSeqWarps * 32, 1) seq_scores_kernel(const SeqArgs a) {
  extern __shared__ float4 sq[];
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int n_chunks = a.d >> 3;  // 16-byte key chunks per row
  const ScoreParams sp = load_score_params(a.params, 1.0f, 0.0f, 1.0f);
  const bool params_ok = score_params_ok(sp, a.use_sigmoid);
  if (!params_ok && blockIdx.x == 0 && threadIdx.x == 0) record_status(a.status, kStatusDeviceCheck);

  for (int64_t q0 = 0; q0 < a.B; q0 += QB) {
    const int nq = static_cast<int>(a.B - q0 < QB ? a.B - q0 : QB);
    __syncthreads();  // the previous pass is done with the queries
    for (int t = threadIdx.x; t < QB * n_chunks * 2; t += blockDim.x) {
      const int c = t % n_chunks;
      const int ih = t / n_chunks;  // 2 i + h
      const int i = ih >> 1, h = ih & 1;
      float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
      if (i < nq) {
        const float* src = a.q + (q0 + i) * a.ldq + 8 * c + 4 * h;
        v = make_float4(src[0], src[1], src[2], src[3]);
      }
      sq[static_cast<size_t>(ih) * n_chunks + c] = v;
    }
    __syncthreads();

    const int64_t stride = static_cast<int64_t>(gridDim.x) * kSeqWarps * kSeqRows;
    for (int64_t r0 = (static_cast<int64_t>(blockIdx.x) * kSeqWarps + warp) * kSeqRows; r0 < a.N;
         r0 += stride) {
      float acc[QB * kSeqRows];
#pragma unroll
      for (int e = 0; e < QB * kSeqRows; ++e) acc[e] = 0.f;
      const uint16_t* rowp[kSeqRows];
      bool in[kSeqRows];
#pragma unroll
      for (int r = 0; r < kSeqRows; ++r) {
        in[r] = r0 + r < a.N;
        rowp[r] = a.keys + (in[r] ? (r0 + r) : r0) * a.ldk;
      }
      uint4 cur[kSeqRows];
      int c = lane;
#pragma unroll
      for (int r = 0; r < kSeqRows; ++r)
        cur[r] = (c < n_chunks && in[r]) ? ld_stream16(rowp[r] + 8 * c) : make_uint4(0, 0, 0, 0);
      for (; c < n_chunks; c += 32) {
        uint4 nxt[kSeqRows];
        const int cn = c + 32;
#pragma unroll
        for (int r = 0; r < kSeqRows; ++r)
          nxt[r] = (cn < n_chunks && in[r]) ? ld_stream16(rowp[r] + 8 * cn) : make_uint4(0, 0, 0, 0);
#pragma unroll
        for (int i = 0; i < QB; ++i) {
          const float4 qa = sq[static_cast<size_t>(2 * i) * n_chunks + c];
          const float4 qb = sq[static_cast<size_t>(2 * i + 1) * n_chunks + c];
#pragma unroll
          for (int r = 0; r < kSeqRows; ++r) {
            float s = acc[i * kSeqRows + r];
            s = fmaf(qa.x, bf16_lo(cur[r].x), s);
            s = fmaf(qa.y, bf16_hi(cur[r].x), s);
            s = fmaf(qa.z, bf16_lo(cur[r].y), s);
            s = fmaf(qa.w, bf16_hi(cur[r].y), s);
            s = fmaf(qb.x, bf16_lo(cur[r].z), s);
            s = fmaf(qb.y, bf16_hi(cur[r].z), s);
            s = fmaf(qb.z, bf16_lo(cur[r].w), s);
            s = fmaf(qb.w, bf16_hi(cur[r].w), s);
            acc[i * kSeqRows + r] = s;
          }
        }
#pragma unroll
        for (int r = 0; r < kSeqRows; ++r) cur[r] = nxt[r];
      }
      // Transpose-reduction over the 32 lanes: each halving step keeps one
      // half of the values and adds the partner lane's copy of it, so after
      // log2(32) steps lane l holds the full sums of values 2l and 2l + 1
      // (QB * kSeqRows = 64) or of value l (= 32).
      constexpr int V = QB * kSeqRows;
      static_assert(V == 32 || V == 64, "the reduction below handles 32 or 64 values");
#pragma unroll
      for (int step = 0; step < 5; ++step) {
        const int o = 16 >> step;       // partner lane distance
        const int H = V >> (step + 1);  // values kept after this step
        const bool up = (lane & o) != 0;
#pragma unroll
        for (int i = 0; i < H; ++i) {
          const float send = up ? acc[i] : acc[i + H];
          const float keep = up ? acc[i + H] : acc[i];
          acc[i] = keep + __shfl_xor_sync(0xffffffffu, send, o);
        }
      }
      constexpr int kPer = V / 32;  // values per lane after the reduction
#pragma unroll
      for (int j = 0; j < kPer; ++j) {
        const int e = kPer * lane + j;
        const int i = e / kSeqRows, r = e % kSeqRows;
        const int64_t n = r0 + r;
        if (i < nq && n < a.N) {
          const float s = acc[j];
          a.sims[(q0 + i) * a.lds + n] = s;
          if (a.fused != nullptr) {
            float v = NAN;
            if (params_ok) {
              v = expf(s / sp.T);
              if (a.use_sigmoid) v *= 1.0f / (1.0f + expf(-(sp.lambda_sharp * (s - sp.tau))));
            }
            a.fused[(q0 + i) * a.ldf + n] = v;
          }
        }
      }
    }
  }
}

template <int QB>
cudaError_t launch_qb(const SeqArgs& a, cudaStream_t stream) {
  const size_t smem = static_cast<size_t>(QB) * a.d * 4;
  cudaError_t e = cudaFuncSetAttribute(seq_scores_kernel<QB>,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       static_cast<int>(smem));
  if (e != cudaSuccess) return e;
  int dev = 0, sms = 148;
  if (cudaGetDevice(&dev) == cudaSuccess)
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int64_t per_block = static_cast<int64_t>(kSeqWarps) * kSeqRows;
  const int64_t blocks = std::min<int64_t>((a.N + per_block - 1) / per_block, sms);
  seq_scores_kernel<QB><<<static_cast<unsigned>(blocks), kSeqWarps * 32, smem, stream>>>(a);
  return cudaGetLastError();
}

// ---------------------------------------------------------------- tensor-core path
// For up to kSqMaxQ queries whose split operand fits in shared memory: the
// product runs on the tensor cores as D[128 keys x npad] = K_tile . Qs^T, the
// key tiles streamed by TMA through a kSqStages-deep ring and the accumulators
// double-buffered in TMEM, so the kernel is bound by reading the keys once
// from HBM, not by CUDA-core issue.  The fp32 queries enter the bf16 MMA as
// three bf16 parts q = hi + mid + lo (hi = bf16(q), mid = bf16(q - hi),
// lo = bf16(q - hi - mid), which represent q exactly), rows 3 b + p of the
// staged operand: every product with a bf16 key is exact in fp32 and the MMA
// accumulates in fp32, so sims = (D[3b] + D[3b+1]) + D[3b+2] keeps the fp32
// product of the reference.  Persistent CTAs take key tiles t = blockIdx.x +
// i gridDim.x; warp 0 issues the TMA loads, warp 1 the MMAs, warps 2-5 read
// the accumulators (one key per thread) and write sims / fused.
constexpr int kSqKeys = 128;     // keys per tile = TMEM lanes
constexpr int kSqK = 64;         // d per k-block: 128-byte rows
constexpr int kSqStages = 4;
constexpr int kSqThreads = 192;
constexpr int kSqMaxQ = 10;      // 3 parts each: <= 30 of the 32 accumulator columns
constexpr int kSqStageBytes = kSqKeys * kSqK * 2;  // 16 KB
constexpr int kSqBarBytes = 256;

struct SeqMmaArgs {
  const float* q;
  int64_t ldq;
  int nq;        // queries of this launch (<= kSqMaxQ)
  int npad;      // operand rows: 3 nq rounded up to 16
  int64_t N;
  int d, num_kb;
  int64_t n_tiles;
  const float* params;
  int use_sigmoid;
  float* sims;
  int64_t lds;
  float* fused;
  int64_t ldf;
  int* status;
};

size_t seq_mma_smem_bytes(int npad, int num_kb) {
  return 1024 + static_cast<size_t>(num_kb) * npad * 128 +
         static_cast<size_t>(kSqStages) * kSqStageBytes + kSqBarBytes;
}

__global__ void __launch_bounds__(kSqThreads, 1)
    seq_scores_mma_kernel(const __grid_constant__ CUtensorMap tmap_k, const SeqMmaArgs a) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_addr = smem_u32(smem_raw);
  const uint32_t base = (raw_addr + 1023u) & ~1023u;
  uint8_t* smem = smem_raw + (base - raw_addr);
  const uint32_t q_tile_bytes = static_cast<uint32_t>(a.npad) * 128u;  // one k-block of the operand
  const uint32_t qop = base;
  const uint32_t ring = base + static_cast<uint32_t>(a.num_kb) * q_tile_bytes;
  uint8_t* bar_area = smem + static_cast<size_t>(a.num_kb) * q_tile_bytes +
                      static_cast<size_t>(kSqStages) * kSqStageBytes;
  const uint32_t bar0 = smem_u32(bar_area);
  auto full_bar = [&](int s) { return bar0 + 8u * s; };
  auto empty_bar = [&](int s) { return bar0 + 8u * (kSqStages + s); };
  auto tfull_bar = [&](int acc) { return bar0 + 8u * (2 * kSqStages + acc); };
  auto tempty_bar = [&](int acc) { return bar0 + 8u * (2 * kSqStages + 2 + acc); };
  const uint32_t drain_bar = bar0 + 8u * (2 * kSqStages + 4);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bar_area + 8 * (2 * kSqStages + 5));
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  int* n_issued = reinterpret_cast<int*>(tmem_slot + 2);
  int* n_consumed = reinterpret_cast<int*>(tmem_slot + 3);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t my_tiles =
      blockIdx.x < a.n_tiles ? (a.n_tiles - 1 - blockIdx.x) / gridDim.x + 1 : 0;

  // The split-query operand, all k-blocks, in the TMA 128-byte-swizzle layout
  // (row r, 16-byte chunk c of a k-block at (r / 8) 1024 + (r % 8) 128 +
  // ((c ^ (r % 8)) 16)); zeros beyond d and beyond 3 nq rows.
  const int chunks = a.num_kb * a.npad * 8;
  for (int idx = threadIdx.x; idx < chunks; idx += blockDim.x) {
    const int kb = idx / (a.npad * 8);
    const int rem = idx - kb * a.npad * 8;
    const int r = rem >> 3, c = rem & 7;
    const int b = r / 3, part = r - 3 * b;
    uint32_t w[4];
#pragma unroll
    for (int e2 = 0; e2 < 4; ++e2) {
      uint32_t h2 = 0;
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int col = kb * kSqK + c * 8 + 2 * e2 + h;
        const float x = (b < a.nq && col < a.d) ? __ldg(a.q + b * a.ldq + col) : 0.f;
        const __nv_bfloat16 hi = __float2bfloat16_rn(x);
        const float r1 = x - __bfloat162float(hi);
        const __nv_bfloat16 mid = __float2bfloat16_rn(r1);
        const __nv_bfloat16 lo = __float2bfloat16_rn(r1 - __bfloat162float(mid));
        const __nv_bfloat16 v = part == 0 ? hi : part == 1 ? mid : lo;
        h2 |= static_cast<uint32_t>(__bfloat16_as_ushort(v)) << (16 * h);
      }
      w[e2] = h2;
    }
    const uint32_t off = static_cast<uint32_t>(kb) * q_tile_bytes + (r >> 3) * 1024u +
                         (r & 7) * 128u + static_cast<uint32_t>((c ^ (r & 7)) * 16);
    *reinterpret_cast<uint4*>(smem + off) = make_uint4(w[0], w[1], w[2], w[3]);
  }
  fence_proxy_async_smem();
  if (threadIdx.x == 0) {
    for (int s = 0; s < kSqStages; ++s) {
      mbar_init(full_bar(s), 1);
      mbar_init(empty_bar(s), 1);
    }
    for (int acc = 0; acc < 2; ++acc) {
      mbar_init(tfull_bar(acc), 1);
      mbar_init(tempty_bar(acc), 4);  // the four epilogue warps
    }
    mbar_init(drain_bar, 1);
    *abort_flag = 0;
    *n_issued = 0;
    *n_consumed = 0;
    fence_mbar_init();
    tma_prefetch_desc(&tmap_k);
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(tmem_slot), 64);  // two accumulators of 32 columns
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      const uint64_t pol = l2_policy_evict_first();  // the keys are read once
      int it = 0;
      bool ok = true;
      for (int64_t i = 0; i < my_tiles && ok; ++i) {
        const int32_t krow = static_cast<int32_t>((blockIdx.x + i * gridDim.x) * kSqKeys);
        for (int kb = 0; kb < a.num_kb; ++kb, ++it) {
          const int s = it % kSqStages;
          const uint32_t ph = static_cast<uint32_t>(it / kSqStages);
          if (!mbar_wait(empty_bar(s), (ph & 1u) ^ 1u, a.status, abort_flag)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(full_bar(s), kSqStageBytes);
          tma_load_2d(ring + s * kSqStageBytes, &tmap_k, full_bar(s), kb * kSqK, krow, pol);
        }
      }
      *n_issued = it;
    }
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t idesc = umma_idesc_bf16_f32(kSqKeys, a.npad);
      int it = 0;
      bool ok = true;
      for (int64_t i = 0; i < my_tiles && ok; ++i) {
        const int acc = static_cast<int>(i & 1);
        const uint32_t use = static_cast<uint32_t>(i >> 1);
        if (!mbar_wait(tempty_bar(acc), (use & 1u) ^ 1u, a.status, abort_flag)) break;
        tc_fence_after();
        const uint32_t tmem_d = tmem_base + static_cast<uint32_t>(acc * 32);
        for (int kb = 0; kb < a.num_kb; ++kb, ++it) {
          const int s = it % kSqStages;
          const uint32_t ph = static_cast<uint32_t>(it / kSqStages);
          if (!mbar_wait(full_bar(s), ph & 1u, a.status, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t ad = sw128_kmajor_desc(ring + s * kSqStageBytes);
          const uint64_t bd = sw128_kmajor_desc(qop + static_cast<uint32_t>(kb) * q_tile_bytes);
#pragma unroll
          for (int kk = 0; kk < kSqK / 16; ++kk)
            umma_bf16_ss(tmem_d, ad + 2u * kk, bd + 2u * kk, idesc, (kb | kk) != 0 ? 1u : 0u);
          umma_commit(empty_bar(s));
        }
        if (ok) umma_commit(tfull_bar(acc));
      }
      *n_consumed = it;
      // every MMA must finish (it writes TMEM, reads shared memory) before release
      umma_commit(drain_bar);
      mbar_wait(drain_bar, 0u, a.status, nullptr);
    }
  } else {
    const int quarter = warp & 3;  // TMEM lanes this warp may read
    const int row = quarter * 32 + lane;
    const ScoreParams sp = load_score_params(a.params, 1.0f, 0.0f, 1.0f);
    const bool params_ok = score_params_ok(sp, a.use_sigmoid);
    if (!params_ok && blockIdx.x == 0 && threadIdx.x == 64) record_status(a.status, kStatusDeviceCheck);
    for (int64_t i = 0; i < my_tiles; ++i) {
      const int acc = static_cast<int>(i & 1);
      const uint32_t use = static_cast<uint32_t>(i >> 1);
      const bool got = mbar_wait(tfull_bar(acc), use & 1u, a.status, abort_flag);
      if (!__all_sync(0xffffffffu, got)) break;
      tc_fence_after();
      float v[32];
      tmem_ld_32x32b_x32_sync(tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) +
                                  static_cast<uint32_t>(acc * 32),
                              v);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(tempty_bar(acc));
      const int64_t n = (blockIdx.x + i * gridDim.x) * kSqKeys + row;
      if (n < a.N) {
#pragma unroll
        for (int b = 0; b < kSqMaxQ; ++b) {
          if (b < a.nq) {
            const float sv = (v[3 * b] + v[3 * b + 1]) + v[3 * b + 2];
            a.sims[b * a.lds + n] = sv;
            if (a.fused != nullptr) {
              float f = NAN;
              if (params_ok) {
                f = expf(sv / sp.T);
                if (a.use_sigmoid) f *= 1.0f / (1.0f + expf(-(sp.lambda_sharp * (sv - sp.tau))));
              }
              a.fused[b * a.ldf + n] = f;
            }
          }
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (threadIdx.x == 0) {
    // Loads issued but never consumed (only after an abort) must land before exit.
    for (int i = *n_consumed; i < *n_issued; ++i)
      mbar_wait(full_bar(i % kSqStages), static_cast<uint32_t>(i / kSqStages) & 1u, a.status, nullptr);
  }
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, 64);
  }
}

}  // namespace

cudaError_t launch_seq_scores(const float* q, int64_t B, int64_t ldq, const void* keys, int64_t N,
                              int64_t ldk, int d, const float* params, int use_sigmoid,
                              float* sims, int64_t lds, float* fused, int64_t ldf, int* status,
                              cudaStream_t stream) {
  if (B <= 0 || N <= 0) return cudaSuccess;
  // Tensor cores when all queries fit one launch and their split operand
  // leaves the ring its stages; CUDA cores otherwise.
  if (B <= kSqMaxQ) {
    const int npad = static_cast<int>((3 * B + 15) / 16 * 16);
    const int num_kb = (d + kSqK - 1) / kSqK;
    const size_t smem = seq_mma_smem_bytes(npad, num_kb);
    CUtensorMap mk;
    if (smem <= 232448 && (reinterpret_cast<uintptr_t>(keys) & 15u) == 0 && ldk % 8 == 0 &&
        N <= INT32_MAX - kSqKeys &&
        make_bf16_tile_map(&mk, keys, static_cast<uint64_t>(d), static_cast<uint64_t>(N),
                           static_cast<uint64_t>(ldk), kSqK, kSqKeys)) {
      SeqMmaArgs m{q, ldq, static_cast<int>(B), npad, N, d, num_kb,
                   (N + kSqKeys - 1) / kSqKeys, params, use_sigmoid, sims, lds, fused, ldf,
                   status};
      cudaError_t e = cudaFuncSetAttribute(seq_scores_mma_kernel,
                                           cudaFuncAttributeMaxDynamicSharedMemorySize,
                                           static_cast<int>(smem));
      if (e != cudaSuccess) return e;
      const int64_t grid = std::min<int64_t>(m.n_tiles, device_sm_count());
      seq_scores_mma_kernel<<<static_cast<unsigned>(grid), kSqThreads, smem, stream>>>(mk, m);
      return cudaGetLastError();
    }
  }
  SeqArgs a{q, B, ldq, static_cast<const uint16_t*>(keys), N, ldk, d, params, use_sigmoid,
            sims, lds, fused, ldf, status};
  if (B <= 4 && 4ll * 4 * d <= kSmemLimit) return launch_qb<4>(a, stream);
  if (8ll * 4 * d <= kSmemLimit) return launch_qb<8>(a, stream);
  if (4ll * 4 * d <= kSmemLimit) return launch_qb<4>(a, stream);
  return cudaErrorInvalidValue;
}

int seq_scores_max_d() { return kSmemLimit / 16; }

}  // namespace dwa
