// seq_scores.cu — the sequence-mean auxiliary scores of the retrieval.
//
// pallas_hybrid_forward (src/model/retrieval.py:332-341) returns, besides the
// per-position top-k, one score row per sequence for its auxiliary losses:
//     sims_seq[b, n]      = <q_mean_w[b], keys_w[n]>            (336)
//     alpha_raw_seq[b, n] = sigmoid(lambda (sims - tau)) * exp(sims / T)
//                           or exp(sims / T)                    (338-341)
// for the B sequence-mean queries (B = batch, a handful of rows) against every
// key of the shard.  With B this small the product is a skinny
// [B, d] x [d, N] whose cost is reading the key shard once from HBM, so it
// runs on the CUDA cores, not the tensor pipe: each warp streams KR key rows
// at a time with 16-byte loads (the next chunk's loads are in flight while the
// current chunk's FMAs run), the QB queries of a pass sit in shared memory in
// fp32 (the reference computes this product in fp32), and the KR x QB dot
// products of a warp are summed across its lanes with one transpose-reduction.
// B > QB takes several passes over the keys.
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdint>

#include "dwa_internal.h"
#include "score_params.cuh"

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

}  // namespace

cudaError_t launch_seq_scores(const float* q, int64_t B, int64_t ldq, const void* keys, int64_t N,
                              int64_t ldk, int d, const float* params, int use_sigmoid,
                              float* sims, int64_t lds, float* fused, int64_t ldf, int* status,
                              cudaStream_t stream) {
  if (B <= 0 || N <= 0) return cudaSuccess;
  SeqArgs a{q, B, ldq, static_cast<const uint16_t*>(keys), N, ldk, d, params, use_sigmoid,
            sims, lds, fused, ldf, status};
  if (B <= 4 && 4ll * 4 * d <= kSmemLimit) return launch_qb<4>(a, stream);
  if (8ll * 4 * d <= kSmemLimit) return launch_qb<8>(a, stream);
  if (4ll * 4 * d <= kSmemLimit) return launch_qb<4>(a, stream);
  return cudaErrorInvalidValue;
}

int seq_scores_max_d() { return kSmemLimit / 16; }

}  // namespace dwa
