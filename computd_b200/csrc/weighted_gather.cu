// weighted_gather.cu — alpha normalisation + gathered pool-row weighted sum.
//
// Reference: alpha = top_vals / (sum(top_vals) + 1e-8)   (src/model/retrieval.py:326)
//            selected = vectors[idx]                      (src/model/assembly.py:104)
//            b_delta = einsum('...k,...kj->...j', alpha, b_vecs)   (assembly.py:127)
// The reference gathers [B, seq, k, D] into HBM (and, on a sharded pool, has
// GSPMD all-gather the whole pool first, dwa.py:190-192).  Here one warp owns
// one query row: it normalises the k weights, compacts the entries whose rows
// this shard owns, then streams those bf16 rows with 16-byte read-only loads
// and accumulates in fp32 registers.  The [M, k, d] gather is never stored.
#include <cuda_runtime.h>

#include <cstdint>

#include "dwa_internal.h"

namespace dwa {

namespace {

constexpr int kWarps = 8;
constexpr int kMaxGatherK = 128;

struct GatherArgs {
  const float* vals;
  const int32_t* gidx;
  const uint16_t* values;
  int64_t M, row_begin, row_end, ldv;
  int k, d;
  float* out;
  float* alpha_out;
};

__device__ __forceinline__ void bf16x8_to_f32(const uint4 x, float (&f)[8]) {
  f[0] = __uint_as_float(x.x << 16);
  f[1] = __uint_as_float(x.x & 0xFFFF0000u);
  f[2] = __uint_as_float(x.y << 16);
  f[3] = __uint_as_float(x.y & 0xFFFF0000u);
  f[4] = __uint_as_float(x.z << 16);
  f[5] = __uint_as_float(x.z & 0xFFFF0000u);
  f[6] = __uint_as_float(x.w << 16);
  f[7] = __uint_as_float(x.w & 0xFFFF0000u);
}

__global__ void __launch_bounds__(kWarps * 32) weighted_gather_kernel(const GatherArgs a) {
  __shared__ float s_alpha[kWarps][kMaxGatherK];
  __shared__ int32_t s_row[kWarps][kMaxGatherK];
  const int w = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int64_t m = static_cast<int64_t>(blockIdx.x) * kWarps + w;
  if (m >= a.M) return;  // warp-uniform; only warp-level synchronisation below

  const float* v = a.vals + m * a.k;
  const int32_t* g = a.gidx + m * a.k;

  // Sum of the k fused scores: lane-strided partial sums, then a fixed butterfly.
  float part = 0.f;
  for (int j = lane; j < a.k; j += 32) part += v[j];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) part += __shfl_xor_sync(0xffffffffu, part, o);
  const float denom = part + 1e-8f;

  // Normalise and compact the entries owned by this shard (order preserved).
  int n_own = 0;
  for (int j0 = 0; j0 < a.k; j0 += 32) {
    const int j = j0 + lane;
    float al = 0.f;
    int32_t gi = -1;
    if (j < a.k) {
      al = v[j] / denom;
      gi = g[j];
      if (a.alpha_out) a.alpha_out[m * a.k + j] = al;
    }
    const bool own = j < a.k && gi >= a.row_begin && gi < a.row_end;
    const uint32_t mask = __ballot_sync(0xffffffffu, own);
    if (own) {
      const int pos = n_own + __popc(mask & ((1u << lane) - 1u));
      s_alpha[w][pos] = al;
      s_row[w][pos] = static_cast<int32_t>(gi - a.row_begin);
    }
    n_own += __popc(mask);
  }
  __syncwarp();
  if (a.out == nullptr) return;  // alpha only

  float* orow = a.out + m * a.d;
  for (int c0 = 0; c0 < a.d; c0 += 256) {
    const int col = c0 + lane * 8;
    if (col >= a.d) continue;  // d % 8 == 0: a lane's 8 columns are all in range or all out
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    int j = 0;
    for (; j + 4 <= n_own; j += 4) {
      uint4 x[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const uint16_t* src = a.values + static_cast<int64_t>(s_row[w][j + u]) * a.ldv + col;
        x[u] = __ldg(reinterpret_cast<const uint4*>(src));
      }
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        float f[8];
        bf16x8_to_f32(x[u], f);
        const float al = s_alpha[w][j + u];
#pragma unroll
        for (int e = 0; e < 8; ++e) acc[e] = fmaf(al, f[e], acc[e]);
      }
    }
    for (; j < n_own; ++j) {
      const uint16_t* src = a.values + static_cast<int64_t>(s_row[w][j]) * a.ldv + col;
      float f[8];
      bf16x8_to_f32(__ldg(reinterpret_cast<const uint4*>(src)), f);
      const float al = s_alpha[w][j];
#pragma unroll
      for (int e = 0; e < 8; ++e) acc[e] = fmaf(al, f[e], acc[e]);
    }
    float4* dst = reinterpret_cast<float4*>(orow + col);
    dst[0] = make_float4(acc[0], acc[1], acc[2], acc[3]);
    dst[1] = make_float4(acc[4], acc[5], acc[6], acc[7]);
  }
}

}  // namespace

cudaError_t launch_weighted_gather(const float* vals, const int32_t* gidx, int64_t M, int k,
                                   const void* values, int64_t row_begin, int64_t row_end,
                                   int64_t ldv, int d, float* out, float* alpha_out,
                                   cudaStream_t stream) {
  if (M <= 0) return cudaSuccess;
  if (k > kMaxGatherK) return cudaErrorInvalidValue;
  GatherArgs a;
  a.vals = vals;
  a.gidx = gidx;
  a.values = static_cast<const uint16_t*>(values);
  a.M = M;
  a.row_begin = row_begin;
  a.row_end = row_end;
  a.ldv = ldv;
  a.k = k;
  a.d = d;
  a.out = out;
  a.alpha_out = alpha_out;
  const int64_t blocks = (M + kWarps - 1) / kWarps;
  weighted_gather_kernel<<<static_cast<unsigned>(blocks), kWarps * 32, 0, stream>>>(a);
  return cudaGetLastError();
}

}  // namespace dwa
