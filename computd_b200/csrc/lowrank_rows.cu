// lowrank_rows.cu — row-stationary low-rank weight assembly for sm_100a (B200).
//
// Same result as dwa_lowrank_delta (assembly.cu), the consumer of the
// retrieved pool rows in WeightAssembler.__call__ (src/model/assembly.py:
// 104, 123-127):
//     delta[m] = sum_e alpha[m, e] (U_j (V_j h[m]) + b_j),  j = idx[m, e]
// but organised by pool row instead of by token.  The per-token kernel reads
// every selected row once per token that selected it: at the reference's 1B
// layout (8192 tokens x k = 16 over 16,384 rows of 43.5 KB) that is 5.7 GB of
// row reads from a 713 MB pool.  Here:
//   1. sort the (token, entry) pairs by owned row (pair_sort.cu; the order
//      inside a row is irrelevant: every pair writes its own slot);
//   2. each CTA takes 32 consecutive pairs of that list, stages each row it
//      meets (U | V | b, 43.5 KB) in shared memory once, and one warp per pair
//      computes alpha (U_j (V_j h[m]) + b_j) into the pair's own fp32 slot
//      part[m, e, :] (fixed-size pair chunks keep the load even when a few
//      rows are selected by many tokens);
//   3. one pass sums the k slots of each token in entry order.
// Rows are read about once (1.47x at the 1B layout: rows split between two
// 32-pair chunks are staged by both), the slots cost one write and one read
// of M k d_B floats, and nothing uses float atomics, so the result is the
// same on every run (CUDA-graph replay equals eager execution bit for bit).
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdint>

#include "dwa_internal.h"

namespace dwa {

namespace {

constexpr int kRowThreads = 256;
constexpr int kRowWarps = kRowThreads / 32;
constexpr int kPairsPerCta = 32;

size_t up256(size_t x) { return (x + 255) & ~size_t(255); }

// Workspace: the row-sorted pair list (pair_sort.cu), then the per-pair slots.
float* part_slots(void* ws, int64_t n_pairs, int64_t n_rows) {
  return reinterpret_cast<float*>(static_cast<uint8_t*>(ws) +
                                  up256(pair_sort_workspace_bytes(n_pairs, n_rows)));
}

// ---------------------------------------------------------------- rows x their tokens
struct RowsArgs {
  const void* h;
  int64_t ldh;
  const float* alpha;
  const int32_t* gidx;
  int k;
  const __nv_bfloat16* vectors;
  int64_t row_begin, ldv;
  int d_A, d_B, r;
  int row_words;  // 16-byte words of U | V | b
  const int32_t* offsets;
  const int32_t* pairs;
  int64_t n_rows;
  float* part;
};

__device__ __forceinline__ float bf_lo(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float bf_hi(uint32_t w) { return __uint_as_float(w & 0xFFFF0000u); }

__device__ __forceinline__ float dot8(const uint4 w, const float (&x)[8]) {
  float s = bf_lo(w.x) * x[0];
  s = fmaf(bf_hi(w.x), x[1], s);
  s = fmaf(bf_lo(w.y), x[2], s);
  s = fmaf(bf_hi(w.y), x[3], s);
  s = fmaf(bf_lo(w.z), x[4], s);
  s = fmaf(bf_hi(w.z), x[5], s);
  s = fmaf(bf_lo(w.w), x[6], s);
  s = fmaf(bf_hi(w.w), x[7], s);
  return s;
}

// One warp applies the staged row (U | V | b in row_s) to pair pid:
// hV = alpha V_j h[m] (lanes over d_A, butterfly sums), then
// part[pid, i] = sum_t U_j[i, t] hV[t] + alpha b_j[i] (lanes over i).
template <int RMAX, bool HBF16, bool VEC_U>
__device__ __forceinline__ void apply_pair(const RowsArgs& a, const uint4* row_s, int32_t pid,
                                           int lane, int v_word0, int a_words, int b_elem0) {
  const int r = a.r;
  const __nv_bfloat16* row_bf = reinterpret_cast<const __nv_bfloat16*>(row_s);
  const int64_t m = pid / a.k;
  const float al = a.alpha[pid];
  float acc[RMAX];
#pragma unroll
  for (int t = 0; t < RMAX; ++t) acc[t] = 0.f;
#pragma unroll 4
  for (int c = lane; c < a_words; c += 32) {  // unrolled: the h loads (L2) go out together
    float x[8];
    if constexpr (HBF16) {
      const uint4 hw =
          __ldg(reinterpret_cast<const uint4*>(static_cast<const __nv_bfloat16*>(a.h) +
                                               m * a.ldh) + c);
      x[0] = bf_lo(hw.x); x[1] = bf_hi(hw.x); x[2] = bf_lo(hw.y); x[3] = bf_hi(hw.y);
      x[4] = bf_lo(hw.z); x[5] = bf_hi(hw.z); x[6] = bf_lo(hw.w); x[7] = bf_hi(hw.w);
    } else {
      const float4* hp = reinterpret_cast<const float4*>(static_cast<const float*>(a.h) +
                                                         m * a.ldh) + 2 * c;
      const float4 u0 = __ldg(hp), u1 = __ldg(hp + 1);
      x[0] = u0.x; x[1] = u0.y; x[2] = u0.z; x[3] = u0.w;
      x[4] = u1.x; x[5] = u1.y; x[6] = u1.z; x[7] = u1.w;
    }
#pragma unroll
    for (int t = 0; t < RMAX; ++t)
      if (t < r) acc[t] += dot8(row_s[v_word0 + t * a_words + c], x);
  }
#pragma unroll
  for (int t = 0; t < RMAX; ++t) {
    if (t < r) {
#pragma unroll
      for (int o = 16; o; o >>= 1) acc[t] += __shfl_xor_sync(0xffffffffu, acc[t], o);
      acc[t] *= al;  // every lane holds alpha hV[t]
    }
  }
  float* out = a.part + static_cast<int64_t>(pid) * a.d_B;
#pragma unroll 4
  for (int i = lane; i < a.d_B; i += 32) {
    float u = 0.f;
    if constexpr (VEC_U) {
      const int uw = r >> 3;
#pragma unroll
      for (int c8 = 0; c8 < RMAX / 8; ++c8) {
        if (c8 < uw) {
          float hv8[8];
#pragma unroll
          for (int t = 0; t < 8; ++t) hv8[t] = acc[c8 * 8 + t];
          u += dot8(row_s[i * uw + c8], hv8);
        }
      }
    } else {
#pragma unroll
      for (int t = 0; t < RMAX; ++t)
        if (t < r) u = fmaf(__bfloat162float(row_bf[i * r + t]), acc[t], u);
    }
    out[i] = u + al * __bfloat162float(row_bf[b_elem0 + i]);
  }
}

// CTA = 32 consecutive pairs of the row-sorted list.  Each run of pairs with
// the same row is one segment: the CTA stages that row's U | V | b in shared
// memory (read once from HBM), then warp w takes the segment's pairs w, w + 8,
// ...: hV = alpha V_j h[m] (lanes over d_A, butterfly sums), then
// part[pair, i] = sum_t U_j[i, t] hV[t] + alpha b_j[i] (lanes over i).
// RMAX bounds r (register arrays); VEC_U: r % 8 == 0 (U rows of whole words).
template <int RMAX, bool HBF16, bool VEC_U>
__global__ void __launch_bounds__(kRowThreads) lowrank_rows_kernel(const RowsArgs a) {
  extern __shared__ uint4 row_s[];
  __shared__ int32_t seg_pair[kPairsPerCta];
  __shared__ int32_t seg_row[kPairsPerCta];
  __shared__ int seg_start[kPairsPerCta + 1];
  __shared__ int n_seg_s;

  const int32_t total = a.offsets[a.n_rows];
  const int64_t p0 = static_cast<int64_t>(blockIdx.x) * kPairsPerCta;
  if (p0 >= total) return;
  const int n = static_cast<int>(min(static_cast<int64_t>(kPairsPerCta), total - p0));
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (warp == 0) {
    int32_t pid = 0, row = -1;
    if (lane < n) {
      pid = a.pairs[p0 + lane];
      row = static_cast<int32_t>(a.gidx[pid] - a.row_begin);
      seg_pair[lane] = pid;
      seg_row[lane] = row;
    }
    const int32_t prev = __shfl_up_sync(0xffffffffu, row, 1);
    const bool starts = lane < n && (lane == 0 || row != prev);
    const uint32_t bal = __ballot_sync(0xffffffffu, starts);
    if (starts) seg_start[__popc(bal & ((1u << lane) - 1u))] = lane;
    if (lane == 0) {
      n_seg_s = __popc(bal);
      seg_start[__popc(bal)] = n;
    }
  }
  __syncthreads();
  const int n_seg = n_seg_s;
  const int r = a.r;
  const int a_words = a.d_A >> 3;
  const int v_word0 = (a.d_B * r) >> 3;  // V follows U (d_B x r); both whole words
  const int b_elem0 = a.d_B * r + r * a.d_A;
  for (int sgi = 0; sgi < n_seg; ++sgi) {
    const int q0 = seg_start[sgi], q1 = seg_start[sgi + 1];
    const uint4* src =
        reinterpret_cast<const uint4*>(a.vectors + static_cast<int64_t>(seg_row[q0]) * a.ldv);
    for (int w = threadIdx.x; w < a.row_words; w += kRowThreads) row_s[w] = __ldg(src + w);
    __syncthreads();
    for (int q = q0 + warp; q < q1; q += kRowWarps)
      apply_pair<RMAX, HBF16, VEC_U>(a, row_s, seg_pair[q], lane, v_word0, a_words, b_elem0);
    __syncthreads();  // the next segment overwrites the staged row
  }
}

// ---------------------------------------------------------------- per-token sums
// delta[m, 4c..4c+3] = sum over the owned entries e of part[m k + e, 4c..], in entry order.
__global__ void lowrank_rows_sum_kernel(const float* part, const int32_t* gidx, int64_t M, int k,
                                        int d_B, int64_t row_begin, int64_t row_end,
                                        float* delta) {
  const int q = d_B >> 2;
  const int64_t t = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (t >= M * q) return;
  const int64_t m = t / q;
  const int c = static_cast<int>(t - m * q);
  float4 s = make_float4(0.f, 0.f, 0.f, 0.f);
  for (int e = 0; e < k; ++e) {
    const int32_t g = gidx[m * k + e];
    if (g >= row_begin && g < row_end) {
      const float4 v =
          __ldcs(reinterpret_cast<const float4*>(part + (m * k + e) * d_B) + c);  // read once
      s.x += v.x;
      s.y += v.y;
      s.z += v.z;
      s.w += v.w;
    }
  }
  reinterpret_cast<float4*>(delta + m * d_B)[c] = s;
}

}  // namespace

size_t lowrank_rows_workspace_bytes(int64_t M, int k, int64_t n_rows, int d_B) {
  const int64_t n_pairs = M * k;
  return up256(pair_sort_workspace_bytes(n_pairs, n_rows)) +
         up256(static_cast<size_t>(n_pairs) * static_cast<size_t>(d_B) * 4);
}

int lowrank_rows_smem_bytes(int d_A, int d_B, int r) {
  const int64_t elems = static_cast<int64_t>(d_B) * r + static_cast<int64_t>(r) * d_A + d_B;
  return static_cast<int>(elems * 2);
}

namespace {
template <int RMAX, bool HBF16, bool VEC_U>
cudaError_t launch_rows_variant(const RowsArgs& a, unsigned grid, int smem, cudaStream_t stream) {
  cudaError_t e = cudaFuncSetAttribute(lowrank_rows_kernel<RMAX, HBF16, VEC_U>,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) return e;
  lowrank_rows_kernel<RMAX, HBF16, VEC_U><<<grid, kRowThreads, smem, stream>>>(a);
  return cudaGetLastError();
}
}  // namespace

cudaError_t launch_lowrank_rows(const void* h, int h_bf16, int64_t ldh, const float* alpha,
                                const int32_t* gidx, int64_t M, int k, const void* vectors,
                                int64_t row_begin, int64_t row_end, int64_t ldv, int d_A, int d_B,
                                int r, float* delta, void* ws, cudaStream_t stream) {
  const int64_t n_rows = row_end - row_begin;
  const int64_t n_pairs = M * k;
  const int64_t sum_threads = M * (d_B / 4);
  if (n_rows == 0) {  // nothing owned: the partial sum is zero
    return cudaMemsetAsync(delta, 0, static_cast<size_t>(M) * d_B * 4, stream);
  }
  PairSort sorted;
  cudaError_t e = launch_sort_pairs_by_row(gidx, n_pairs, row_begin, row_end, ws, &sorted, stream);
  if (e != cudaSuccess) return e;
  float* part = part_slots(ws, n_pairs, n_rows);

  RowsArgs a{h, ldh, alpha, gidx, k, static_cast<const __nv_bfloat16*>(vectors), row_begin, ldv,
             d_A, d_B, r, lowrank_rows_smem_bytes(d_A, d_B, r) / 16, sorted.offsets, sorted.pairs,
             n_rows, part};
  const unsigned row_grid = static_cast<unsigned>((n_pairs + kPairsPerCta - 1) / kPairsPerCta);
  const int smem = a.row_words * 16;
  const bool vec_u = r % 8 == 0;
  if (r <= 8) {
    if (h_bf16)
      e = vec_u ? launch_rows_variant<8, true, true>(a, row_grid, smem, stream)
                : launch_rows_variant<8, true, false>(a, row_grid, smem, stream);
    else
      e = vec_u ? launch_rows_variant<8, false, true>(a, row_grid, smem, stream)
                : launch_rows_variant<8, false, false>(a, row_grid, smem, stream);
  } else {
    if (h_bf16)
      e = vec_u ? launch_rows_variant<32, true, true>(a, row_grid, smem, stream)
                : launch_rows_variant<32, true, false>(a, row_grid, smem, stream);
    else
      e = vec_u ? launch_rows_variant<32, false, true>(a, row_grid, smem, stream)
                : launch_rows_variant<32, false, false>(a, row_grid, smem, stream);
  }
  if (e != cudaSuccess) return e;
  lowrank_rows_sum_kernel<<<static_cast<unsigned>((sum_threads + 255) / 256), 256, 0, stream>>>(
      part, gidx, M, k, d_B, row_begin, row_end, delta);
  return cudaGetLastError();
}

}  // namespace dwa
