// merge_topk.cu — k-way merge of per-split / per-shard top-k candidate lists.
//
// Two callers:
//  * dwa_score_topk: merges the key-range splits of the fused kernel (raw
//    scores s), sorts, evaluates v(s) = [sigmoid(lambda (s - tau))] * exp(s / T)
//    on the k survivors (tiled_topk.py:172-175) and adds the shard's global
//    index offset (retrieval.py:292-293).
//  * dwa_merge_topk: the cross-shard merge after the all-gather, i.e. the
//    transpose/reshape + top_k + take of _chip_topk (retrieval.py:299-302).
//    Flattening [P, M, k] chip-major and taking top_k with lower position first
//    among ties equals ordering by (v desc, global index asc), because shard p's
//    global indices all precede shard p+1's and each list is already sorted.
//
// One thread per query row; its k-entry heap sits in shared memory.
#include <cuda_runtime.h>

#include <cmath>

#include "dwa_internal.h"
#include "topk_heap.cuh"

namespace dwa {

namespace {

struct MergeArgs {
  const float* cv;
  const int32_t* ci;
  int64_t stride_list, stride_pos, stride_row;
  int64_t M;
  int64_t idx_offset;
  int n_lists, k_in, k;
  int transform, use_sigmoid;
  float lambda_sharp, tau, T;
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

template <int TPB>
__global__ void __launch_bounds__(TPB) merge_topk_kernel(const MergeArgs a) {
  extern __shared__ uint8_t smem[];
  float* hs = reinterpret_cast<float*>(smem);
  int32_t* hi = reinterpret_cast<int32_t*>(smem + static_cast<size_t>(a.k) * TPB * 4);
  const int t = threadIdx.x;
  const int64_t row = static_cast<int64_t>(blockIdx.x) * TPB + t;
  if (row >= a.M) return;  // each thread touches only its own heap column

  const SmemHeap heap{hs, hi, TPB, a.k};
  heap.init(t);
  float rs = -INFINITY;
  int32_t ri = kSentinelIdx;
  for (int l = 0; l < a.n_lists; ++l) {
    const float* vp = a.cv + l * a.stride_list + row * a.stride_row;
    const int32_t* ip = a.ci + l * a.stride_list + row * a.stride_row;
    int p = 0;
    for (; p + 4 <= a.k_in; p += 4) {
      float s[4];
      int32_t ix[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        s[u] = __ldg(vp + (p + u) * a.stride_pos);
        ix[u] = __ldg(ip + (p + u) * a.stride_pos);
      }
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        if (topk_worse(rs, ri, s[u], ix[u])) {
          heap.replace_root(t, s[u], ix[u]);
          rs = heap.S(0, t);
          ri = heap.I(0, t);
        }
      }
    }
    for (; p < a.k_in; ++p) {
      const float s = __ldg(vp + p * a.stride_pos);
      const int32_t ix = __ldg(ip + p * a.stride_pos);
      if (topk_worse(rs, ri, s, ix)) {
        heap.replace_root(t, s, ix);
        rs = heap.S(0, t);
        ri = heap.I(0, t);
      }
    }
  }
  heap.sort_best_first(t);

  if (a.transform) {
    for (int p = 0; p < a.k; ++p)
      heap.S(p, t) = fused_score(heap.S(p, t), a.use_sigmoid, a.lambda_sharp, a.tau, a.T);
    // v is non-decreasing in s, so the list is ordered by v already; entries
    // whose v became equal must still be ordered by lower index first.
    for (int p = 1; p < a.k; ++p) {
      const float vs = heap.S(p, t);
      const int32_t vi = heap.I(p, t);
      int q = p - 1;
      while (q >= 0 && topk_worse(heap.S(q, t), heap.I(q, t), vs, vi)) {
        heap.S(q + 1, t) = heap.S(q, t);
        heap.I(q + 1, t) = heap.I(q, t);
        --q;
      }
      heap.S(q + 1, t) = vs;
      heap.I(q + 1, t) = vi;
    }
  }

  float* ov = a.out_v + row * a.k;
  int32_t* oi = a.out_i + row * a.k;
  for (int p = 0; p < a.k; ++p) {
    const int32_t ix = heap.I(p, t);
    ov[p] = heap.S(p, t);
    oi[p] = ix == kSentinelIdx ? -1 : static_cast<int32_t>(ix + a.idx_offset);
  }
}

template <int TPB>
cudaError_t launch_tpb(const MergeArgs& a, cudaStream_t stream) {
  const size_t smem = static_cast<size_t>(a.k) * TPB * 8;
  if (smem > 48 * 1024) {
    cudaError_t e =
        cudaFuncSetAttribute(merge_topk_kernel<TPB>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(smem));
    if (e != cudaSuccess) return e;
  }
  const int64_t blocks = (a.M + TPB - 1) / TPB;
  merge_topk_kernel<TPB><<<static_cast<unsigned>(blocks), TPB, smem, stream>>>(a);
  return cudaGetLastError();
}

}  // namespace

cudaError_t launch_merge_topk(const float* cand_vals, const int32_t* cand_idx, int n_lists,
                              int k_in, int64_t stride_list, int64_t stride_pos,
                              int64_t stride_row, int64_t M, int k, int transform,
                              float lambda_sharp, float tau, float T, int use_sigmoid,
                              int64_t idx_offset, float* out_vals, int32_t* out_idx,
                              cudaStream_t stream) {
  if (M <= 0) return cudaSuccess;
  MergeArgs a;
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
  a.out_v = out_vals;
  a.out_i = out_idx;
  // Keep the per-block heap at <= 32 KB so several blocks share an SM.
  if (k <= 64) return launch_tpb<64>(a, stream);
  return launch_tpb<32>(a, stream);
}

}  // namespace dwa
