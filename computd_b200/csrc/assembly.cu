// assembly.cu — the low-rank weight-assembly consumer of the retrieved pool
// rows, and the pool-usage EMA, for sm_100a (B200).
//
// Reference: WeightAssembler.__call__, per-position (hybrid) idx
// (src/model/assembly.py:75-128).  Each pool row is [U (d_B x r) | V (r x d_A)
// | b (d_B) | unused], row-major blocks (assembly.py:10-14, 110-112):
//     selected = vectors[idx]                               (assembly.py:104)
//     hV       = einsum('...d,...krd->...kr', h_A, V)        (assembly.py:125)
//     h_delta  = einsum('...kr,...kir->...i', hV*alpha, U)   (assembly.py:126)
//     b_delta  = einsum('...k,...kj->...j', alpha, b)        (assembly.py:127)
//     h_mid    = LayerNorm(residual + gamma * (h_A W_base^T + b_base + h_delta + b_delta))
// The reference materialises the gathered [B, S, k, D] rows (4.25 GiB per
// block in its 7B configuration).  Here one CTA per token streams each
// selected row once from HBM: V_j . h (r dot products) then
// alpha_j (U_j hV_j + b_j), accumulated in registers; nothing is gathered
// into memory.  On a row-sharded pool a rank sums only the rows it owns and
// the partial sums are added with one all-reduce before the LayerNorm.
//
// Pool-usage EMA: trainer.py:227-233 scatters alpha / idx.size into a
// per-row usage sum and pool.py:52-55 blends it into the EMA with beta.
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "dwa_internal.h"

namespace dwa {

namespace {

constexpr int kAsmThreads = 256;
constexpr int kAsmWarps = kAsmThreads / 32;

struct LowRankArgs {
  const void* h;
  int h_bf16;
  int64_t ldh;
  const float* alpha;
  const int32_t* gidx;
  int64_t M;
  int k;
  const __nv_bfloat16* vectors;
  int64_t row_begin, row_end, ldv;
  int d_A, d_B, r;
  float* delta;
};

__device__ __forceinline__ float bf16_lo(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float bf16_hi(uint32_t w) { return __uint_as_float(w & 0xFFFF0000u); }

// Dot of 8 bf16 (one 16-byte word) with 8 floats of shared memory.
__device__ __forceinline__ float dot8(const uint4 w, const float* hs) {
  const float4 a = *reinterpret_cast<const float4*>(hs);
  const float4 b = *reinterpret_cast<const float4*>(hs + 4);
  float s = bf16_lo(w.x) * a.x;
  s = fmaf(bf16_hi(w.x), a.y, s);
  s = fmaf(bf16_lo(w.y), a.z, s);
  s = fmaf(bf16_hi(w.y), a.w, s);
  s = fmaf(bf16_lo(w.z), b.x, s);
  s = fmaf(bf16_hi(w.z), b.y, s);
  s = fmaf(bf16_lo(w.w), b.z, s);
  s = fmaf(bf16_hi(w.w), b.w, s);
  return s;
}

// Shared memory: h (d_A floats) | alpha * hV (k * r floats) | owned alpha (k) | owned row (k).
template <bool kVecU>
__global__ void __launch_bounds__(kAsmThreads) lowrank_delta_kernel(const LowRankArgs a) {
  extern __shared__ float4 smem_f4[];
  float* h_s = reinterpret_cast<float*>(smem_f4);
  float* hv_s = h_s + a.d_A;
  float* own_a = hv_s + a.k * a.r;
  int32_t* own_j = reinterpret_cast<int32_t*>(own_a + a.k);
  __shared__ int n_own_s;

  const int64_t m = blockIdx.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // 1. compact this row's owned entries, in entry order (warp 0)
  if (warp == 0) {
    int cnt = 0;
    for (int base = 0; base < a.k; base += 32) {
      const int e = base + lane;
      int32_t g = 0;
      float al = 0.f;
      bool own = false;
      if (e < a.k) {
        g = a.gidx[m * a.k + e];
        al = a.alpha[m * a.k + e];
        own = g >= a.row_begin && g < a.row_end;
      }
      const uint32_t bal = __ballot_sync(0xffffffffu, own);
      if (own) {
        const int pos = cnt + __popc(bal & ((1u << lane) - 1u));
        own_j[pos] = static_cast<int32_t>(g - a.row_begin);
        own_a[pos] = al;
      }
      cnt += __popc(bal);
    }
    if (lane == 0) n_own_s = cnt;
  }
  // 2. this token's h as floats
  if (a.h_bf16) {
    const __nv_bfloat16* hr = static_cast<const __nv_bfloat16*>(a.h) + m * a.ldh;
    for (int d = threadIdx.x; d < a.d_A; d += kAsmThreads) h_s[d] = __bfloat162float(hr[d]);
  } else {
    const float* hr = static_cast<const float*>(a.h) + m * a.ldh;
    for (int d = threadIdx.x; d < a.d_A; d += kAsmThreads) h_s[d] = hr[d];
  }
  __syncthreads();
  const int n_own = n_own_s;
  const int r = a.r;
  // 3. alpha_j * (V_j[ri, :] . h) for every owned j and rank row ri: one warp per
  //    row, two rows per pass so that twice the loads are in flight
  const int n_rows = n_own * r;
  const int chunks = a.d_A >> 3;  // 16-byte words per V row
  auto vrow_of = [&](int q) {
    const int jj = q / r, ri = q - jj * r;
    return reinterpret_cast<const uint4*>(a.vectors + static_cast<int64_t>(own_j[jj]) * a.ldv +
                                          static_cast<int64_t>(a.d_B) * r +
                                          static_cast<int64_t>(ri) * a.d_A);
  };
  for (int q0 = warp; q0 < n_rows; q0 += 2 * kAsmWarps) {
    const int q1 = q0 + kAsmWarps;
    const bool two = q1 < n_rows;  // warp-uniform
    const uint4* v0 = vrow_of(q0);
    const uint4* v1 = two ? vrow_of(q1) : v0;
    float s0 = 0.f, s1 = 0.f;
#pragma unroll 4
    for (int c = lane; c < chunks; c += 32) {
      const uint4 w0 = __ldg(v0 + c);
      const uint4 w1 = __ldg(v1 + c);
      s0 += dot8(w0, h_s + 8 * c);
      s1 += dot8(w1, h_s + 8 * c);
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) {
      s0 += __shfl_xor_sync(0xffffffffu, s0, o);
      s1 += __shfl_xor_sync(0xffffffffu, s1, o);
    }
    if (lane == 0) {
      hv_s[q0] = own_a[q0 / r] * s0;
      if (two) hv_s[q1] = own_a[q1 / r] * s1;
    }
  }
  __syncthreads();
  // 4. delta[i] = sum_j (sum_ri alpha_j hV_j[ri] U_j[i, ri] + alpha_j b_j[i])
  const int64_t off_b = static_cast<int64_t>(a.d_B) * r + static_cast<int64_t>(r) * a.d_A;
  for (int i = threadIdx.x; i < a.d_B; i += kAsmThreads) {
    float acc = 0.f;
#pragma unroll 2
    for (int jj = 0; jj < n_own; ++jj) {
      const __nv_bfloat16* row = a.vectors + static_cast<int64_t>(own_j[jj]) * a.ldv;
      const float* hv = hv_s + jj * r;
      float u = 0.f;
      if constexpr (kVecU) {
        const uint4* urow = reinterpret_cast<const uint4*>(row + static_cast<int64_t>(i) * r);
        for (int c = 0; c < (r >> 3); ++c) u += dot8(__ldg(urow + c), hv + 8 * c);
      } else {
        const __nv_bfloat16* urow = row + static_cast<int64_t>(i) * r;
        for (int ri = 0; ri < r; ++ri) u = fmaf(__bfloat162float(urow[ri]), hv[ri], u);
      }
      acc += u + own_a[jj] * __bfloat162float(row[off_b + i]);
    }
    a.delta[m * a.d_B + i] = acc;
  }
}

struct FinishArgs {
  const void* residual;
  int res_bf16;
  int64_t ldr;
  const float* base;
  const float* delta;
  int64_t M;
  int d_B;
  float gamma;
  const float* ln_scale;
  const float* ln_bias;
  float eps;
  float* out;
};

__device__ __forceinline__ float finish_x(const FinishArgs& a, int64_t m, int i) {
  float x = a.delta[m * a.d_B + i];
  if (a.base) x += a.base[m * a.d_B + i];
  x *= a.gamma;
  if (a.residual) {
    x += a.res_bf16 ? __bfloat162float(static_cast<const __nv_bfloat16*>(a.residual)[m * a.ldr + i])
                    : static_cast<const float*>(a.residual)[m * a.ldr + i];
  }
  return x;
}

// One warp per row: x = residual + gamma * (base + delta); two-pass mean and
// variance; out = (x - mean) / sqrt(var + eps) * scale + bias.
__global__ void __launch_bounds__(256) assemble_finish_kernel(const FinishArgs a) {
  const int64_t m = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (m >= a.M) return;
  float s = 0.f;
  for (int i = lane; i < a.d_B; i += 32) s += finish_x(a, m, i);
#pragma unroll
  for (int o = 16; o; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  const float mean = s / static_cast<float>(a.d_B);
  float v = 0.f;
  for (int i = lane; i < a.d_B; i += 32) {
    const float t = finish_x(a, m, i) - mean;
    v = fmaf(t, t, v);
  }
#pragma unroll
  for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const float inv = rsqrtf(v / static_cast<float>(a.d_B) + a.eps);
  for (int i = lane; i < a.d_B; i += 32) {
    float y = (finish_x(a, m, i) - mean) * inv;
    if (a.ln_scale) y *= a.ln_scale[i];
    if (a.ln_bias) y += a.ln_bias[i];
    a.out[m * a.d_B + i] = y;
  }
}

__global__ void scale_f32_kernel(float* p, int64_t n, float s) {
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i < n) p[i] *= s;
}

__global__ void usage_scatter_kernel(const float* alpha, const int32_t* gidx, int64_t n,
                                     int64_t row_begin, int64_t row_end, float weight, float* ema) {
  const int64_t e = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (e >= n) return;
  const int64_t g = gidx[e];
  if (g >= row_begin && g < row_end) atomicAdd(ema + (g - row_begin), weight * alpha[e]);
}

}  // namespace

size_t lowrank_delta_smem_bytes(int d_A, int k, int r) {
  return (static_cast<size_t>(d_A) + static_cast<size_t>(k) * r + 2u * k) * 4u;
}

cudaError_t launch_lowrank_delta(const void* h, int h_bf16, int64_t ldh, const float* alpha,
                                 const int32_t* gidx, int64_t M, int k, const void* vectors,
                                 int64_t row_begin, int64_t row_end, int64_t ldv, int d_A, int d_B,
                                 int r, float* delta, cudaStream_t stream) {
  LowRankArgs a{h, h_bf16, ldh, alpha, gidx, M, k, static_cast<const __nv_bfloat16*>(vectors),
                row_begin, row_end, ldv, d_A, d_B, r, delta};
  const size_t smem = lowrank_delta_smem_bytes(d_A, k, r);
  const bool vec_u = (r % 8) == 0;
  cudaError_t e;
  if (vec_u) {
    e = cudaFuncSetAttribute(lowrank_delta_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(smem));
    if (e != cudaSuccess) return e;
    lowrank_delta_kernel<true><<<static_cast<unsigned>(M), kAsmThreads, smem, stream>>>(a);
  } else {
    e = cudaFuncSetAttribute(lowrank_delta_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(smem));
    if (e != cudaSuccess) return e;
    lowrank_delta_kernel<false><<<static_cast<unsigned>(M), kAsmThreads, smem, stream>>>(a);
  }
  return cudaGetLastError();
}

cudaError_t launch_assemble_finish(const void* residual, int res_bf16, int64_t ldr,
                                   const float* base, const float* delta, int64_t M, int d_B,
                                   float gamma, const float* ln_scale, const float* ln_bias,
                                   float eps, float* out, cudaStream_t stream) {
  FinishArgs a{residual, res_bf16, ldr, base, delta, M, d_B, gamma, ln_scale, ln_bias, eps, out};
  const int64_t blocks = (M * 32 + 255) / 256;
  assemble_finish_kernel<<<static_cast<unsigned>(blocks), 256, 0, stream>>>(a);
  return cudaGetLastError();
}

cudaError_t launch_usage_ema(const float* alpha, const int32_t* gidx, int64_t n, int64_t row_begin,
                             int64_t row_end, float weight, float beta, float* ema,
                             cudaStream_t stream) {
  const int64_t n_rows = row_end - row_begin;
  if (beta != 1.0f && n_rows > 0) {
    scale_f32_kernel<<<static_cast<unsigned>((n_rows + 255) / 256), 256, 0, stream>>>(ema, n_rows, beta);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
  }
  if (n > 0) {
    usage_scatter_kernel<<<static_cast<unsigned>((n + 255) / 256), 256, 0, stream>>>(
        alpha, gidx, n, row_begin, row_end, weight, ema);
  }
  return cudaGetLastError();
}

}  // namespace dwa
