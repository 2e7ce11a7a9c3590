// backward.cu — gradients of the retrieval path (selected indices fixed).
//
// The reference trains through the plain-jnp path because its Pallas kernel
// has no VJP (src/model/retrieval.py:268-271).  With the top-k indices held
// fixed, the path  out = sum_j alpha_j V[idx_j],  alpha = v / (sum v + 1e-8),
// v = gate(s) * exp(s / T),  s_j = <q, K[idx_j]>  differentiates into:
//
//   dalpha_j = <dout, V[idx_j]>                               gather_dot
//   dv_j     = dalpha_j / (S + e) - (sum_i dalpha_i v_i) / (S + e)^2
//   ds_j     = dv_j * v_j * (lambda (1 - g_j) + 1 / T)  (gate)  or  dv_j * v_j / T
//   dq       = sum_j ds_j K[idx_j]                            gather_rows (raw weights)
//   dV[idx_j] += alpha_j dout,  dK[idx_j] += ds_j q           scatter_add_rows
//   dlambda, dtau, dT: sums over (m, j)                       score_backward
//
// On one GPU the queries side (s, dalpha, ds, dq) runs as one launch,
// retrieval_backward_kernel, reading each selected row once.
//
// Every kernel works on an owned row range [row_begin, row_end) of the pool
// (owner-computes): on a sharded pool each rank's partial dalpha / s / dq are
// summed with one all-reduce, and each rank updates only its own rows.
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "dwa_internal.h"
#include "score_params.cuh"
#include "sm100_ptx.cuh"

namespace dwa {

namespace {

constexpr int kWarps = 8;

__device__ __forceinline__ void bf16x8(const uint4 x, float (&f)[8]) {
  f[0] = __uint_as_float(x.x << 16);
  f[1] = __uint_as_float(x.x & 0xFFFF0000u);
  f[2] = __uint_as_float(x.y << 16);
  f[3] = __uint_as_float(x.y & 0xFFFF0000u);
  f[4] = __uint_as_float(x.z << 16);
  f[5] = __uint_as_float(x.z & 0xFFFF0000u);
  f[6] = __uint_as_float(x.w << 16);
  f[7] = __uint_as_float(x.w & 0xFFFF0000u);
}

// 8 consecutive elements of row vector `a` (f32 or bf16) starting at col.
__device__ __forceinline__ void load_a8(const void* a, int a_bf16, int64_t off, float (&f)[8]) {
  if (a_bf16) {
    bf16x8(__ldg(reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(a) + off)), f);
  } else {
    const float4* p = reinterpret_cast<const float4*>(static_cast<const float*>(a) + off);
    const float4 x = __ldg(p), y = __ldg(p + 1);
    f[0] = x.x; f[1] = x.y; f[2] = x.z; f[3] = x.w;
    f[4] = y.x; f[5] = y.y; f[6] = y.z; f[7] = y.w;
  }
}

// out[m, j] = <a[m, :], rows[idx[m, j] - row_begin, :]> for owned rows, else 0.
// One warp per (m): lanes cover d in 8-wide slices; k dot products per row.
__global__ void __launch_bounds__(kWarps * 32)
    gather_dot_kernel(const void* a, int a_bf16, int64_t lda, const int32_t* idx, int64_t M, int k,
                      const uint16_t* rows, int64_t row_begin, int64_t row_end, int64_t ldr, int d,
                      float* out) {
  const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t m = static_cast<int64_t>(blockIdx.x) * kWarps + w;
  if (m >= M) return;
  for (int j = 0; j < k; ++j) {
    const int32_t g = idx[m * k + j];
    const bool own = g >= row_begin && g < row_end;  // warp-uniform
    float acc = 0.f;
    if (own) {
      const uint16_t* r = rows + static_cast<int64_t>(g - row_begin) * ldr;
      for (int c = lane * 8; c < d; c += 256) {
        float fa[8], fr[8];
        load_a8(a, a_bf16, m * lda + c, fa);
        bf16x8(__ldg(reinterpret_cast<const uint4*>(r + c)), fr);
#pragma unroll
        for (int e = 0; e < 8; ++e) acc = fmaf(fa[e], fr[e], acc);
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
    }
    if (lane == 0) out[m * k + j] = acc;
  }
}

// Per row m (one warp): ds[m, j] from v, s, dalpha; scalar parameter grads
// accumulated into dparams[0..2] = (dlambda, dtau, dT).
__global__ void __launch_bounds__(kWarps * 32)
    score_backward_kernel(const float* v, const float* s, const float* dalpha, int64_t M, int k,
                          float lambda_sharp, float tau, float T, int use_sigmoid, float* ds,
                          float* dparams, const float* params, int* status) {
  const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t m = static_cast<int64_t>(blockIdx.x) * kWarps + w;
  if (m >= M) return;
  if (params != nullptr) {
    // device-held {lambda_sharp, tau, T}: read here, checked here
    const ScoreParams p = load_score_params(params, lambda_sharp, tau, T);
    lambda_sharp = p.lambda_sharp;
    tau = p.tau;
    T = p.T;
    const bool ok = T > 0.0f && isfinite(T) &&
                    (!use_sigmoid || (isfinite(lambda_sharp) && isfinite(tau)));
    if (!ok) {
      if (lane == 0) record_status(status, kStatusDeviceCheck);
      for (int j = lane; j < k; j += 32) ds[m * k + j] = NAN;
      return;
    }
  }
  float sv = 0.f, sdv = 0.f;
  for (int j = lane; j < k; j += 32) {
    const float vj = v[m * k + j];
    sv += vj;
    sdv += dalpha[m * k + j] * vj;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    sv += __shfl_xor_sync(0xffffffffu, sv, o);
    sdv += __shfl_xor_sync(0xffffffffu, sdv, o);
  }
  const float den = sv + 1e-8f;
  float g_lam = 0.f, g_tau = 0.f, g_T = 0.f;
  for (int j = lane; j < k; j += 32) {
    const float vj = v[m * k + j];
    const float sj = s[m * k + j];
    const float dv = dalpha[m * k + j] / den - sdv / (den * den);
    float dvds;
    if (use_sigmoid) {
      const float gj = 1.0f / (1.0f + expf(-(lambda_sharp * (sj - tau))));
      dvds = vj * (lambda_sharp * (1.0f - gj) + 1.0f / T);
      g_lam += dv * vj * (1.0f - gj) * (sj - tau);
      g_tau += -dv * vj * lambda_sharp * (1.0f - gj);
    } else {
      dvds = vj / T;
    }
    g_T += -dv * vj * sj / (T * T);
    ds[m * k + j] = dv * dvds;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    g_lam += __shfl_xor_sync(0xffffffffu, g_lam, o);
    g_tau += __shfl_xor_sync(0xffffffffu, g_tau, o);
    g_T += __shfl_xor_sync(0xffffffffu, g_T, o);
  }
  if (lane == 0 && dparams) {
    atomicAdd(dparams + 0, g_lam);
    atomicAdd(dparams + 1, g_tau);
    atomicAdd(dparams + 2, g_T);
  }
}

// out[m, :] (=|+=) sum_j w[m, j] rows[idx[m, j] - row_begin, :] over owned rows.
__global__ void __launch_bounds__(kWarps * 32)
    gather_rows_kernel(const float* wts, const int32_t* idx, int64_t M, int k,
                       const uint16_t* rows, int64_t row_begin, int64_t row_end, int64_t ldr, int d,
                       float* out, int accumulate) {
  const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t m = static_cast<int64_t>(blockIdx.x) * kWarps + w;
  if (m >= M) return;
  for (int c0 = 0; c0 < d; c0 += 256) {
    const int col = c0 + lane * 8;
    if (col >= d) continue;
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    for (int j = 0; j < k; ++j) {
      const int32_t g = idx[m * k + j];
      if (g < row_begin || g >= row_end) continue;  // warp-uniform
      const float wj = wts[m * k + j];
      float f[8];
      bf16x8(__ldg(reinterpret_cast<const uint4*>(rows + static_cast<int64_t>(g - row_begin) * ldr +
                                                  col)),
             f);
#pragma unroll
      for (int e = 0; e < 8; ++e) acc[e] = fmaf(wj, f[e], acc[e]);
    }
    float4* dst = reinterpret_cast<float4*>(out + m * d + col);
    if (accumulate) {
      const float4 p = dst[0], q = dst[1];
      acc[0] += p.x; acc[1] += p.y; acc[2] += p.z; acc[3] += p.w;
      acc[4] += q.x; acc[5] += q.y; acc[6] += q.z; acc[7] += q.w;
    }
    dst[0] = make_float4(acc[0], acc[1], acc[2], acc[3]);
    dst[1] = make_float4(acc[4], acc[5], acc[6], acc[7]);
  }
}

// grad[idx[m, j] - row_begin, :] += w[m, j] * a[m, :] for owned rows (f32 atomics).
__global__ void __launch_bounds__(kWarps * 32)
    scatter_add_rows_kernel(const float* wts, const int32_t* idx, int64_t M, int k, const void* a,
                            int a_bf16, int64_t lda, int64_t row_begin, int64_t row_end,
                            float* grad, int64_t ldg, int d) {
  const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t m = static_cast<int64_t>(blockIdx.x) * kWarps + w;
  if (m >= M) return;
  for (int j = 0; j < k; ++j) {
    const int32_t g = idx[m * k + j];
    if (g < row_begin || g >= row_end) continue;  // warp-uniform
    const float wj = wts[m * k + j];
    float* gr = grad + static_cast<int64_t>(g - row_begin) * ldg;
    for (int c = lane * 8; c < d; c += 256) {
      float fa[8];
      load_a8(a, a_bf16, m * lda + c, fa);
#pragma unroll
      for (int e = 0; e < 8; e += 4) {
        asm volatile("red.global.add.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(gr + c + e),
                     "f"(wj * fa[e]), "f"(wj * fa[e + 1]), "f"(wj * fa[e + 2]), "f"(wj * fa[e + 3])
                     : "memory");
      }
    }
  }
}

// ---------------------------------------------------------------- fused (one GPU)
// The queries-side backward in one launch when the whole pool is on this GPU
// (no all-reduce between the dot products and the score derivative): CTA = one
// query m.  (1) warps split the k entries: s_j = <q, K_j>, dalpha_j =
// <dout, V_j>, each selected K and V row read once; (2) warp 0: ds_j and the
// lambda / tau / T terms exactly as score_backward_kernel; (3) all threads:
// dq = sum_j ds_j K_j over column slices, re-reading the K rows this CTA just
// read (from L2).  Replaces gather_dot x 2 + score_backward + gather_rows.
// The kernel is bound by how many row bytes are in flight: four CTAs per SM
// (64 registers a thread) with eight 16-byte loads per lane keep ~128 KB per
// SM outstanding.
constexpr int kBwdMaxK = 128;

struct FusedBwdArgs {
  const void* q;
  int q_bf16;
  int64_t ldq;
  const float* dout;
  int64_t ld_dout;
  const uint16_t* keys;
  int64_t ldk;
  int d_k;
  const uint16_t* values;
  int64_t ldv;
  int d_v;
  const float* v;
  const int32_t* idx;
  int64_t M;
  int k;
  int64_t row_begin, row_end;
  float lambda_sharp, tau, T;
  const float* params;
  int use_sigmoid;
  float* ds;
  float* dq;
  float* dparams;
  int* status;
};

__global__ void __launch_bounds__(kWarps * 32, 4) retrieval_backward_kernel(const FusedBwdArgs a) {
  __shared__ int32_t g_s[kBwdMaxK];
  __shared__ float s_s[kBwdMaxK], da_s[kBwdMaxK], ds_s[kBwdMaxK];
  __shared__ int ok_s;
  const int64_t m = blockIdx.x;
  const int tid = threadIdx.x, w = tid >> 5, lane = tid & 31;
  const int k = a.k;
  for (int j = tid; j < k; j += kWarps * 32) g_s[j] = a.idx[m * k + j];
  __syncthreads();
  // (1) s_j and dalpha_j, entries j = w, w + 8, ...  The K rows are read
  // again by (3), so they are loaded with the L2 evict-last policy; the V rows
  // are read once (evict-first).  Each pass of the column loop puts a row's
  // next 1024 columns of K and of V in flight together (8 loads per lane).
  const uint64_t pol_keep = l2_policy_evict_last();
  const uint64_t pol_once = l2_policy_evict_first();
  const int d_max = a.d_k > a.d_v ? a.d_k : a.d_v;
  for (int j = w; j < k; j += kWarps) {
    const int32_t g = g_s[j];
    float sj = 0.f, dj = 0.f;
    if (g >= a.row_begin && g < a.row_end) {  // warp-uniform
      const uint16_t* kr = a.keys + static_cast<int64_t>(g - a.row_begin) * a.ldk;
      const uint16_t* vr = a.values + static_cast<int64_t>(g - a.row_begin) * a.ldv;
      for (int c0 = lane * 8; c0 < d_max; c0 += 1024) {
        uint4 kx[4], vx[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const int c = c0 + 256 * u;
          kx[u] = c < a.d_k ? ld_nc_l2hint_v4(kr + c, pol_keep) : make_uint4(0u, 0u, 0u, 0u);
          vx[u] = c < a.d_v ? ld_nc_l2hint_v4(vr + c, pol_once) : make_uint4(0u, 0u, 0u, 0u);
        }
        // per lane, columns in increasing order (the order of gather_dot_kernel)
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const int c = c0 + 256 * u;
          if (c < a.d_k) {
            float fa[8], fr[8];
            load_a8(a.q, a.q_bf16, m * a.ldq + c, fa);
            bf16x8(kx[u], fr);
#pragma unroll
            for (int e = 0; e < 8; ++e) sj = fmaf(fa[e], fr[e], sj);
          }
          if (c < a.d_v) {
            float fa[8], fr[8];
            load_a8(a.dout, 0, m * a.ld_dout + c, fa);
            bf16x8(vx[u], fr);
#pragma unroll
            for (int e = 0; e < 8; ++e) dj = fmaf(fa[e], fr[e], dj);
          }
        }
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        sj += __shfl_xor_sync(0xffffffffu, sj, o);
        dj += __shfl_xor_sync(0xffffffffu, dj, o);
      }
    }
    if (lane == 0) {
      s_s[j] = sj;
      da_s[j] = dj;
    }
  }
  __syncthreads();
  // (2) ds_j and the scalar-parameter terms (score_backward_kernel's formulas)
  if (w == 0) {
    float lambda_sharp = a.lambda_sharp, tau = a.tau, T = a.T;
    bool ok = true;
    if (a.params != nullptr) {
      const ScoreParams p = load_score_params(a.params, lambda_sharp, tau, T);
      lambda_sharp = p.lambda_sharp;
      tau = p.tau;
      T = p.T;
      ok = T > 0.0f && isfinite(T) && (!a.use_sigmoid || (isfinite(lambda_sharp) && isfinite(tau)));
      if (!ok && lane == 0) record_status(a.status, kStatusDeviceCheck);
    }
    float sv = 0.f, sdv = 0.f;
    for (int j = lane; j < k; j += 32) {
      const float vj = a.v[m * k + j];
      sv += vj;
      sdv += da_s[j] * vj;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      sv += __shfl_xor_sync(0xffffffffu, sv, o);
      sdv += __shfl_xor_sync(0xffffffffu, sdv, o);
    }
    const float den = sv + 1e-8f;
    float g_lam = 0.f, g_tau = 0.f, g_T = 0.f;
    for (int j = lane; j < k; j += 32) {
      const float vj = a.v[m * k + j];
      const float sj = s_s[j];
      const float dv = da_s[j] / den - sdv / (den * den);
      float dvds;
      if (a.use_sigmoid) {
        const float gj = 1.0f / (1.0f + expf(-(lambda_sharp * (sj - tau))));
        dvds = vj * (lambda_sharp * (1.0f - gj) + 1.0f / T);
        g_lam += dv * vj * (1.0f - gj) * (sj - tau);
        g_tau += -dv * vj * lambda_sharp * (1.0f - gj);
      } else {
        dvds = vj / T;
      }
      g_T += -dv * vj * sj / (T * T);
      const float dsj = ok ? dv * dvds : NAN;
      ds_s[j] = dsj;
      a.ds[m * k + j] = dsj;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      g_lam += __shfl_xor_sync(0xffffffffu, g_lam, o);
      g_tau += __shfl_xor_sync(0xffffffffu, g_tau, o);
      g_T += __shfl_xor_sync(0xffffffffu, g_T, o);
    }
    if (lane == 0) {
      ok_s = ok ? 1 : 0;
      if (ok && a.dparams) {
        atomicAdd(a.dparams + 0, g_lam);
        atomicAdd(a.dparams + 1, g_tau);
        atomicAdd(a.dparams + 2, g_T);
      }
    }
  }
  __syncthreads();
  // (3) dq[m, c..c+3] = sum_j ds_j K_j[c..c+3]: 4 columns per thread per step,
  // the k rows in blocks of 8 so eight loads are in flight; the K rows' last
  // read (evict-first)
  const bool ok = ok_s != 0;
  for (int c = tid * 4; c < a.d_k; c += kWarps * 32 * 4) {
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
    for (int j0 = 0; j0 < k; j0 += 8) {
      uint2 raw[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const int j = j0 + u;
        const int32_t g = j < k ? g_s[j] : -1;
        raw[u] = (g >= a.row_begin && g < a.row_end)
                     ? ld_nc_l2hint_v2(a.keys + static_cast<int64_t>(g - a.row_begin) * a.ldk + c,
                                       pol_once)
                     : make_uint2(0u, 0u);
      }
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const int j = j0 + u;
        const float wj = j < k ? ds_s[j] : 0.f;
        acc[0] = fmaf(wj, __uint_as_float(raw[u].x << 16), acc[0]);
        acc[1] = fmaf(wj, __uint_as_float(raw[u].x & 0xFFFF0000u), acc[1]);
        acc[2] = fmaf(wj, __uint_as_float(raw[u].y << 16), acc[2]);
        acc[3] = fmaf(wj, __uint_as_float(raw[u].y & 0xFFFF0000u), acc[3]);
      }
    }
    float4 r = make_float4(acc[0], acc[1], acc[2], acc[3]);
    if (!ok) r = make_float4(NAN, NAN, NAN, NAN);
    *reinterpret_cast<float4*>(a.dq + m * a.d_k + c) = r;
  }
}

// ---------------------------------------------------------------- dense row gradients
// grad[r, :] = sum over the pairs (m, j) that selected owned row r of
// w[m, j] a[m, :] (fp32 sums), written for every owned row (zero where no
// pair selected it) in bf16 or f32: the whole dense gradient in one write,
// from the row-sorted pair list (pair_sort.cu), with no float atomics and no
// separate zero fill or dtype conversion.  One warp per row, 8 columns per lane.
struct RowGradArgs {
  const float* w;
  const int32_t* offsets;
  const int32_t* pairs;
  int k;
  const void* a;
  int a_bf16;
  int64_t lda;
  int64_t n_rows;
  void* grad;
  int64_t ldg;
  int d;
};

template <bool OUT_BF16>
// Six blocks per SM (40 registers, no spills): most rows have no or one entry,
// so a row is a short chain of dependent loads and more rows in flight pay.
__global__ void __launch_bounds__(kWarps * 32, 6) row_gradient_kernel(const RowGradArgs g) {
  const int w = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t r = static_cast<int64_t>(blockIdx.x) * kWarps + w;
  if (r >= g.n_rows) return;
  const int32_t p0 = g.offsets[r], p1 = g.offsets[r + 1];
  for (int c = lane * 8; c < g.d; c += 256) {
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    for (int32_t p = p0; p < p1; ++p) {
      const int32_t pid = g.pairs[p];
      const float wt = g.w[pid];
      float x[8];
      load_a8(g.a, g.a_bf16, static_cast<int64_t>(pid / g.k) * g.lda + c, x);
#pragma unroll
      for (int e = 0; e < 8; ++e) acc[e] = fmaf(wt, x[e], acc[e]);
    }
    if constexpr (OUT_BF16) {
      uint32_t packed[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const uint32_t lo = __bfloat16_as_ushort(__float2bfloat16_rn(acc[2 * e]));
        const uint32_t hi = __bfloat16_as_ushort(__float2bfloat16_rn(acc[2 * e + 1]));
        packed[e] = lo | (hi << 16);
      }
      *reinterpret_cast<uint4*>(static_cast<uint16_t*>(g.grad) + r * g.ldg + c) =
          make_uint4(packed[0], packed[1], packed[2], packed[3]);
    } else {
      float4* dst = reinterpret_cast<float4*>(static_cast<float*>(g.grad) + r * g.ldg + c);
      dst[0] = make_float4(acc[0], acc[1], acc[2], acc[3]);
      dst[1] = make_float4(acc[4], acc[5], acc[6], acc[7]);
    }
  }
}

inline unsigned blocks_for(int64_t M) { return static_cast<unsigned>((M + kWarps - 1) / kWarps); }

}  // namespace

cudaError_t launch_gather_dot(const void* a, int a_bf16, int64_t lda, const int32_t* idx, int64_t M,
                              int k, const void* rows, int64_t row_begin, int64_t row_end,
                              int64_t ldr, int d, float* out, cudaStream_t stream) {
  if (M <= 0) return cudaSuccess;
  gather_dot_kernel<<<blocks_for(M), kWarps * 32, 0, stream>>>(
      a, a_bf16, lda, idx, M, k, static_cast<const uint16_t*>(rows), row_begin, row_end, ldr, d,
      out);
  return cudaGetLastError();
}

cudaError_t launch_score_backward(const float* v, const float* s, const float* dalpha, int64_t M,
                                  int k, float lambda_sharp, float tau, float T, int use_sigmoid,
                                  float* ds, float* dparams, cudaStream_t stream,
                                  const float* params, int* status) {
  if (M <= 0) return cudaSuccess;
  score_backward_kernel<<<blocks_for(M), kWarps * 32, 0, stream>>>(
      v, s, dalpha, M, k, lambda_sharp, tau, T, use_sigmoid, ds, dparams, params, status);
  return cudaGetLastError();
}

cudaError_t launch_gather_rows(const float* wts, const int32_t* idx, int64_t M, int k,
                               const void* rows, int64_t row_begin, int64_t row_end, int64_t ldr,
                               int d, float* out, int accumulate, cudaStream_t stream) {
  if (M <= 0) return cudaSuccess;
  gather_rows_kernel<<<blocks_for(M), kWarps * 32, 0, stream>>>(
      wts, idx, M, k, static_cast<const uint16_t*>(rows), row_begin, row_end, ldr, d, out,
      accumulate);
  return cudaGetLastError();
}

cudaError_t launch_retrieval_backward(const void* q, int q_bf16, int64_t ldq, const float* dout,
                                      int64_t ld_dout, const void* keys, int64_t ldk, int d_k,
                                      const void* values, int64_t ldv, int d_v, const float* v,
                                      const int32_t* idx, int64_t M, int k, int64_t row_begin,
                                      int64_t row_end, float lambda_sharp, float tau, float T,
                                      const float* params, int use_sigmoid, float* ds, float* dq,
                                      float* dparams, int* status, cudaStream_t stream) {
  if (M <= 0) return cudaSuccess;
  if (k < 1 || k > kBwdMaxK) return cudaErrorInvalidValue;
  FusedBwdArgs a{q, q_bf16, ldq, dout, ld_dout, static_cast<const uint16_t*>(keys), ldk, d_k,
                 static_cast<const uint16_t*>(values), ldv, d_v, v, idx, M, k, row_begin,
                 row_end, lambda_sharp, tau, T, params, use_sigmoid, ds, dq, dparams, status};
  retrieval_backward_kernel<<<static_cast<unsigned>(M), kWarps * 32, 0, stream>>>(a);
  return cudaGetLastError();
}

size_t row_gradient_workspace_bytes(int64_t M, int k, int64_t n_rows) {
  return pair_sort_workspace_bytes(M * k, n_rows);
}

cudaError_t launch_row_gradient(const float* w, const int32_t* idx, int64_t M, int k, const void* a,
                                int a_bf16, int64_t lda, int64_t row_begin, int64_t row_end,
                                void* grad, int grad_bf16, int64_t ldg, int d, void* ws,
                                cudaStream_t stream) {
  const int64_t n_rows = row_end - row_begin;
  if (n_rows <= 0) return cudaSuccess;
  const size_t row_bytes = static_cast<size_t>(d) * (grad_bf16 ? 2 : 4);
  if (M <= 0) {  // no pairs: the gradient is zero
    return cudaMemset2DAsync(grad, static_cast<size_t>(ldg) * (grad_bf16 ? 2 : 4), 0, row_bytes,
                             static_cast<size_t>(n_rows), stream);
  }
  PairSort sorted;
  cudaError_t e = launch_sort_pairs_by_row(idx, M * k, row_begin, row_end, ws, &sorted, stream);
  if (e != cudaSuccess) return e;
  RowGradArgs g{w, sorted.offsets, sorted.pairs, k, a, a_bf16, lda, n_rows, grad, ldg, d};
  const unsigned blocks = static_cast<unsigned>((n_rows + kWarps - 1) / kWarps);
  if (grad_bf16)
    row_gradient_kernel<true><<<blocks, kWarps * 32, 0, stream>>>(g);
  else
    row_gradient_kernel<false><<<blocks, kWarps * 32, 0, stream>>>(g);
  return cudaGetLastError();
}

cudaError_t launch_scatter_add_rows(const float* wts, const int32_t* idx, int64_t M, int k,
                                    const void* a, int a_bf16, int64_t lda, int64_t row_begin,
                                    int64_t row_end, float* grad, int64_t ldg, int d,
                                    cudaStream_t stream) {
  if (M <= 0) return cudaSuccess;
  scatter_add_rows_kernel<<<blocks_for(M), kWarps * 32, 0, stream>>>(
      wts, idx, M, k, a, a_bf16, lda, row_begin, row_end, grad, ldg, d);
  return cudaGetLastError();
}

}  // namespace dwa
