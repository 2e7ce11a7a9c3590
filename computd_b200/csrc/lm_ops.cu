// lm_ops.cu — fused elementwise steps of the DWA language model's block
// around the retrieval (the call site, src/model/dwa.py:77-130 and
// src/model/parts.py:17-83 of the reference).
//
//  * rope_qk_kernel: the rotary embedding of the attention's queries and keys
//    (parts.py:17-25: x1 = x[..., 0::2], x2 = x[..., 1::2],
//    [x1 cos - x2 sin, x1 sin + x2 cos]) read straight from the QKV
//    projection's rows and written token-major, [B, S, H, dh], the layout
//    attention reads through a (1, 2)-transposed view and writes its output
//    in, so the output projection needs no transposing copy.  Each product,
//    sum and difference is rounded to bf16 as the elementwise bf16 tensor ops
//    do, so the result is bit-identical to them; one pass instead of six
//    elementwise kernels and a concatenation per tensor.
//  * aspect_queries_kernel: the packed aspect queries of the hybrid score
//    (retrieval.py:159-168): w = softmax(aspect_logits), and per row m and
//    aspect s, q[m, s, :] sqrt(w_s) / (|q[m, s, :]| + 1e-8) in bf16; block 0
//    also writes w and the score's device scalars {lambda_sharp,
//    tau = w . tau_param (gate on) or 0, T}.  One launch instead of a float
//    copy, a norm reduction, the scale arithmetic, the bf16 cast, the softmax,
//    the dot product and the scalar fill.
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "dwa_internal.h"

namespace dwa {

namespace {

__device__ __forceinline__ float bf(uint16_t u) { return __uint_as_float(static_cast<uint32_t>(u) << 16); }
__device__ __forceinline__ uint16_t to_bf(float x) {
  return __bfloat16_as_ushort(__float2bfloat16_rn(x));
}
__device__ __forceinline__ float rbf(float x) { return bf(to_bf(x)); }  // round to bf16 and back

// One thread = 4 rotation pairs (8 input elements) of one (token, head) of q
// or of k.  half = dh / 2 (a multiple of 4).
__global__ void rope_qk_kernel(const uint16_t* __restrict__ qkv, int64_t B, int64_t S, int H,
                               int dh, int64_t ld_qkv, const uint16_t* __restrict__ cosv,
                               const uint16_t* __restrict__ sinv, int64_t ld_cs,
                               uint16_t* __restrict__ q_out, uint16_t* __restrict__ k_out) {
  const int half = dh >> 1;
  const int groups = half >> 2;  // 4-pair groups per head
  const int64_t per_tensor = B * S * H * groups;
  const int64_t t = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (t >= 2 * per_tensor) return;
  const int which = t >= per_tensor ? 1 : 0;  // 0: q, 1: k
  int64_t r = t - which * per_tensor;
  const int g = static_cast<int>(r % groups);
  r /= groups;
  const int h = static_cast<int>(r % H);
  r /= H;
  const int64_t s = r % S;
  const int64_t b = r / S;
  const int j0 = 4 * g;  // first pair
  const uint16_t* x = qkv + (b * S + s) * ld_qkv + static_cast<int64_t>(which) * H * dh +
                      static_cast<int64_t>(h) * dh + 2 * j0;
  const uint4 xv = *reinterpret_cast<const uint4*>(x);  // x[2 j0 .. 2 j0 + 7]
  const uint2 cv = *reinterpret_cast<const uint2*>(cosv + s * ld_cs + j0);
  const uint2 sv = *reinterpret_cast<const uint2*>(sinv + s * ld_cs + j0);
  const uint32_t xw[4] = {xv.x, xv.y, xv.z, xv.w};
  const uint32_t cw[2] = {cv.x, cv.y}, sw[2] = {sv.x, sv.y};
  uint16_t lo[4], hi[4];
#pragma unroll
  for (int p = 0; p < 4; ++p) {
    const float x1 = bf(static_cast<uint16_t>(xw[p] & 0xFFFFu));
    const float x2 = bf(static_cast<uint16_t>(xw[p] >> 16));
    const float c = bf(static_cast<uint16_t>((cw[p >> 1] >> (16 * (p & 1))) & 0xFFFFu));
    const float sn = bf(static_cast<uint16_t>((sw[p >> 1] >> (16 * (p & 1))) & 0xFFFFu));
    lo[p] = to_bf(rbf(x1 * c) - rbf(x2 * sn));
    hi[p] = to_bf(rbf(x1 * sn) + rbf(x2 * c));
  }
  uint16_t* o = (which ? k_out : q_out) + ((b * S + s) * H + h) * dh;
  uint2 lw, hw;
  lw.x = static_cast<uint32_t>(lo[0]) | (static_cast<uint32_t>(lo[1]) << 16);
  lw.y = static_cast<uint32_t>(lo[2]) | (static_cast<uint32_t>(lo[3]) << 16);
  hw.x = static_cast<uint32_t>(hi[0]) | (static_cast<uint32_t>(hi[1]) << 16);
  hw.y = static_cast<uint32_t>(hi[2]) | (static_cast<uint32_t>(hi[3]) << 16);
  *reinterpret_cast<uint2*>(o + j0) = lw;
  *reinterpret_cast<uint2*>(o + half + j0) = hw;
}

constexpr int kMaxAspects = 64;

// One thread = one (row m, aspect s) group of d_k elements.
__global__ void aspect_queries_kernel(const uint16_t* __restrict__ q, int64_t M, int S, int d_k,
                                      int64_t ldq, const float* __restrict__ logits,
                                      const float* __restrict__ tau_param, float lambda_sharp,
                                      float T, int use_sigmoid, uint16_t* __restrict__ out,
                                      int64_t ldo, float* w_out, float* params_out) {
  // w = softmax(logits), every thread for itself (S <= kMaxAspects values)
  float mx = -INFINITY;
  for (int i = 0; i < S; ++i) mx = fmaxf(mx, __ldg(logits + i));
  float den = 0.f;
  for (int i = 0; i < S; ++i) den += expf(__ldg(logits + i) - mx);
  const int64_t t = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (t == 0) {
    float tau = 0.f;
    for (int i = 0; i < S; ++i) {
      const float wi = expf(__ldg(logits + i) - mx) / den;
      if (w_out != nullptr) w_out[i] = wi;
      if (use_sigmoid) tau += wi * __ldg(tau_param + i);
    }
    if (params_out != nullptr) {
      params_out[0] = lambda_sharp;
      params_out[1] = tau;
      params_out[2] = T;
    }
  }
  if (t >= M * S) return;
  const int s = static_cast<int>(t % S);
  const int64_t m = t / S;
  const float ws = expf(__ldg(logits + s) - mx) / den;
  const uint16_t* src = q + m * ldq + static_cast<int64_t>(s) * d_k;
  float ss = 0.f;
  for (int c = 0; c < d_k; c += 8) {
    const uint4 v = *reinterpret_cast<const uint4*>(src + c);
    const uint32_t w4[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float a = bf(static_cast<uint16_t>(w4[e] & 0xFFFFu));
      const float b2 = bf(static_cast<uint16_t>(w4[e] >> 16));
      ss = fmaf(a, a, ss);
      ss = fmaf(b2, b2, ss);
    }
  }
  const float scale = sqrtf(ws) / (sqrtf(ss) + 1e-8f);
  uint16_t* dst = out + m * ldo + static_cast<int64_t>(s) * d_k;
  for (int c = 0; c < d_k; c += 8) {
    const uint4 v = *reinterpret_cast<const uint4*>(src + c);
    const uint32_t w4[4] = {v.x, v.y, v.z, v.w};
    uint32_t o4[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float a = bf(static_cast<uint16_t>(w4[e] & 0xFFFFu)) * scale;
      const float b2 = bf(static_cast<uint16_t>(w4[e] >> 16)) * scale;
      o4[e] = static_cast<uint32_t>(to_bf(a)) | (static_cast<uint32_t>(to_bf(b2)) << 16);
    }
    *reinterpret_cast<uint4*>(dst + c) = make_uint4(o4[0], o4[1], o4[2], o4[3]);
  }
}

}  // namespace

int lm_max_aspects() { return kMaxAspects; }

cudaError_t launch_rope_qk(const void* qkv, int64_t B, int64_t S, int H, int dh, int64_t ld_qkv,
                           const void* cosv, const void* sinv, int64_t ld_cs, void* q_out,
                           void* k_out, cudaStream_t stream) {
  const int64_t threads = 2 * B * S * H * (dh / 8);
  if (threads == 0) return cudaSuccess;
  const int block = 256;
  rope_qk_kernel<<<static_cast<unsigned>((threads + block - 1) / block), block, 0, stream>>>(
      static_cast<const uint16_t*>(qkv), B, S, H, dh, ld_qkv, static_cast<const uint16_t*>(cosv),
      static_cast<const uint16_t*>(sinv), ld_cs, static_cast<uint16_t*>(q_out),
      static_cast<uint16_t*>(k_out));
  return cudaGetLastError();
}

cudaError_t launch_aspect_queries(const void* q, int64_t M, int S, int d_k, int64_t ldq,
                                  const float* logits, const float* tau_param, float lambda_sharp,
                                  float T, int use_sigmoid, void* out, int64_t ldo, float* w_out,
                                  float* params_out, cudaStream_t stream) {
  const int64_t threads = M * S > 0 ? M * S : 1;  // block 0 still writes w and params
  const int block = 256;
  aspect_queries_kernel<<<static_cast<unsigned>((threads + block - 1) / block), block, 0,
                          stream>>>(static_cast<const uint16_t*>(q), M, S, d_k, ldq, logits,
                                    tau_param, lambda_sharp, T, use_sigmoid,
                                    static_cast<uint16_t*>(out), ldo, w_out, params_out);
  return cudaGetLastError();
}

}  // namespace dwa
