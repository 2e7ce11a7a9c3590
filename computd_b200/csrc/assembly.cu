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

#include <algorithm>
#include <cstdint>

#include "dwa_internal.h"
#include "sm100_ptx.cuh"

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

// ---------------------------------------------------------------------------
// Staged variant: two persistent CTAs per SM; a producer warp bulk-copies each
// selected row's V block, then its U and b blocks, into a ring of shared-memory
// stages with cp.async.bulk (completion counted on mbarriers), so many
// kilobytes per SM are in flight from HBM at once; eight consumer warps
// compute from shared memory.  All waits are bounded; a wait that runs out
// raises a CTA abort flag and every role leaves its loop.
constexpr int kStgConsumers = 256;
constexpr int kStgWarps = kStgConsumers / 32;
constexpr int kStgThreads = kStgConsumers + 32;
constexpr int kStgMaxOut = 16;      // outputs per consumer thread: d_B <= 4096
constexpr int kStgMaxStages = 4;
constexpr int kStgCtasPerSm = 2;  // a second CTA overlaps each CTA's per-row barrier bubbles

struct StagedArgs {
  LowRankArgs a;
  int stages;
  uint32_t stage_bytes, v_bytes, u_bytes, b_bytes, h_bytes, h_slot_bytes;
  uint32_t meta_off, bar_off;  // byte offsets in shared memory
};

template <bool kHBf16>
__global__ void __launch_bounds__(kStgThreads, kStgCtasPerSm) lowrank_delta_staged_kernel(const StagedArgs sa) {
  const LowRankArgs& a = sa.a;
  extern __shared__ __align__(128) uint8_t sm[];
  const int S = sa.stages;
  const int k = a.k, r = a.r;
  uint8_t* hslot0 = sm + static_cast<size_t>(S) * sa.stage_bytes;
  int32_t* meta_j = reinterpret_cast<int32_t*>(sm + sa.meta_off);  // [2][k]
  float* meta_a = reinterpret_cast<float*>(meta_j + 2 * k);          // [2][k]
  int* meta_n = reinterpret_cast<int*>(meta_a + 2 * k);              // [2]
  float* hv = reinterpret_cast<float*>(meta_n + 4);                  // [4][r]
  const uint32_t bar0 = smem_u32(sm + sa.bar_off);
  auto full = [&](int st) { return bar0 + 8u * st; };
  auto empty = [&](int st) { return bar0 + 8u * (S + st); };
  auto hfull = [&](int sl) { return bar0 + 8u * (2 * S + sl); };
  auto hempty = [&](int sl) { return bar0 + 8u * (2 * S + 2 + sl); };
  auto hvbar = [&](int sl) { return bar0 + 8u * (2 * S + 4 + sl); };  // 4 of them
  int* ctl = reinterpret_cast<int*>(sm + sa.bar_off + 8 * (2 * S + 8));
  volatile int* abort_flag = ctl;
  int* n_issued = ctl + 1;
  int* n_consumed = ctl + 2;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int st = 0; st < S; ++st) {
      mbar_init(full(st), 1);
      mbar_init(empty(st), kStgWarps);
    }
    for (int sl = 0; sl < 2; ++sl) {
      mbar_init(hfull(sl), 1);
      mbar_init(hempty(sl), kStgWarps);
    }
    for (int sl = 0; sl < 4; ++sl) mbar_init(hvbar(sl), kStgWarps);
    *abort_flag = 0;
    *n_issued = 0;
    *n_consumed = 0;
    fence_mbar_init();
  }
  __syncthreads();

  const int64_t off_b = static_cast<int64_t>(a.d_B) * r + static_cast<int64_t>(r) * a.d_A;
  const int h_elem = kHBf16 ? 2 : 4;
  if (warp == kStgWarps) {
    // ------------------------------------------------------------ producer
    int it = 0, tk = 0;
    bool ok = true;
    for (int64_t m = blockIdx.x; m < a.M && ok; m += gridDim.x, ++tk) {
      const int slot = tk & 1;
      const uint32_t use = static_cast<uint32_t>(tk >> 1);
      bool got = true;
      if (lane == 0) got = mbar_wait(hempty(slot), (use & 1u) ^ 1u, nullptr, abort_flag);
      if (!__shfl_sync(0xffffffffu, got, 0)) break;
      int cnt = 0;  // owned entries of token m, in entry order
      for (int base = 0; base < k; base += 32) {
        const int e = base + lane;
        int32_t g = 0;
        float al = 0.f;
        bool own = false;
        if (e < k) {
          g = a.gidx[m * k + e];
          al = a.alpha[m * k + e];
          own = g >= a.row_begin && g < a.row_end;
        }
        const uint32_t bal = __ballot_sync(0xffffffffu, own);
        if (own) {
          const int pos = cnt + __popc(bal & ((1u << lane) - 1u));
          meta_j[slot * k + pos] = static_cast<int32_t>(g - a.row_begin);
          meta_a[slot * k + pos] = al;
        }
        cnt += __popc(bal);
      }
      if (lane == 0) meta_n[slot] = cnt;
      __syncwarp();
      if (lane == 0) {
        mbar_arrive_expect_tx(hfull(slot), sa.h_bytes);
        bulk_load(smem_u32(hslot0 + slot * sa.h_slot_bytes),
                  static_cast<const uint8_t*>(a.h) + m * a.ldh * h_elem, sa.h_bytes, hfull(slot));
        for (int jj = 0; jj < cnt && ok; ++jj) {
          const __nv_bfloat16* row = a.vectors + static_cast<int64_t>(meta_j[slot * k + jj]) * a.ldv;
          for (int piece = 0; piece < 2; ++piece, ++it) {
            const int st = it % S;
            const uint32_t rr = static_cast<uint32_t>(it / S);
            if (!mbar_wait(empty(st), (rr & 1u) ^ 1u, nullptr, abort_flag)) {
              ok = false;
              break;
            }
            const uint32_t dst = smem_u32(sm + static_cast<size_t>(st) * sa.stage_bytes);
            if (piece == 0) {
              mbar_arrive_expect_tx(full(st), sa.v_bytes);
              bulk_load(dst, row + static_cast<int64_t>(a.d_B) * r, sa.v_bytes, full(st));
            } else {
              mbar_arrive_expect_tx(full(st), sa.u_bytes + sa.b_bytes);
              bulk_load(dst, row, sa.u_bytes, full(st));
              bulk_load(dst + sa.u_bytes, row + off_b, sa.b_bytes, full(st));
            }
          }
        }
      }
      ok = __shfl_sync(0xffffffffu, ok, 0);
    }
    if (lane == 0) *n_issued = it;
  } else {
    // ------------------------------------------------------------ consumers
    // Per token: pieces it0 + 2j (V_j) and it0 + 2j + 1 (U_j | b_j).  A warp
    // computes its rows of alpha_j V_j h for row j + 1 before it waits for the
    // other warps' rows of row j and accumulates row j, so no warp idles at
    // the per-row barrier.  alpha_j hV_j lives in buffer g % 4 (g counts rows
    // over all tokens): a warp writing buffer g + 2 has passed barrier g,
    // which every warp reached only after finishing row g - 2.
    const int tid = threadIdx.x;
    const int words = a.d_A >> 3;
    const int uw = r >> 3;  // 16-byte words per U row
    int it0 = 0, tk = 0, g0 = 0;
    bool ok = true;
    auto v_phase = [&](int j, int g, const float* oa, const uint8_t* hs) -> bool {
      const int piece = it0 + 2 * j;
      const int st = piece % S;
      bool got = mbar_wait(full(st), static_cast<uint32_t>(piece / S) & 1u, nullptr, abort_flag);
      if (!__all_sync(0xffffffffu, got)) return false;
      const uint4* V = reinterpret_cast<const uint4*>(sm + static_cast<size_t>(st) * sa.stage_bytes);
      float* hvj = hv + (g & 3) * r;
      for (int ri = warp; ri < r; ri += kStgWarps) {
        float sacc = 0.f;
        for (int c = lane; c < words; c += 32) {
          const uint4 w = V[ri * words + c];
          if constexpr (kHBf16) {
            const uint4 hw = reinterpret_cast<const uint4*>(hs)[c];
            sacc = fmaf(bf16_lo(w.x), bf16_lo(hw.x), sacc);
            sacc = fmaf(bf16_hi(w.x), bf16_hi(hw.x), sacc);
            sacc = fmaf(bf16_lo(w.y), bf16_lo(hw.y), sacc);
            sacc = fmaf(bf16_hi(w.y), bf16_hi(hw.y), sacc);
            sacc = fmaf(bf16_lo(w.z), bf16_lo(hw.z), sacc);
            sacc = fmaf(bf16_hi(w.z), bf16_hi(hw.z), sacc);
            sacc = fmaf(bf16_lo(w.w), bf16_lo(hw.w), sacc);
            sacc = fmaf(bf16_hi(w.w), bf16_hi(hw.w), sacc);
          } else {
            sacc += dot8(w, reinterpret_cast<const float*>(hs) + 8 * c);
          }
        }
#pragma unroll
        for (int o = 16; o; o >>= 1) sacc += __shfl_xor_sync(0xffffffffu, sacc, o);
        if (lane == 0) hvj[ri] = oa[j] * sacc;
      }
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(empty(st));
        mbar_arrive(hvbar(g & 3));  // this warp's rows of alpha_j hV_j are written
      }
      return true;
    };
    for (int64_t m = blockIdx.x; m < a.M; m += gridDim.x, ++tk) {
      const int slot = tk & 1;
      const uint32_t use = static_cast<uint32_t>(tk >> 1);
      ok = mbar_wait(hfull(slot), use & 1u, nullptr, abort_flag);
      if (!__all_sync(0xffffffffu, ok)) {
        ok = false;
        break;
      }
      const int n = meta_n[slot];
      const float* oa = meta_a + slot * k;
      const uint8_t* hs = hslot0 + slot * sa.h_slot_bytes;
      float acc[kStgMaxOut];
#pragma unroll
      for (int u = 0; u < kStgMaxOut; ++u) acc[u] = 0.f;
      if (n > 0) ok = v_phase(0, g0, oa, hs);
      for (int jj = 0; jj < n && ok; ++jj) {
        const int g = g0 + jj;
        if (jj + 1 < n) ok = v_phase(jj + 1, g + 1, oa, hs);
        if (!ok) break;
        bool got = mbar_wait(hvbar(g & 3), static_cast<uint32_t>(g >> 2) & 1u, nullptr, abort_flag);
        const int piece = it0 + 2 * jj + 1;
        const int st = piece % S;
        got = got && mbar_wait(full(st), static_cast<uint32_t>(piece / S) & 1u, nullptr, abort_flag);
        if (!__all_sync(0xffffffffu, got)) {
          ok = false;
          break;
        }
        const uint8_t* ub = sm + static_cast<size_t>(st) * sa.stage_bytes;
        const uint4* U = reinterpret_cast<const uint4*>(ub);
        const __nv_bfloat16* bv = reinterpret_cast<const __nv_bfloat16*>(ub + sa.u_bytes);
        const float* hvj = hv + (g & 3) * r;
        const float aj = oa[jj];
#pragma unroll
        for (int u = 0; u < kStgMaxOut; ++u) {
          const int i = tid + u * kStgConsumers;
          if (i < a.d_B) {
            float t = aj * __bfloat162float(bv[i]);
            for (int c = 0; c < uw; ++c) t += dot8(U[i * uw + c], hvj + 8 * c);
            acc[u] += t;
          }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(empty(st));
      }
      if (!ok) break;
      it0 += 2 * n;
      g0 += n;
#pragma unroll
      for (int u = 0; u < kStgMaxOut; ++u) {
        const int i = tid + u * kStgConsumers;
        if (i < a.d_B) a.delta[m * a.d_B + i] = acc[u];
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(hempty(slot));
    }
    if (!ok) *abort_flag = 1;
    if (tid == 0) *n_consumed = it0;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    // copies issued but never consumed (only after an abort) must land before exit
    for (int i = *n_consumed; i < *n_issued; ++i)
      mbar_wait(full(i % S), static_cast<uint32_t>(i / S) & 1u, nullptr, nullptr);
  }
  __syncthreads();
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
// Rows of NV x 128 elements (d_B = 128 NV, 16-byte aligned rows): lane l holds
// elements 128 j + 4 l .. + 3 in registers, read once with 16-byte loads.
template <int NV>
__global__ void __launch_bounds__(256) assemble_finish_reg_kernel(const FinishArgs a) {
  const int64_t m = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (m >= a.M) return;
  float4 x[NV];
  float s = 0.f;
#pragma unroll
  for (int j = 0; j < NV; ++j) {
    const int i = 128 * j + 4 * lane;
    float4 v = *reinterpret_cast<const float4*>(a.delta + m * a.d_B + i);
    if (a.base) {
      const float4 bv = *reinterpret_cast<const float4*>(a.base + m * a.d_B + i);
      v.x += bv.x; v.y += bv.y; v.z += bv.z; v.w += bv.w;
    }
    v.x *= a.gamma; v.y *= a.gamma; v.z *= a.gamma; v.w *= a.gamma;
    if (a.residual) {
      if (a.res_bf16) {
        const uint2 r = *reinterpret_cast<const uint2*>(
            static_cast<const __nv_bfloat16*>(a.residual) + m * a.ldr + i);
        v.x += __uint_as_float(r.x << 16);
        v.y += __uint_as_float(r.x & 0xFFFF0000u);
        v.z += __uint_as_float(r.y << 16);
        v.w += __uint_as_float(r.y & 0xFFFF0000u);
      } else {
        const float4 r = *reinterpret_cast<const float4*>(
            static_cast<const float*>(a.residual) + m * a.ldr + i);
        v.x += r.x; v.y += r.y; v.z += r.z; v.w += r.w;
      }
    }
    x[j] = v;
    s += (v.x + v.y) + (v.z + v.w);
  }
#pragma unroll
  for (int o = 16; o; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  const float mean = s / static_cast<float>(a.d_B);
  float var = 0.f;
#pragma unroll
  for (int j = 0; j < NV; ++j) {
    const float dx = x[j].x - mean, dy = x[j].y - mean, dz = x[j].z - mean, dw = x[j].w - mean;
    var = fmaf(dx, dx, var);
    var = fmaf(dy, dy, var);
    var = fmaf(dz, dz, var);
    var = fmaf(dw, dw, var);
  }
#pragma unroll
  for (int o = 16; o; o >>= 1) var += __shfl_xor_sync(0xffffffffu, var, o);
  const float inv = rsqrtf(var / static_cast<float>(a.d_B) + a.eps);
#pragma unroll
  for (int j = 0; j < NV; ++j) {
    const int i = 128 * j + 4 * lane;
    float4 y = make_float4((x[j].x - mean) * inv, (x[j].y - mean) * inv, (x[j].z - mean) * inv,
                           (x[j].w - mean) * inv);
    if (a.ln_scale) {
      const float4 sc = *reinterpret_cast<const float4*>(a.ln_scale + i);
      y.x *= sc.x; y.y *= sc.y; y.z *= sc.z; y.w *= sc.w;
    }
    if (a.ln_bias) {
      const float4 bi = *reinterpret_cast<const float4*>(a.ln_bias + i);
      y.x += bi.x; y.y += bi.y; y.z += bi.z; y.w += bi.w;
    }
    *reinterpret_cast<float4*>(a.out + m * a.d_B + i) = y;
  }
}

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
  // Staged path: U rows of whole 16-byte words, outputs fit the consumers'
  // registers, h rows 16-byte aligned, and at least two stages fit.
  if (r % 8 == 0 && d_B <= kStgMaxOut * kStgConsumers && row_end > row_begin &&
      (ldh * (h_bf16 ? 2 : 4)) % 16 == 0 && (reinterpret_cast<uintptr_t>(h) % 16) == 0) {
    StagedArgs sa{};
    sa.a = a;
    sa.v_bytes = static_cast<uint32_t>(r) * d_A * 2;
    sa.u_bytes = static_cast<uint32_t>(d_B) * r * 2;
    sa.b_bytes = static_cast<uint32_t>(d_B) * 2;
    sa.h_bytes = static_cast<uint32_t>(d_A) * (h_bf16 ? 2 : 4);
    auto up128 = [](uint32_t x) { return (x + 127u) & ~127u; };
    sa.stage_bytes = up128(std::max(sa.v_bytes, sa.u_bytes + sa.b_bytes));
    sa.h_slot_bytes = up128(sa.h_bytes);
    const uint32_t meta_bytes = up128(static_cast<uint32_t>(4 * k * 4 + 16 + 4 * r * 4));
    const uint32_t bar_bytes = 8u * (2 * kStgMaxStages + 8) + 16u;
    // per CTA: half of an SM's shared memory; 128 more for the barrier area's alignment
    const uint32_t budget = 110u * 1024u - 2u * sa.h_slot_bytes - meta_bytes - bar_bytes - 128u;
    const int stages = static_cast<int>(std::min<uint32_t>(kStgMaxStages, budget / sa.stage_bytes));
    if (stages >= 2) {
      sa.stages = stages;
      sa.meta_off = static_cast<uint32_t>(stages) * sa.stage_bytes + 2u * sa.h_slot_bytes;
      sa.bar_off = up128(sa.meta_off + meta_bytes);
      const size_t smem = sa.bar_off + bar_bytes;
      int dev = 0, sms = 148;
      if (cudaGetDevice(&dev) == cudaSuccess)
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
      const unsigned grid = static_cast<unsigned>(std::min<int64_t>(M, kStgCtasPerSm * sms));
      cudaError_t e;
      if (h_bf16) {
        e = cudaFuncSetAttribute(lowrank_delta_staged_kernel<true>,
                                 cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
        if (e != cudaSuccess) return e;
        lowrank_delta_staged_kernel<true><<<grid, kStgThreads, smem, stream>>>(sa);
      } else {
        e = cudaFuncSetAttribute(lowrank_delta_staged_kernel<false>,
                                 cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
        if (e != cudaSuccess) return e;
        lowrank_delta_staged_kernel<false><<<grid, kStgThreads, smem, stream>>>(sa);
      }
      return cudaGetLastError();
    }
  }
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
  auto al16 = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; };
  const bool vec = d_B % 128 == 0 && d_B <= 2048 && al16(delta) && al16(out) &&
                   (base == nullptr || al16(base)) &&
                   (residual == nullptr ||
                    ((reinterpret_cast<uintptr_t>(residual) & (res_bf16 ? 7u : 15u)) == 0 &&
                     ldr % 4 == 0)) &&
                   (ln_scale == nullptr || al16(ln_scale)) && (ln_bias == nullptr || al16(ln_bias));
  if (vec) {
    switch (d_B / 128) {
#define DWA_FINISH_CASE(n) \
  case n: assemble_finish_reg_kernel<n><<<static_cast<unsigned>(blocks), 256, 0, stream>>>(a); break;
      DWA_FINISH_CASE(1) DWA_FINISH_CASE(2) DWA_FINISH_CASE(3) DWA_FINISH_CASE(4)
      DWA_FINISH_CASE(5) DWA_FINISH_CASE(6) DWA_FINISH_CASE(7) DWA_FINISH_CASE(8)
      DWA_FINISH_CASE(9) DWA_FINISH_CASE(10) DWA_FINISH_CASE(11) DWA_FINISH_CASE(12)
      DWA_FINISH_CASE(13) DWA_FINISH_CASE(14) DWA_FINISH_CASE(15) DWA_FINISH_CASE(16)
#undef DWA_FINISH_CASE
    }
    return cudaGetLastError();
  }
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
