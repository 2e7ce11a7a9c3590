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
#include "sm100_ptx.cuh"

namespace dwa {

namespace {

constexpr int kWarps = 8;
constexpr int kMaxGatherK = 128;
constexpr int kMaxPeerRanks = 16;

struct GatherArgs {
  const float* vals;
  const int32_t* gidx;
  const uint16_t* values;
  int64_t M, row_begin, row_end, ldv;
  int k, d;
  float* out;
  float* alpha_out;
  // NVLink mode (n_peers > 0): row m's partial sum goes to the inbox of the
  // rank owning row block m / block_rows, in this rank's slot
  float* inbox[kMaxPeerRanks];
  int n_peers, rank;
  int64_t block_rows;
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
  if (a.out == nullptr && a.n_peers == 0) return;  // alpha only

  float* orow = a.out + m * a.d;
  if (a.n_peers > 0) {
    const int64_t o = m / a.block_rows;
    orow = a.inbox[o] + (static_cast<int64_t>(a.rank) * a.block_rows + (m - o * a.block_rows)) * a.d;
  }
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
  GatherArgs a{};
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

namespace {

struct ReduceArgs {
  const float* inbox;  // this rank's [P][block_rows][d] partials
  float* outs[kMaxPeerRanks];
  const int32_t* flags;  // "partials ready" flag word of each rank, on this GPU
  int* status;
  int64_t block_rows, M;
  int P, rank, d, step;
  uint64_t wait_ns;  // limit of the wait for the peers' flags
};

__device__ __forceinline__ int32_t ld_acquire_sys_i32(const int32_t* p) {
  int32_t v;
  asm volatile("ld.acquire.sys.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Bounded wait of one thread for flags[0..P) >= step (gives up after wait_ns).
__device__ bool wait_flags(const int32_t* flags, int P, int step, uint64_t wait_ns) {
  const uint64_t t0 = globaltimer_ns();
  for (int p = 0; p < P; ++p) {
    while (ld_acquire_sys_i32(flags + p) < step) {
      if (globaltimer_ns() - t0 > wait_ns) return false;
    }
  }
  return true;
}

// One thread per 4 columns of one row of this rank's block: the sum of the P
// partials, written to every rank's output (NVLink stores for the others).
__global__ void __launch_bounds__(256) reduce_broadcast_kernel(const ReduceArgs a) {
  __shared__ int ready;
  if (threadIdx.x == 0) {
    ready = wait_flags(a.flags, a.P, a.step, a.wait_ns) ? 1 : 0;
    if (!ready) atomicCAS(a.status, 0, kStatusTimeout);
  }
  __syncthreads();
  if (!ready) return;
  const int c4 = a.d >> 2;
  const int64_t t = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  const int64_t row = t / c4;
  const int col = static_cast<int>(t - row * c4) * 4;
  const int64_t grow = static_cast<int64_t>(a.rank) * a.block_rows + row;
  if (row >= a.block_rows || grow >= a.M) return;
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
  for (int r = 0; r < a.P; ++r) {
    const float4 x = *reinterpret_cast<const float4*>(
        a.inbox + (static_cast<int64_t>(r) * a.block_rows + row) * a.d + col);
    acc.x += x.x;
    acc.y += x.y;
    acc.z += x.z;
    acc.w += x.w;
  }
  for (int p = 0; p < a.P; ++p)
    *reinterpret_cast<float4*>(a.outs[p] + grow * a.d + col) = acc;
}

__global__ void peer_wait_kernel(const int32_t* flags, int P, int step, uint64_t wait_ns,
                                 int* status) {
  if (threadIdx.x == 0 && !wait_flags(flags, P, step, wait_ns)) atomicCAS(status, 0, kStatusTimeout);
}

}  // namespace

cudaError_t launch_weighted_gather_peers(const float* vals, const int32_t* gidx, int64_t M, int k,
                                         const void* values, int64_t row_begin, int64_t row_end,
                                         int64_t ldv, int d, float* const* inboxes, int P, int rank,
                                         int64_t block_rows, float* alpha_out, cudaStream_t stream) {
  if (M <= 0) return cudaSuccess;
  if (k > kMaxGatherK || P < 1 || P > kMaxPeerRanks || block_rows < 1) return cudaErrorInvalidValue;
  GatherArgs a{};
  a.vals = vals;
  a.gidx = gidx;
  a.values = static_cast<const uint16_t*>(values);
  a.M = M;
  a.row_begin = row_begin;
  a.row_end = row_end;
  a.ldv = ldv;
  a.k = k;
  a.d = d;
  a.out = nullptr;
  a.alpha_out = alpha_out;
  for (int p = 0; p < P; ++p) a.inbox[p] = inboxes[p];
  a.n_peers = P;
  a.rank = rank;
  a.block_rows = block_rows;
  const int64_t blocks = (M + kWarps - 1) / kWarps;
  weighted_gather_kernel<<<static_cast<unsigned>(blocks), kWarps * 32, 0, stream>>>(a);
  return cudaGetLastError();
}

cudaError_t launch_reduce_broadcast_peers(const float* inbox, int P, int rank, int64_t block_rows,
                                          int64_t M, int d, float* const* outs, const int32_t* flags,
                                          int step, uint64_t wait_ns, int* status,
                                          cudaStream_t stream) {
  if (P < 1 || P > kMaxPeerRanks || block_rows < 1 || d % 4 != 0) return cudaErrorInvalidValue;
  ReduceArgs a{};
  a.inbox = inbox;
  for (int p = 0; p < P; ++p) a.outs[p] = outs[p];
  a.flags = flags;
  a.status = status;
  a.block_rows = block_rows;
  a.M = M;
  a.P = P;
  a.rank = rank;
  a.d = d;
  a.step = step;
  a.wait_ns = wait_ns;
  const int64_t threads = block_rows * (d / 4);
  const int64_t blocks = (threads + 255) / 256;
  reduce_broadcast_kernel<<<static_cast<unsigned>(blocks), 256, 0, stream>>>(a);
  return cudaGetLastError();
}

cudaError_t launch_peer_wait(const int32_t* flags, int P, int step, uint64_t wait_ns, int* status,
                             cudaStream_t stream) {
  if (P < 1 || P > kMaxPeerRanks) return cudaErrorInvalidValue;
  peer_wait_kernel<<<1, 32, 0, stream>>>(flags, P, step, wait_ns, status);
  return cudaGetLastError();
}

}  // namespace dwa
