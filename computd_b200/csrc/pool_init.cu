// pool_init.cu — counter-based normal initialisation of pool shards and queries.
//
// Counterpart of VectorPool's per-shard creation (src/model/pool.py:19-40),
// which draws each device's rows with jax.random.normal(fold_in(key, dev)).
// Here element (r, c) depends only on (seed, global row, column): the shard
// [row_offset, row_offset + rows) comes out identical for every shard count,
// so 1-, 2-, 4- and 8-GPU runs retrieve from the same pool.
//
// Generator: Philox4x32-10 (Salmon, Moraes, Dror, Shaw, "Parallel random
// numbers: as easy as 1, 2, 3", SC'11), counter = (column group, row lo,
// row hi, tag), key = seed; the four 32-bit outputs feed two Box-Muller pairs
// (24-bit uniforms in (0, 1)), giving four N(0,1) values per column group of 4.
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "dwa_internal.h"

namespace dwa {

namespace {

constexpr uint32_t kPhiloxM0 = 0xD2511F53u;
constexpr uint32_t kPhiloxM1 = 0xCD9E8D57u;
constexpr uint32_t kPhiloxW0 = 0x9E3779B9u;
constexpr uint32_t kPhiloxW1 = 0xBB67AE85u;
constexpr uint32_t kCounterTag = 0x706F6F6Cu;  // fourth counter word

__device__ __forceinline__ uint4 philox4x32_10(uint4 c, uint2 k) {
#pragma unroll
  for (int r = 0; r < 10; ++r) {
    if (r > 0) {
      k.x += kPhiloxW0;
      k.y += kPhiloxW1;
    }
    const uint32_t hi0 = __umulhi(kPhiloxM0, c.x);
    const uint32_t lo0 = kPhiloxM0 * c.x;
    const uint32_t hi1 = __umulhi(kPhiloxM1, c.z);
    const uint32_t lo1 = kPhiloxM1 * c.z;
    c = make_uint4(hi1 ^ c.y ^ k.x, lo1, hi0 ^ c.w ^ k.y, lo0);
  }
  return c;
}

__device__ __forceinline__ float unit_open(uint32_t x) {
  return (static_cast<float>(x >> 8) + 0.5f) * 5.9604644775390625e-08f;  // 2^-24
}

__global__ void pool_init_kernel(__nv_bfloat16* out, int64_t rows, int64_t cols, int64_t ld,
                                 int64_t row_offset, uint2 key, float stddev) {
  const int64_t groups = (cols + 3) / 4;
  const int64_t total = rows * groups;
  for (int64_t g = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; g < total;
       g += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t r = g / groups;
    const int64_t cg = g - r * groups;
    const uint64_t grow = static_cast<uint64_t>(row_offset + r);
    const uint4 x = philox4x32_10(
        make_uint4(static_cast<uint32_t>(cg), static_cast<uint32_t>(grow),
                   static_cast<uint32_t>(grow >> 32), kCounterTag),
        key);
    float z[4];
    {
      const float rad = sqrtf(-2.0f * logf(unit_open(x.x)));
      float sn, cs;
      sincospif(2.0f * unit_open(x.y), &sn, &cs);
      z[0] = rad * cs;
      z[1] = rad * sn;
    }
    {
      const float rad = sqrtf(-2.0f * logf(unit_open(x.z)));
      float sn, cs;
      sincospif(2.0f * unit_open(x.w), &sn, &cs);
      z[2] = rad * cs;
      z[3] = rad * sn;
    }
    __nv_bfloat16* dst = out + r * ld + cg * 4;
    const int64_t c0 = cg * 4;
#pragma unroll
    for (int e = 0; e < 4; ++e)
      if (c0 + e < cols) dst[e] = __float2bfloat16_rn(z[e] * stddev);
  }
}

}  // namespace

cudaError_t launch_pool_init_normal(void* out, int64_t rows, int64_t cols, int64_t ld,
                                    int64_t row_offset, uint64_t seed, float stddev,
                                    cudaStream_t stream) {
  if (rows <= 0 || cols <= 0) return cudaSuccess;
  const int64_t total = rows * ((cols + 3) / 4);
  const int threads = 256;
  int64_t blocks = (total + threads - 1) / threads;
  const int64_t cap = static_cast<int64_t>(device_sm_count()) * 16;
  if (blocks > cap) blocks = cap;
  const uint2 key = make_uint2(static_cast<uint32_t>(seed), static_cast<uint32_t>(seed >> 32));
  pool_init_kernel<<<static_cast<unsigned>(blocks), threads, 0, stream>>>(
      static_cast<__nv_bfloat16*>(out), rows, cols, ld, row_offset, key, stddev);
  return cudaGetLastError();
}

}  // namespace dwa
