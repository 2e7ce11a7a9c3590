// pair_sort.cu — the (query, entry) pairs of a top-k index array sorted by
// the pool row they selected, for the row-stationary consumers: the low-rank
// assembly (lowrank_rows.cu) and the dense row gradients (backward.cu).
//
// For gidx [n_pairs] (global row ids) and an owned row range [row_begin,
// row_end): offsets[r] .. offsets[r + 1] delimit the pairs of owned row r in
// pairs[] (pair ids i into gidx), offsets[n_rows] = the number of owned pairs.
// Counting sort: per-row counts (int atomics), an exclusive scan (per-tile
// scans, a scan of the tile totals, a fix-up), and a scatter through per-row
// cursors.  The order of the pairs inside a row is not fixed (atomics); the
// consumers either write one output per pair or accept any order.
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdint>

#include "dwa_internal.h"

namespace dwa {

namespace {

constexpr int kScanThreads = 1024;
constexpr int kScanPerThread = 4;
constexpr int kScanTile = kScanThreads * kScanPerThread;  // elements per scan block

size_t up256(size_t x) { return (x + 255) & ~size_t(255); }

__global__ void count_rows_kernel(const int32_t* gidx, int64_t n_pairs, int64_t row_begin,
                                  int64_t row_end, int32_t* counts) {
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n_pairs;
       i += stride) {
    const int32_t g = gidx[i];
    if (g >= row_begin && g < row_end) atomicAdd(counts + (g - row_begin), 1);
  }
}

// Exclusive scan of v over the block's 1024 threads; *total receives the sum.
__device__ __forceinline__ int32_t block_exclusive_scan(int32_t v, int32_t* warp_sums,
                                                        int32_t* total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int32_t x = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int32_t y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  if (lane == 31) warp_sums[warp] = x;
  __syncthreads();
  if (warp == 0) {
    int32_t w = warp_sums[lane];
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int32_t y = __shfl_up_sync(0xffffffffu, w, o);
      if (lane >= o) w += y;
    }
    warp_sums[lane] = w;  // inclusive over warps
  }
  __syncthreads();
  const int32_t before_warp = warp > 0 ? warp_sums[warp - 1] : 0;
  *total = warp_sums[31];
  __syncthreads();  // warp_sums is reused by the caller's next scan
  return before_warp + x - v;
}

// Per tile of kScanTile counts: tile-local exclusive offsets and the tile total.
__global__ void __launch_bounds__(kScanThreads) scan_tiles_kernel(const int32_t* counts,
                                                                  int64_t n, int32_t* offsets,
                                                                  int32_t* block_sums) {
  __shared__ int32_t warp_sums[32];
  const int64_t base = static_cast<int64_t>(blockIdx.x) * kScanTile + threadIdx.x * kScanPerThread;
  int32_t c[kScanPerThread];
  int32_t sum = 0;
#pragma unroll
  for (int u = 0; u < kScanPerThread; ++u) {
    c[u] = base + u < n ? counts[base + u] : 0;
    sum += c[u];
  }
  int32_t total;
  int32_t run = block_exclusive_scan(sum, warp_sums, &total);
#pragma unroll
  for (int u = 0; u < kScanPerThread; ++u) {
    if (base + u < n) offsets[base + u] = run;
    run += c[u];
  }
  if (threadIdx.x == 0) block_sums[blockIdx.x] = total;
}

// One block: exclusive scan of the tile totals in place, the grand total after them.
__global__ void __launch_bounds__(kScanThreads) scan_block_sums_kernel(int32_t* block_sums,
                                                                       int64_t n_blocks) {
  __shared__ int32_t warp_sums[32];
  int32_t carry = 0;
  for (int64_t b0 = 0; b0 < n_blocks; b0 += kScanThreads) {
    const int64_t i = b0 + threadIdx.x;
    const int32_t v = i < n_blocks ? block_sums[i] : 0;
    int32_t total;
    const int32_t ex = block_exclusive_scan(v, warp_sums, &total);
    if (i < n_blocks) block_sums[i] = carry + ex;
    carry += total;
  }
  if (threadIdx.x == 0) block_sums[n_blocks] = carry;
}

// offsets += tile base; offsets[n] = total; cursor = offsets.
__global__ void scan_finish_kernel(int32_t* offsets, int32_t* cursor, const int32_t* block_sums,
                                   int64_t n, int64_t n_blocks) {
  const int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i < n) {
    const int32_t o = offsets[i] + block_sums[i / kScanTile];
    offsets[i] = o;
    cursor[i] = o;
  } else if (i == n) {
    offsets[n] = block_sums[n_blocks];
  }
}

__global__ void scatter_pairs_kernel(const int32_t* gidx, int64_t n_pairs, int64_t row_begin,
                                     int64_t row_end, int32_t* cursor, int32_t* pairs) {
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n_pairs;
       i += stride) {
    const int32_t g = gidx[i];
    if (g >= row_begin && g < row_end) {
      const int32_t pos = atomicAdd(cursor + (g - row_begin), 1);
      pairs[pos] = static_cast<int32_t>(i);
    }
  }
}

}  // namespace

size_t pair_sort_workspace_bytes(int64_t n_pairs, int64_t n_rows) {
  const int64_t n_blocks = (n_rows + kScanTile - 1) / kScanTile;
  return up256(static_cast<size_t>(n_rows + 1) * 4) + up256(static_cast<size_t>(n_rows) * 4) +
         up256(static_cast<size_t>(n_pairs) * 4) + up256(static_cast<size_t>(n_blocks + 1) * 4);
}

cudaError_t launch_sort_pairs_by_row(const int32_t* gidx, int64_t n_pairs, int64_t row_begin,
                                     int64_t row_end, void* ws, PairSort* out,
                                     cudaStream_t stream) {
  const int64_t n_rows = row_end - row_begin;
  const int64_t n_blocks = (n_rows + kScanTile - 1) / kScanTile;
  uint8_t* p = static_cast<uint8_t*>(ws);
  int32_t* offsets = reinterpret_cast<int32_t*>(p);
  p += up256(static_cast<size_t>(n_rows + 1) * 4);
  int32_t* cursor = reinterpret_cast<int32_t*>(p);
  p += up256(static_cast<size_t>(n_rows) * 4);
  int32_t* pairs = reinterpret_cast<int32_t*>(p);
  p += up256(static_cast<size_t>(n_pairs) * 4);
  int32_t* block_sums = reinterpret_cast<int32_t*>(p);
  out->offsets = offsets;
  out->pairs = pairs;
  if (n_rows <= 0 || n_pairs <= 0) return cudaErrorInvalidValue;
  int dev = 0, sms = 148;
  if (cudaGetDevice(&dev) == cudaSuccess)
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const unsigned pair_grid =
      static_cast<unsigned>(std::min<int64_t>((n_pairs + 255) / 256, static_cast<int64_t>(sms) * 8));
  cudaError_t e = cudaMemsetAsync(cursor, 0, static_cast<size_t>(n_rows) * 4, stream);
  if (e != cudaSuccess) return e;
  count_rows_kernel<<<pair_grid, 256, 0, stream>>>(gidx, n_pairs, row_begin, row_end, cursor);
  scan_tiles_kernel<<<static_cast<unsigned>(n_blocks), kScanThreads, 0, stream>>>(
      cursor, n_rows, offsets, block_sums);
  scan_block_sums_kernel<<<1, kScanThreads, 0, stream>>>(block_sums, n_blocks);
  scan_finish_kernel<<<static_cast<unsigned>((n_rows + 1 + 255) / 256), 256, 0, stream>>>(
      offsets, cursor, block_sums, n_rows, n_blocks);
  scatter_pairs_kernel<<<pair_grid, 256, 0, stream>>>(gidx, n_pairs, row_begin, row_end, cursor,
                                                      pairs);
  return cudaGetLastError();
}

}  // namespace dwa
