// score_topk_noalloc.cu — dwa_score_topk for callers that cannot allocate
// device memory.
//
// Some hosts of this library cannot hand it a workspace: a plugin running
// inside a framework whose caching allocator has already claimed most of the
// GPU's memory (so a cudaMalloc from the plugin fails or fragments the pool),
// or a binding whose calling convention has no scratch-buffer argument and no
// allocator callback.  dwa_score_topk_noalloc serves them from a fixed scratch
// array compiled into this library instead of a caller-provided workspace.
//
// The scratch is a file-scope __device__ array of kNoAllocScratchBytes
// (128 MiB).  The CUDA runtime places it in the device memory of every GPU on
// which this file's module is loaded (with the default lazy module loading,
// at the first dwa_score_topk_noalloc call on that GPU) and keeps it there
// until the process exits.  Host code cannot use the array's name as a device
// address, so the first call on each device, with that device current, looks
// the address up once with cudaGetSymbolAddress; that first call should
// therefore happen before any stream capture.
//
// All calls on a device share the one array: the status word and the per-row
// admission bounds are re-initialised by every call (stream-ordered), and the
// partial lists are fully overwritten, but two calls whose kernels overlap on
// the GPU (different streams without ordering) race on the scratch.
//
// The scratch used is the current device's, so the stream must belong to the
// current device (a stream of another GPU is refused with
// DWA_ERR_INVALID_ARG).  Only a successful address lookup is remembered: a
// lookup that failed (for example because the first call ran inside a stream
// capture) is tried again by the next call.
#include <cuda_runtime.h>

#include <cstdint>
#include <cstdio>
#include <mutex>

#include "dwa_retrieval.h"
#include "dwa_internal.h"

namespace {

constexpr size_t kNoAllocScratchBytes = size_t(128) << 20;
constexpr int kMaxDevices = 64;

static __device__ __align__(256) uint8_t g_noalloc_scratch[kNoAllocScratchBytes];

struct DeviceScratch {
  std::mutex mu;
  void* ptr = nullptr;  // set once a lookup has succeeded
};
DeviceScratch g_scratch[kMaxDevices];

// Address of this device's scratch array (dev must be current).
cudaError_t scratch_address(int dev, void** out) {
  DeviceScratch& s = g_scratch[dev];
  std::lock_guard<std::mutex> lock(s.mu);
  if (s.ptr == nullptr) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || p == nullptr) return e != cudaSuccess ? e : cudaErrorInvalidSymbol;
    s.ptr = p;
  }
  *out = s.ptr;
  return cudaSuccess;
}

}  // namespace

extern "C" {

DWA_API dwa_status dwa_score_topk_noalloc(const void* q, int64_t M, int64_t ldq, const void* keys,
                                          int64_t N_local, int64_t ldk, int32_t d, int32_t k,
                                          float lambda_sharp, float tau, float T,
                                          int32_t use_sigmoid, int64_t idx_offset,
                                          float* out_vals, int32_t* out_idx, dwa_stream_t stream) {
  if (M > 0 && N_local > 0 && d > 0 && k > 0 && k <= DWA_MAX_K) {
    const size_t need = dwa_score_topk_workspace(M, N_local, d, k);
    if (need > kNoAllocScratchBytes) {
      char msg[256];
      snprintf(msg, sizeof(msg),
               "dwa_score_topk_noalloc: this shape needs %zu bytes of scratch, more than the "
               "built-in %zu; call dwa_score_topk with a caller-provided workspace",
               need, kNoAllocScratchBytes);
      return dwa::record_error(DWA_ERR_UNSUPPORTED_SHAPE, msg);
    }
  }
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
    char msg[256];
    snprintf(msg, sizeof(msg), "dwa_score_topk_noalloc: no usable current device (%s)",
             cudaGetErrorString(e));
    return dwa::record_error(DWA_ERR_CUDA, msg);
  }
  if (M <= 0) {
    // nothing to launch: the workspace entry point validates and returns
    return dwa_score_topk(q, M, ldq, keys, N_local, ldk, d, k, lambda_sharp, tau, T, use_sigmoid,
                          idx_offset, out_vals, out_idx, nullptr, 0, stream);
  }
  int stream_dev = dev;
  e = cudaStreamGetDevice(static_cast<cudaStream_t>(stream), &stream_dev);
  if (e != cudaSuccess) {
    char msg[256];
    snprintf(msg, sizeof(msg), "dwa_score_topk_noalloc: cudaStreamGetDevice failed (%s)",
             cudaGetErrorString(e));
    return dwa::record_error(DWA_ERR_CUDA, msg);
  }
  if (stream_dev != dev) {
    char msg[256];
    snprintf(msg, sizeof(msg),
             "dwa_score_topk_noalloc: the stream belongs to device %d but device %d is current; "
             "the built-in scratch used is the current device's",
             stream_dev, dev);
    return dwa::record_error(DWA_ERR_INVALID_ARG, msg);
  }
  void* scratch = nullptr;
  e = scratch_address(dev, &scratch);
  if (e != cudaSuccess) {
    char msg[256];
    snprintf(msg, sizeof(msg),
             "dwa_score_topk_noalloc: cudaGetSymbolAddress of the built-in scratch failed (%s); "
             "the next call tries again",
             cudaGetErrorString(e));
    return dwa::record_error(DWA_ERR_CUDA, msg);
  }
  // Same validation, kernels and results as dwa_score_topk; only the
  // workspace comes from the built-in array.
  return dwa_score_topk(q, M, ldq, keys, N_local, ldk, d, k, lambda_sharp, tau, T, use_sigmoid,
                        idx_offset, out_vals, out_idx, scratch, kNoAllocScratchBytes, stream);
}

}  // extern "C"
