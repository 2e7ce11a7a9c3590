// score_params.cuh — the runtime scalars of the fused score (lambda_sharp,
// tau, T), taken either from host values or from a device array.
//
// The reference passes them to its kernel as (1,)-shaped f32 operands so that
// a learned tau never forces a recompile or a host read
// (src/kernels/tiled_topk.py:26-29, 112-115).  The *_dev entry points of the
// C ABI keep that property: `params` points at three device floats
// {lambda_sharp, tau, T} read by the kernel itself, so the caller's stream
// never waits for the host.  Values the selection cannot honour (T <= 0, a
// negative or non-finite lambda with the gate on) are caught on the device:
// the kernel records DWA_ERR_DEVICE_CHECK in its status word and writes NaN
// scores / -1 indices instead of a wrong top-k.
#pragma once

#include <cmath>
#include <cstdint>

namespace dwa {

constexpr int kStatusDeviceCheck = 5;  // DWA_ERR_DEVICE_CHECK

struct ScoreParams {
  float lambda_sharp, tau, T;
};

// `dev` (three floats) wins over the host values when non-null.
__device__ __forceinline__ ScoreParams load_score_params(const float* dev, float lambda_sharp,
                                                         float tau, float T) {
  if (dev != nullptr) return ScoreParams{__ldg(dev), __ldg(dev + 1), __ldg(dev + 2)};
  return ScoreParams{lambda_sharp, tau, T};
}

// v(s) = [sigmoid(lambda (s - tau))] * exp(s / T) is strictly increasing in s
// exactly when these hold, which is what selection on raw scores needs.
__device__ __forceinline__ bool score_params_ok(const ScoreParams& p, int use_sigmoid) {
  if (!(p.T > 0.0f) || !isfinite(p.T)) return false;
  if (use_sigmoid && (!(p.lambda_sharp >= 0.0f) || !isfinite(p.lambda_sharp) || !isfinite(p.tau)))
    return false;
  return true;
}

// 2^x and 1/x as single special-function-unit instructions (PTX ex2.approx and
// rcp.approx, subnormals flushed to zero).
__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
__device__ __forceinline__ float rcp_approx(float x) {
  float y;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
constexpr float kLog2e = 1.4426950408889634f;  // log2(e): e^x = 2^(x log2 e)

__device__ __forceinline__ void record_status(int* status, int code) {
  if (status != nullptr) atomicCAS(status, 0, code);
}

}  // namespace dwa
