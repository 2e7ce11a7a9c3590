// capi.cu — the exported C ABI (include/dwa_retrieval.h).
//
// Every entry point validates its arguments on the host before enqueueing
// anything; a rejected call launches nothing and leaves a message in
// dwa_last_error().  The reference raises Python exceptions at trace time for
// the same conditions (e.g. lax.top_k with k > N); here they are status codes.
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <string>

#include "dwa_retrieval.h"
#include "dwa_lm.h"
#include "dwa_internal.h"

namespace {

thread_local std::string g_last_error;

dwa_status fail(dwa_status s, const char* fmt, ...) __attribute__((format(printf, 2, 3)));
dwa_status fail(dwa_status s, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return s;
}

dwa_status cuda_fail(cudaError_t e, const char* where, const char* detail = nullptr) {
  return fail(DWA_ERR_CUDA, "%s: %s%s%s", where, cudaGetErrorString(e), detail ? " — " : "",
              detail ? detail : "");
}

bool aligned(const void* p, uintptr_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

uint64_t peer_wait_ns(int64_t wait_ns) {
  if (wait_ns <= 0) return dwa::kPeerWaitDefaultNs;
  return std::min<uint64_t>(static_cast<uint64_t>(wait_ns), dwa::kPeerWaitMaxNs);
}

dwa_status ok() {
  g_last_error.clear();
  return DWA_OK;
}

}  // namespace

namespace dwa {
// Lets other translation units of the library report through dwa_last_error().
dwa_status record_error(dwa_status s, const char* msg) {
  g_last_error = msg ? msg : "";
  return s;
}
}  // namespace dwa

extern "C" {

int32_t dwa_abi_version(void) { return DWA_ABI_VERSION; }

const char* dwa_status_string(dwa_status s) {
  switch (s) {
    case DWA_OK: return "DWA_OK";
    case DWA_ERR_INVALID_ARG: return "DWA_ERR_INVALID_ARG";
    case DWA_ERR_UNSUPPORTED_SHAPE: return "DWA_ERR_UNSUPPORTED_SHAPE";
    case DWA_ERR_CUDA: return "DWA_ERR_CUDA";
    case DWA_ERR_TIMEOUT: return "DWA_ERR_TIMEOUT";
    case DWA_ERR_DEVICE_CHECK: return "DWA_ERR_DEVICE_CHECK";
    case DWA_ERR_WORKSPACE: return "DWA_ERR_WORKSPACE";
    default: return "DWA_ERR_UNKNOWN";
  }
}

const char* dwa_last_error(void) { return g_last_error.c_str(); }

size_t dwa_score_topk_workspace(int64_t M, int64_t N_local, int32_t d, int32_t k) {
  if (M <= 0 || N_local <= 0 || d <= 0 || k <= 0 || k > DWA_MAX_K) return 0;
  dwa::ScoreTopkPlan plan;
  if (!dwa::plan_score_topk(M, N_local, d, k, dwa::device_sm_count(), &plan)) return 0;
  return plan.ws_bytes;
}

}  // extern "C"

namespace {
// dwa_score_topk with the runtime scalars either as host values (params ==
// nullptr, checked here) or as a device array {lambda_sharp, tau, T}
// (checked by the merge kernel, which records DWA_ERR_DEVICE_CHECK).
dwa_status score_topk_impl(const char* fn, const void* q, int64_t M, int64_t ldq,
                           const void* keys, int64_t N_local, int64_t ldk, int32_t d, int32_t k,
                           float lambda_sharp, float tau, float T, const float* params,
                           int32_t use_sigmoid, int64_t idx_offset, float* out_vals,
                           int32_t* out_idx, void* ws, size_t ws_bytes, dwa_stream_t stream,
                           const dwa::SeqMeanOut* seq_mean = nullptr) {
  if (M < 0 || N_local < 0) return fail(DWA_ERR_INVALID_ARG, "%s: negative size (M=%lld, N=%lld)",
                                        fn, (long long)M, (long long)N_local);
  if (M == 0) return ok();
  if (!q || !keys || !out_vals || !out_idx)
    return fail(DWA_ERR_INVALID_ARG, "null queries/keys/output pointer");
  if (N_local == 0) return fail(DWA_ERR_INVALID_ARG, "empty key shard (N_local = 0)");
  if (k < 1 || k > N_local)
    return fail(DWA_ERR_INVALID_ARG, "k=%d must satisfy 1 <= k <= N_local=%lld", k,
                (long long)N_local);
  if (k > DWA_MAX_K)
    return fail(DWA_ERR_UNSUPPORTED_SHAPE, "k=%d exceeds DWA_MAX_K=%d", k, DWA_MAX_K);
  if (d < 8 || d % 8 != 0)
    return fail(DWA_ERR_UNSUPPORTED_SHAPE, "d=%d must be a positive multiple of 8", d);
  if (ldq < d || ldk < d)
    return fail(DWA_ERR_INVALID_ARG, "row stride below d (ldq=%lld, ldk=%lld, d=%d)",
                (long long)ldq, (long long)ldk, d);
  if (ldq % 8 != 0 || ldk % 8 != 0)
    return fail(DWA_ERR_UNSUPPORTED_SHAPE, "row strides must be multiples of 8 elements");
  if (!aligned(q, 16) || !aligned(keys, 16))
    return fail(DWA_ERR_INVALID_ARG, "queries and keys must be 16-byte aligned");
  if (M > INT32_MAX || N_local > INT32_MAX)
    return fail(DWA_ERR_UNSUPPORTED_SHAPE, "M and N_local must be < 2^31");
  if (idx_offset < 0 || N_local + idx_offset > INT32_MAX)
    return fail(DWA_ERR_INVALID_ARG, "idx_offset=%lld out of the int32 index range",
                (long long)idx_offset);
  if (params != nullptr) {
    if (!aligned(params, 4)) return fail(DWA_ERR_INVALID_ARG, "%s: params must be 4-byte aligned", fn);
  } else {
    if (!(T > 0.f) || !std::isfinite(T))
      return fail(DWA_ERR_UNSUPPORTED_SHAPE, "temperature T must be finite and > 0");
    if (use_sigmoid && (!(lambda_sharp >= 0.f) || !std::isfinite(lambda_sharp) ||
                        !std::isfinite(tau)))
      return fail(DWA_ERR_UNSUPPORTED_SHAPE,
                  "the gate needs finite lambda_sharp >= 0 and finite tau (selection on raw "
                  "scores requires a monotone gate)");
  }
  dwa::ScoreTopkPlan plan;
  if (!dwa::plan_score_topk(M, N_local, d, k, dwa::device_sm_count(), &plan))
    return fail(DWA_ERR_UNSUPPORTED_SHAPE, "no launch plan for this shape");
  if (!ws || !aligned(ws, 256))
    return fail(DWA_ERR_WORKSPACE, "workspace must be non-null and 256-byte aligned");
  if (ws_bytes < plan.ws_bytes)
    return fail(DWA_ERR_WORKSPACE, "workspace too small: %zu < %zu bytes", ws_bytes,
                plan.ws_bytes);
  const char* detail = nullptr;
  cudaError_t e = dwa::launch_score_topk(plan, q, ldq, keys, ldk, lambda_sharp, tau, T,
                                         use_sigmoid ? 1 : 0, idx_offset, out_vals, out_idx, ws,
                                         static_cast<cudaStream_t>(stream), &detail, params,
                                         seq_mean);
  if (e != cudaSuccess) return cuda_fail(e, fn, detail);
  return ok();
}

dwa_status project_keys_impl(const char* fn, const void* vectors, int64_t N, int64_t ldv, int32_t D,
                             const void* w_k, int64_t ldw, int32_t S, int32_t d_k,
                             const float* aspect_w, void* keys_out, int64_t ldo, int32_t* status,
                             dwa_stream_t stream, bool packed) {
  if (N < 0) return fail(DWA_ERR_INVALID_ARG, "%s: negative N", fn);
  if (N == 0) return ok();
  if (!vectors || !w_k || !aspect_w || !keys_out)
    return fail(DWA_ERR_INVALID_ARG, "%s: null argument", fn);
  if (d_k != 32 && d_k != 64 && d_k != 128)
    return fail(DWA_ERR_UNSUPPORTED_SHAPE, "%s: d_k=%d must be 32, 64 or 128", fn, d_k);
  if (S < 1 || static_cast<int64_t>(S) * d_k > (1 << 20))
    return fail(DWA_ERR_UNSUPPORTED_SHAPE, "%s: S=%d outside [1, 2^20 / d_k]", fn, S);
  if (D < 8 || D % 8 != 0)
    return fail(DWA_ERR_UNSUPPORTED_SHAPE, "%s: D=%d must be a positive multiple of 8", fn, D);
  if (N > INT32_MAX - 256) return fail(DWA_ERR_UNSUPPORTED_SHAPE, "%s: N too large", fn);
  const int64_t out_cols = packed ? static_cast<int64_t>(S) * d_k : d_k;
  if (ldv < D || ldw < D || ldo < out_cols)
    return fail(DWA_ERR_INVALID_ARG, "%s: a row stride is below its row length", fn);
  if (ldv % 8 || ldw % 8 || ldo % 8 || !aligned(vectors, 16) || !aligned(w_k, 16) ||
      !aligned(keys_out, 16))
    return fail(DWA_ERR_UNSUPPORTED_SHAPE,
                "%s: 16-byte aligned bases and strides (multiples of 8) required", fn);
  cudaError_t e = dwa::launch_project_keys(vectors, N, ldv, D, w_k, ldw, S, d_k, aspect_w, keys_out,
                                           ldo, status, static_cast<cudaStream_t>(stream), packed);
  if (e != cudaSuccess) return cuda_fail(e, fn);
  return ok();
}
}  // namespace

extern "C" {

dwa_status dwa_score_topk(const void* q, int64_t M, int64_t ldq, const void* keys,
                          int64_t N_local, int64_t ldk, int32_t d, int32_t k, float lambda_sharp,
                          float tau, float T, int32_t use_sigmoid, int64_t idx_offset,
                          float* out_vals, int32_t* out_idx, void* ws, size_t ws_bytes,
                          dwa_stream_t stream) {
  return score_topk_impl("dwa_score_topk", q, M, ldq, keys, N_local, ldk, d, k, lambda_sharp, tau,
                         T, nullptr, use_sigmoid, idx_offset, out_vals, out_idx, ws, ws_bytes,
                         stream);
}

dwa_status dwa_score_topk_dev(const void* q, int64_t M, int64_t ldq, const void* keys,
                              int64_t N_local, int64_t ldk, int32_t d, int32_t k,
                              const float* params, int32_t use_sigmoid, int64_t idx_offset,
                              float* out_vals, int32_t* out_idx, void* ws, size_t ws_bytes,
                              dwa_stream_t stream) {
  if (M > 0 && !params) return fail(DWA_ERR_INVALID_ARG, "dwa_score_topk_dev: null params");
  return score_topk_impl("dwa_score_topk_dev", q, M, ldq, keys, N_local, ldk, d, k, 0.f, 0.f, 1.f,
                         params, use_sigmoid, idx_offset, out_vals, out_idx, ws, ws_bytes, stream);
}

dwa_status dwa_score_topk_seqmean(const void* q, int64_t M, int64_t ldq, const void* keys,
                                  int64_t N_local, int64_t ldk, int32_t d, int32_t k,
                                  const float* params, int32_t use_sigmoid, int64_t idx_offset,
                                  int64_t seq, float* fused_mean, int64_t ld_mean, float* out_vals,
                                  int32_t* out_idx, void* ws, size_t ws_bytes,
                                  dwa_stream_t stream) {
  if (M > 0) {
    if (!params) return fail(DWA_ERR_INVALID_ARG, "dwa_score_topk_seqmean: null params");
    if (!fused_mean) return fail(DWA_ERR_INVALID_ARG, "dwa_score_topk_seqmean: null fused_mean");
    if (seq < 1 || M % seq != 0)
      return fail(DWA_ERR_INVALID_ARG, "dwa_score_topk_seqmean: seq=%lld must divide M=%lld",
                  (long long)seq, (long long)M);
    if (ld_mean < N_local)
      return fail(DWA_ERR_INVALID_ARG, "dwa_score_topk_seqmean: ld_mean below N_local");
    if (!aligned(fused_mean, 4))
      return fail(DWA_ERR_INVALID_ARG, "dwa_score_topk_seqmean: fused_mean must be 4-byte aligned");
  }
  dwa::SeqMeanOut sm{fused_mean, ld_mean, seq < 1 ? 1 : seq};
  return score_topk_impl("dwa_score_topk_seqmean", q, M, ldq, keys, N_local, ldk, d, k, 0.f, 0.f,
                         1.f, params, use_sigmoid, idx_offset, out_vals, out_idx, ws, ws_bytes,
                         stream, &sm);
}

dwa_status dwa_seq_scores(const float* q, int64_t B, int64_t ldq, const void* keys, int64_t N,
                          int64_t ldk, int32_t d, const float* params, int32_t use_sigmoid,
                          float* sims, int64_t lds, float* fused, int64_t ldf, int32_t* status,
                          dwa_stream_t stream) {
  if (B < 0 || N < 0) return fail(DWA_ERR_INVALID_ARG, "dwa_seq_scores: negative size");
  if (B == 0 || N == 0) return ok();
  if (!q || !keys || !sims) return fail(DWA_ERR_INVALID_ARG, "dwa_seq_scores: null q/keys/sims");
  if (fused && !params)
    return fail(DWA_ERR_INVALID_ARG, "dwa_seq_scores: the fused scores need the params array");
  if (d < 8 || d % 8 != 0 || d > dwa::seq_scores_max_d())
    return fail(DWA_ERR_UNSUPPORTED_SHAPE, "dwa_seq_scores: d=%d must be a multiple of 8 in [8, %d]",
                d, dwa::seq_scores_max_d());
  if (ldq < d || ldk < d || lds < N || (fused && ldf < N))
    return fail(DWA_ERR_INVALID_ARG, "dwa_seq_scores: a row stride is below its row length");
  if (ldk % 8 != 0 || !aligned(keys, 16))
    return fail(DWA_ERR_UNSUPPORTED_SHAPE, "dwa_seq_scores: keys need 16-byte aligned rows");
  if (!aligned(q, 4) || !aligned(sims, 4) || (fused && !aligned(fused, 4)) ||
      (params && !aligned(params, 4)))
    return fail(DWA_ERR_INVALID_ARG, "dwa_seq_scores: f32 arrays must be 4-byte aligned");
  if (N > INT32_MAX) return fail(DWA_ERR_UNSUPPORTED_SHAPE, "dwa_seq_scores: N too large");
  cudaError_t e = dwa::launch_seq_scores(q, B, ldq, keys, N, ldk, d, params, use_sigmoid ? 1 : 0,
                                         sims, lds, fused, ldf, status,
                                         static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "dwa_seq_scores launch");
  return ok();
}

dwa_status dwa_merge_topk(const float* cand_vals, const int32_t* cand_idx, int32_t P, int64_t M,
                          int32_t k, float* out_vals, int32_t* out_idx, dwa_stream_t stream) {
  if (M < 0) return fail(DWA_ERR_INVALID_ARG, "negative M");
  if (M == 0) return ok();
  if (!cand_vals || !cand_idx || !out_vals || !out_idx)
    return fail(DWA_ERR_INVALID_ARG, "null pointer");
  if (P < 1) return fail(DWA_ERR_INVALID_ARG, "P=%d must be >= 1", P);
  if (P > dwa::kMaxSplits)
    return fail(DWA_ERR_UNSUPPORTED_SHAPE, "P=%d exceeds %d lists", P, dwa::kMaxSplits);
  if (k < 1) return fail(DWA_ERR_INVALID_ARG, "k=%d must be >= 1", k);
  if (k > DWA_MAX_K)
    return fail(DWA_ERR_UNSUPPORTED_SHAPE, "k=%d exceeds DWA_MAX_K=%d", k, DWA_MAX_K);
  if (static_cast<const void*>(out_vals) == static_cast<const void*>(cand_vals) ||
      static_cast<const void*>(out_idx) == static_cast<const void*>(cand_idx))
    return fail(DWA_ERR_INVALID_ARG, "outputs must not alias the candidate lists");
  cudaError_t e = dwa::launch_merge_topk(
      cand_vals, cand_idx, P, k, M * static_cast<int64_t>(k), 1, k, M, k, /*transform=*/0, 0.f,
      0.f, 1.f, 0, /*idx_offset=*/0, out_vals, out_idx, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "dwa_merge_topk launch");
  return ok();
}

dwa_status dwa_merge_topk_strided(const float* cand_vals, const int32_t* cand_idx, int32_t P,
                                  int64_t M, int32_t k, int64_t stride_list, int64_t stride_pos,
                                  int64_t stride_row, float* out_vals, int32_t* out_idx,
                                  dwa_stream_t stream) {
  if (M < 0) return fail(DWA_ERR_INVALID_ARG, "negative M");
  if (M == 0) return ok();
  if (!cand_vals || !cand_idx || !out_vals || !out_idx)
    return fail(DWA_ERR_INVALID_ARG, "null pointer");
  if (P < 1) return fail(DWA_ERR_INVALID_ARG, "P=%d must be >= 1", P);
  if (P > dwa::kMaxSplits)
    return fail(DWA_ERR_UNSUPPORTED_SHAPE, "P=%d exceeds %d lists", P, dwa::kMaxSplits);
  if (k < 1) return fail(DWA_ERR_INVALID_ARG, "k=%d must be >= 1", k);
  if (k > DWA_MAX_K)
    return fail(DWA_ERR_UNSUPPORTED_SHAPE, "k=%d exceeds DWA_MAX_K=%d", k, DWA_MAX_K);
  if (stride_list < 0 || stride_pos < 0 || stride_row < 0)
    return fail(DWA_ERR_INVALID_ARG, "negative stride");
  if (!aligned(cand_vals, 4) || !aligned(cand_idx, 4))
    return fail(DWA_ERR_INVALID_ARG, "candidate arrays must be 4-byte aligned");
  cudaError_t e = dwa::launch_merge_topk(cand_vals, cand_idx, P, k, stride_list, stride_pos,
                                         stride_row, M, k, /*transform=*/0, 0.f, 0.f, 1.f, 0,
                                         /*idx_offset=*/0, out_vals, out_idx,
                                         static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "dwa_merge_topk_strided launch");
  return ok();
}

dwa_status dwa_weighted_gather(const float* vals, const int32_t* gidx, int64_t M, int32_t k,
                               const void* values, int64_t row_begin, int64_t row_end,
                               int64_t ldv, int32_t d, float* out, float* alpha_out,
                               dwa_stream_t stream) {
  if (M < 0) return fail(DWA_ERR_INVALID_ARG, "negative M");
  if (M == 0) return ok();
  if (!vals || !gidx) return fail(DWA_ERR_INVALID_ARG, "null vals/gidx pointer");
  if (!out && row_end > row_begin)
    return fail(DWA_ERR_INVALID_ARG, "null out with a non-empty owned row range");
  if (!out && !alpha_out) return fail(DWA_ERR_INVALID_ARG, "nothing to compute (out and alpha_out null)");
  if (k < 1) return fail(DWA_ERR_INVALID_ARG, "k=%d must be >= 1", k);
  if (k > DWA_MAX_K)
    return fail(DWA_ERR_UNSUPPORTED_SHAPE, "k=%d exceeds DWA_MAX_K=%d", k, DWA_MAX_K);
  if (d < 8 || d % 8 != 0)
    return fail(DWA_ERR_UNSUPPORTED_SHAPE, "d=%d must be a positive multiple of 8", d);
  if (row_begin < 0 || row_end < row_begin || row_end > INT32_MAX)
    return fail(DWA_ERR_INVALID_ARG, "bad owned row range [%lld, %lld)", (long long)row_begin,
                (long long)row_end);
  if (row_end > row_begin) {
    if (!values) return fail(DWA_ERR_INVALID_ARG, "null values with a non-empty row range");
    if (ldv < d) return fail(DWA_ERR_INVALID_ARG, "ldv=%lld below d=%d", (long long)ldv, d);
    if (ldv % 8 != 0)
      return fail(DWA_ERR_UNSUPPORTED_SHAPE, "ldv must be a multiple of 8 elements");
    if (!aligned(values, 16))
      return fail(DWA_ERR_INVALID_ARG, "values must be 16-byte aligned");
  }
  if (out && !aligned(out, 16)) return fail(DWA_ERR_INVALID_ARG, "out must be 16-byte aligned");
  cudaError_t e = dwa::launch_weighted_gather(vals, gidx, M, k, values, row_begin, row_end, ldv, d,
                                              out, alpha_out, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "dwa_weighted_gather launch");
  return ok();
}

namespace {
// Shared checks of the backward entry points; returns DWA_OK or a failure.
dwa_status check_rows_args(const char* fn, const int32_t* gidx, int64_t M, int32_t k,
                           const void* rows_or_grad, int64_t row_begin, int64_t row_end,
                           int64_t ld, int32_t d, int ld_mult) {
  if (!gidx) return fail(DWA_ERR_INVALID_ARG, "%s: null index array", fn);
  if (k < 1) return fail(DWA_ERR_INVALID_ARG, "%s: k=%d must be >= 1", fn, k);
  if (d < 8 || d % 8 != 0)
    return fail(DWA_ERR_UNSUPPORTED_SHAPE, "%s: d=%d must be a positive multiple of 8", fn, d);
  if (row_begin < 0 || row_end < row_begin || row_end > INT32_MAX)
    return fail(DWA_ERR_INVALID_ARG, "%s: bad owned row range", fn);
  if (row_end > row_begin) {
    if (!rows_or_grad) return fail(DWA_ERR_INVALID_ARG, "%s: null rows with a non-empty range", fn);
    if (ld < d) return fail(DWA_ERR_INVALID_ARG, "%s: row stride below d", fn);
    if (ld % ld_mult != 0)
      return fail(DWA_ERR_UNSUPPORTED_SHAPE, "%s: row stride must be a multiple of %d", fn, ld_mult);
    if (!aligned(rows_or_grad, 16)) return fail(DWA_ERR_INVALID_ARG, "%s: rows not 16-byte aligned", fn);
  }
  (void)M;
  return DWA_OK;
}
dwa_status check_vec_arg(const char* fn, const void* a, int32_t a_bf16, int64_t lda, int32_t d) {
  if (!a) return fail(DWA_ERR_INVALID_ARG, "%s: null row-vector array", fn);
  if (lda < d) return fail(DWA_ERR_INVALID_ARG, "%s: lda below d", fn);
  if (lda % (a_bf16 ? 8 : 4) != 0 || !aligned(a, 16))
    return fail(DWA_ERR_UNSUPPORTED_SHAPE, "%s: row vectors need 16-byte aligned rows", fn);
  return DWA_OK;
}
}  // namespace

dwa_status dwa_gather_dot(const void* a, int32_t a_is_bf16, int64_t lda, const int32_t* gidx,
                          int64_t M, int32_t k, const void* rows, int64_t row_begin,
                          int64_t row_end, int64_t ldr, int32_t d, float* out,
                          dwa_stream_t stream) {
  if (M < 0) return fail(DWA_ERR_INVALID_ARG, "negative M");
  if (M == 0) return ok();
  if (!out) return fail(DWA_ERR_INVALID_ARG, "dwa_gather_dot: null out");
  dwa_status st = check_rows_args("dwa_gather_dot", gidx, M, k, rows, row_begin, row_end, ldr, d, 8);
  if (st == DWA_OK) st = check_vec_arg("dwa_gather_dot", a, a_is_bf16, lda, d);
  if (st != DWA_OK) return st;
  cudaError_t e = dwa::launch_gather_dot(a, a_is_bf16 ? 1 : 0, lda, gidx, M, k, rows, row_begin,
                                         row_end, ldr, d, out, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "dwa_gather_dot launch");
  return ok();
}

dwa_status dwa_score_backward(const float* vals, const float* scores, const float* dalpha,
                              int64_t M, int32_t k, float lambda_sharp, float tau, float T,
                              int32_t use_sigmoid, float* dscores, float* dparams,
                              dwa_stream_t stream) {
  if (M < 0) return fail(DWA_ERR_INVALID_ARG, "negative M");
  if (M == 0) return ok();
  if (!vals || !scores || !dalpha || !dscores)
    return fail(DWA_ERR_INVALID_ARG, "dwa_score_backward: null pointer");
  if (k < 1) return fail(DWA_ERR_INVALID_ARG, "k=%d must be >= 1", k);
  if (!(T > 0.f) || !std::isfinite(T))
    return fail(DWA_ERR_UNSUPPORTED_SHAPE, "temperature T must be finite and > 0");
  cudaError_t e = dwa::launch_score_backward(vals, scores, dalpha, M, k, lambda_sharp, tau, T,
                                             use_sigmoid ? 1 : 0, dscores, dparams,
                                             static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "dwa_score_backward launch");
  return ok();
}

dwa_status dwa_score_backward_dev(const float* vals, const float* scores, const float* dalpha,
                                  int64_t M, int32_t k, const float* params, int32_t use_sigmoid,
                                  float* dscores, float* dparams, int32_t* status,
                                  dwa_stream_t stream) {
  if (M < 0) return fail(DWA_ERR_INVALID_ARG, "negative M");
  if (M == 0) return ok();
  if (!vals || !scores || !dalpha || !dscores || !params)
    return fail(DWA_ERR_INVALID_ARG, "dwa_score_backward_dev: null pointer");
  if (!aligned(params, 4)) return fail(DWA_ERR_INVALID_ARG, "dwa_score_backward_dev: params misaligned");
  if (k < 1) return fail(DWA_ERR_INVALID_ARG, "k=%d must be >= 1", k);
  cudaError_t e = dwa::launch_score_backward(vals, scores, dalpha, M, k, 0.f, 0.f, 1.f,
                                             use_sigmoid ? 1 : 0, dscores, dparams,
                                             static_cast<cudaStream_t>(stream), params, status);
  if (e != cudaSuccess) return cuda_fail(e, "dwa_score_backward_dev launch");
  return ok();
}

dwa_status dwa_retrieval_backward(const void* q, int32_t q_is_bf16, int64_t ldq,
                                  const float* dout, int64_t ld_dout, const void* keys,
                                  int64_t ldk, int32_t d_k, const void* values, int64_t ldv,
                                  int32_t d_v, const float* vals, const int32_t* gidx, int64_t M,
                                  int32_t k, int64_t row_begin, int64_t row_end,
                                  float lambda_sharp, float tau, float T, const float* params,
                                  int32_t use_sigmoid, float* dscores, float* dq, float* dparams,
                                  int32_t* status, dwa_stream_t stream) {
  const char* fn = "dwa_retrieval_backward";
  if (M < 0) return fail(DWA_ERR_INVALID_ARG, "%s: negative M", fn);
  if (M == 0) return ok();
  if (M > INT32_MAX) return fail(DWA_ERR_UNSUPPORTED_SHAPE, "%s: M too large", fn);
  if (k > 128) return fail(DWA_ERR_UNSUPPORTED_SHAPE, "%s: k=%d above 128", fn, k);
  if (!vals || !dscores || !dq) return fail(DWA_ERR_INVALID_ARG, "%s: null vals/dscores/dq", fn);
  if (!aligned(dq, 16) || d_k % 4 != 0)
    return fail(DWA_ERR_INVALID_ARG, "%s: dq must be 16-byte aligned", fn);
  if (params && !status)
    return fail(DWA_ERR_INVALID_ARG, "%s: device params need a status word", fn);
  if (!params && (!(T > 0.f) || !std::isfinite(T)))
    return fail(DWA_ERR_UNSUPPORTED_SHAPE, "%s: temperature T must be finite and > 0", fn);
  dwa_status st = check_rows_args(fn, gidx, M, k, keys, row_begin, row_end, ldk, d_k, 8);
  if (st == DWA_OK) st = check_rows_args(fn, gidx, M, k, values, row_begin, row_end, ldv, d_v, 8);
  if (st == DWA_OK) st = check_vec_arg(fn, q, q_is_bf16, ldq, d_k);
  if (st == DWA_OK) st = check_vec_arg(fn, dout, 0, ld_dout, d_v);
  if (st != DWA_OK) return st;
  cudaError_t e = dwa::launch_retrieval_backward(
      q, q_is_bf16 ? 1 : 0, ldq, dout, ld_dout, keys, ldk, d_k, values, ldv, d_v, vals, gidx, M, k,
      row_begin, row_end, lambda_sharp, tau, T, params, use_sigmoid ? 1 : 0, dscores, dq, dparams,
      status, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "dwa_retrieval_backward launch");
  return ok();
}

size_t dwa_row_gradient_workspace(int64_t M, int32_t k, int64_t n_rows) {
  if (M < 0 || k < 1 || n_rows < 0) return 0;
  return dwa::row_gradient_workspace_bytes(M, k, n_rows);
}

dwa_status dwa_row_gradient(const float* weights, const int32_t* gidx, int64_t M, int32_t k,
                            const void* a, int32_t a_is_bf16, int64_t lda, int64_t row_begin,
                            int64_t row_end, void* grad, int32_t grad_is_bf16, int64_t ldg,
                            int32_t d, void* workspace, size_t workspace_bytes,
                            dwa_stream_t stream) {
  const char* fn = "dwa_row_gradient";
  if (M < 0) return fail(DWA_ERR_INVALID_ARG, "%s: negative M", fn);
  if (M * static_cast<int64_t>(k) > INT32_MAX)
    return fail(DWA_ERR_UNSUPPORTED_SHAPE, "%s: M k above INT32_MAX", fn);
  dwa_status st = check_rows_args(fn, gidx, M, k, grad, row_begin, row_end, ldg, d, 8);
  if (st != DWA_OK) return st;
  if (row_end == row_begin) return ok();  // no owned rows: nothing to write
  if (M > 0) {
    if (!weights) return fail(DWA_ERR_INVALID_ARG, "%s: null weights", fn);
    st = check_vec_arg(fn, a, a_is_bf16, lda, d);
    if (st != DWA_OK) return st;
    const size_t need = dwa::row_gradient_workspace_bytes(M, k, row_end - row_begin);
    if (!workspace || workspace_bytes < need || !aligned(workspace, 256))
      return fail(DWA_ERR_WORKSPACE, "%s: workspace needs %zu bytes, 256-byte aligned (got %zu)",
                  fn, need, workspace_bytes);
  }
  cudaError_t e = dwa::launch_row_gradient(weights, gidx, M, k, a, a_is_bf16 ? 1 : 0, lda,
                                           row_begin, row_end, grad, grad_is_bf16 ? 1 : 0, ldg, d,
                                           workspace, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "dwa_row_gradient launch");
  return ok();
}

dwa_status dwa_gather_rows(const float* weights, const int32_t* gidx, int64_t M, int32_t k,
                           const void* rows, int64_t row_begin, int64_t row_end, int64_t ldr,
                           int32_t d, float* out, int32_t accumulate, dwa_stream_t stream) {
  if (M < 0) return fail(DWA_ERR_INVALID_ARG, "negative M");
  if (M == 0) return ok();
  if (!weights || !out) return fail(DWA_ERR_INVALID_ARG, "dwa_gather_rows: null pointer");
  if (!aligned(out, 16)) return fail(DWA_ERR_INVALID_ARG, "dwa_gather_rows: out not 16-byte aligned");
  dwa_status st = check_rows_args("dwa_gather_rows", gidx, M, k, rows, row_begin, row_end, ldr, d, 8);
  if (st != DWA_OK) return st;
  cudaError_t e = dwa::launch_gather_rows(weights, gidx, M, k, rows, row_begin, row_end, ldr, d,
                                          out, accumulate ? 1 : 0,
                                          static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "dwa_gather_rows launch");
  return ok();
}

dwa_status dwa_scatter_add_rows(const float* weights, const int32_t* gidx, int64_t M, int32_t k,
                                const void* a, int32_t a_is_bf16, int64_t lda, int64_t row_begin,
                                int64_t row_end, float* grad, int64_t ldg, int32_t d,
                                dwa_stream_t stream) {
  if (M < 0) return fail(DWA_ERR_INVALID_ARG, "negative M");
  if (M == 0) return ok();
  if (!weights) return fail(DWA_ERR_INVALID_ARG, "dwa_scatter_add_rows: null weights");
  dwa_status st =
      check_rows_args("dwa_scatter_add_rows", gidx, M, k, grad, row_begin, row_end, ldg, d, 4);
  if (st == DWA_OK) st = check_vec_arg("dwa_scatter_add_rows", a, a_is_bf16, lda, d);
  if (st != DWA_OK) return st;
  cudaError_t e = dwa::launch_scatter_add_rows(weights, gidx, M, k, a, a_is_bf16 ? 1 : 0, lda,
                                               row_begin, row_end, grad, ldg, d,
                                               static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "dwa_scatter_add_rows launch");
  return ok();
}

dwa_status dwa_pool_init_normal(void* out, int64_t rows, int64_t cols, int64_t ld,
                                int64_t row_offset, uint64_t seed, float stddev,
                                dwa_stream_t stream) {
  if (rows < 0 || cols < 0 || row_offset < 0)
    return fail(DWA_ERR_INVALID_ARG, "negative rows/cols/row_offset");
  if (rows == 0 || cols == 0) return ok();
  if (!out) return fail(DWA_ERR_INVALID_ARG, "null output");
  if (ld < cols) return fail(DWA_ERR_INVALID_ARG, "ld below cols");
  if (!aligned(out, 2)) return fail(DWA_ERR_INVALID_ARG, "output must be 2-byte aligned");
  if (!std::isfinite(stddev)) return fail(DWA_ERR_INVALID_ARG, "stddev must be finite");
  cudaError_t e = dwa::launch_pool_init_normal(out, rows, cols, ld, row_offset, seed, stddev,
                                               static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "dwa_pool_init_normal launch");
  return ok();
}

dwa_status dwa_weighted_gather_peers(const float* vals, const int32_t* gidx, int64_t M, int32_t k,
                                     const void* values, int64_t row_begin, int64_t row_end,
                                     int64_t ldv, int32_t d, void* const* inboxes, int32_t P,
                                     int32_t rank, int64_t block_rows, float* alpha_out,
                                     dwa_stream_t stream) {
  if (M < 0) return fail(DWA_ERR_INVALID_ARG, "dwa_weighted_gather_peers: negative M");
  if (M == 0) return ok();
  if (!vals || !gidx || !inboxes) return fail(DWA_ERR_INVALID_ARG, "dwa_weighted_gather_peers: null argument");
  if (P < 1 || P > DWA_MAX_PEERS || rank < 0 || rank >= P)
    return fail(DWA_ERR_INVALID_ARG, "dwa_weighted_gather_peers: P=%d rank=%d", P, rank);
  if (block_rows < 1 || block_rows * P < M)
    return fail(DWA_ERR_INVALID_ARG, "dwa_weighted_gather_peers: P * block_rows must cover M");
  if (k < 1 || k > DWA_MAX_K)
    return fail(k < 1 ? DWA_ERR_INVALID_ARG : DWA_ERR_UNSUPPORTED_SHAPE, "dwa_weighted_gather_peers: k=%d", k);
  if (d < 8 || d % 8 != 0)
    return fail(DWA_ERR_UNSUPPORTED_SHAPE, "dwa_weighted_gather_peers: d=%d must be a positive multiple of 8", d);
  if (row_begin < 0 || row_end < row_begin || row_end > INT32_MAX)
    return fail(DWA_ERR_INVALID_ARG, "dwa_weighted_gather_peers: bad owned row range");
  if (row_end > row_begin && (!values || ldv < d || ldv % 8 != 0 || !aligned(values, 16)))
    return fail(DWA_ERR_INVALID_ARG, "dwa_weighted_gather_peers: values need 16-byte aligned rows");
  float* boxes[DWA_MAX_PEERS];
  for (int p = 0; p < P; ++p) {
    if (!inboxes[p] || !aligned(inboxes[p], 16))
      return fail(DWA_ERR_INVALID_ARG, "dwa_weighted_gather_peers: bad inbox of rank %d", p);
    boxes[p] = static_cast<float*>(inboxes[p]);
  }
  cudaError_t e = dwa::launch_weighted_gather_peers(vals, gidx, M, k, values, row_begin, row_end, ldv,
                                                    d, boxes, P, rank, block_rows, alpha_out,
                                                    static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "dwa_weighted_gather_peers launch");
  return ok();
}

dwa_status dwa_reduce_broadcast_peers(const float* inbox, int32_t P, int32_t rank, int64_t block_rows,
                                      int64_t M, int32_t d, void* const* outs, const int32_t* flags,
                                      int32_t step, int64_t wait_ns, int32_t* status,
                                      dwa_stream_t stream) {
  if (!inbox || !outs || !flags || !status)
    return fail(DWA_ERR_INVALID_ARG, "dwa_reduce_broadcast_peers: null argument");
  if (P < 1 || P > DWA_MAX_PEERS || rank < 0 || rank >= P)
    return fail(DWA_ERR_INVALID_ARG, "dwa_reduce_broadcast_peers: P=%d rank=%d", P, rank);
  if (M < 0 || block_rows < 1 || block_rows * P < M)
    return fail(DWA_ERR_INVALID_ARG, "dwa_reduce_broadcast_peers: P * block_rows must cover M");
  if (d < 8 || d % 8 != 0 || !aligned(inbox, 16))
    return fail(DWA_ERR_UNSUPPORTED_SHAPE, "dwa_reduce_broadcast_peers: d %% 8 and 16-byte inbox required");
  float* o[DWA_MAX_PEERS];
  for (int p = 0; p < P; ++p) {
    if (!outs[p] || !aligned(outs[p], 16))
      return fail(DWA_ERR_INVALID_ARG, "dwa_reduce_broadcast_peers: bad output of rank %d", p);
    o[p] = static_cast<float*>(outs[p]);
  }
  cudaError_t e = dwa::launch_reduce_broadcast_peers(inbox, P, rank, block_rows, M, d, o, flags, step,
                                                     peer_wait_ns(wait_ns), status,
                                                     static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "dwa_reduce_broadcast_peers launch");
  return ok();
}

dwa_status dwa_peer_wait(const int32_t* flags, int32_t P, int32_t step, int64_t wait_ns,
                         int32_t* status, dwa_stream_t stream) {
  if (!flags || !status) return fail(DWA_ERR_INVALID_ARG, "dwa_peer_wait: null argument");
  if (P < 1 || P > DWA_MAX_PEERS) return fail(DWA_ERR_INVALID_ARG, "dwa_peer_wait: P=%d", P);
  cudaError_t e = dwa::launch_peer_wait(flags, P, step, peer_wait_ns(wait_ns), status,
                                        static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "dwa_peer_wait launch");
  return ok();
}

dwa_status dwa_project_keys(const void* vectors, int64_t N, int64_t ldv, int32_t D, const void* w_k,
                            int64_t ldw, int32_t S, int32_t d_k, const float* aspect_w,
                            void* keys_out, int64_t ldo, int32_t* status, dwa_stream_t stream) {
  return project_keys_impl("dwa_project_keys", vectors, N, ldv, D, w_k, ldw, S, d_k, aspect_w,
                           keys_out, ldo, status, stream, false);
}

dwa_status dwa_project_keys_packed(const void* vectors, int64_t N, int64_t ldv, int32_t D,
                                   const void* w_k, int64_t ldw, int32_t S, int32_t d_k,
                                   const float* aspect_w, void* keys_out, int64_t ldo,
                                   int32_t* status, dwa_stream_t stream) {
  return project_keys_impl("dwa_project_keys_packed", vectors, N, ldv, D, w_k, ldw, S, d_k,
                           aspect_w, keys_out, ldo, status, stream, true);
}

dwa_status dwa_peer_alloc(size_t bytes, void** out_ptr, void* out_handle) {
  if (!out_ptr || !out_handle || bytes == 0)
    return fail(DWA_ERR_INVALID_ARG, "dwa_peer_alloc: null output or zero size");
  static_assert(sizeof(cudaIpcMemHandle_t) == DWA_IPC_HANDLE_BYTES, "IPC handle size");
  void* p = nullptr;
  cudaError_t e = cudaMalloc(&p, bytes);
  if (e != cudaSuccess) return cuda_fail(e, "dwa_peer_alloc cudaMalloc");
  e = cudaMemset(p, 0, bytes);
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  if (e == cudaSuccess) e = cudaIpcGetMemHandle(static_cast<cudaIpcMemHandle_t*>(out_handle), p);
  if (e != cudaSuccess) {
    cudaFree(p);
    return cuda_fail(e, "dwa_peer_alloc");
  }
  *out_ptr = p;
  return ok();
}

dwa_status dwa_peer_open(const void* handle, void** out_ptr) {
  if (!handle || !out_ptr) return fail(DWA_ERR_INVALID_ARG, "dwa_peer_open: null argument");
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle, sizeof(h));
  cudaError_t e = cudaIpcOpenMemHandle(out_ptr, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) return cuda_fail(e, "dwa_peer_open cudaIpcOpenMemHandle");
  return ok();
}

dwa_status dwa_peer_close(void* ptr) {
  if (!ptr) return fail(DWA_ERR_INVALID_ARG, "dwa_peer_close: null pointer");
  cudaError_t e = cudaIpcCloseMemHandle(ptr);
  if (e != cudaSuccess) return cuda_fail(e, "dwa_peer_close");
  return ok();
}

dwa_status dwa_peer_free(void* ptr) {
  if (!ptr) return fail(DWA_ERR_INVALID_ARG, "dwa_peer_free: null pointer");
  cudaError_t e = cudaFree(ptr);
  if (e != cudaSuccess) return cuda_fail(e, "dwa_peer_free");
  return ok();
}

dwa_status dwa_peer_signal(void* const* flag_bases, int32_t P, int32_t my_rank, int32_t value,
                           dwa_stream_t stream) {
  if (!flag_bases) return fail(DWA_ERR_INVALID_ARG, "dwa_peer_signal: null flag table");
  if (P < 1 || P > DWA_MAX_PEERS || my_rank < 0 || my_rank >= P)
    return fail(DWA_ERR_INVALID_ARG, "dwa_peer_signal: P=%d / rank %d", P, my_rank);
  int32_t* bases[DWA_MAX_PEERS];
  for (int p = 0; p < P; ++p) {
    if (!flag_bases[p] || !aligned(flag_bases[p], 4))
      return fail(DWA_ERR_INVALID_ARG, "dwa_peer_signal: bad flag array of rank %d", p);
    bases[p] = static_cast<int32_t*>(flag_bases[p]);
  }
  cudaError_t e = dwa::launch_peer_signal(bases, P, my_rank, value, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "dwa_peer_signal launch");
  return ok();
}

dwa_status dwa_merge_topk_peers(const void* const* packed, int32_t P, int64_t M, int32_t k,
                                const int32_t* flags, int32_t step, int64_t wait_ns,
                                float* out_vals, int32_t* out_idx, int32_t* status,
                                dwa_stream_t stream) {
  if (M < 0) return fail(DWA_ERR_INVALID_ARG, "dwa_merge_topk_peers: negative M");
  if (M == 0) return ok();
  if (!packed || !flags || !out_vals || !out_idx || !status)
    return fail(DWA_ERR_INVALID_ARG, "dwa_merge_topk_peers: null argument");
  if (P < 1 || P > DWA_MAX_PEERS) return fail(DWA_ERR_INVALID_ARG, "dwa_merge_topk_peers: P=%d", P);
  if (k < 2 || k > DWA_MERGE_MAX_K || k % 2 != 0)
    return fail(DWA_ERR_UNSUPPORTED_SHAPE, "dwa_merge_topk_peers: k=%d must be even in [2, %d]", k,
                DWA_MERGE_MAX_K);
  if (M > (int64_t)INT32_MAX * 8) return fail(DWA_ERR_UNSUPPORTED_SHAPE, "dwa_merge_topk_peers: M too large");
  const int32_t* lists[DWA_MAX_PEERS];
  for (int p = 0; p < P; ++p) {
    if (!packed[p] || !aligned(packed[p], 16))
      return fail(DWA_ERR_INVALID_ARG, "dwa_merge_topk_peers: bad list pointer of rank %d", p);
    lists[p] = static_cast<const int32_t*>(packed[p]);
  }
  cudaError_t e = dwa::launch_merge_topk_peers(lists, P, M, k, flags, step, peer_wait_ns(wait_ns),
                                               out_vals, out_idx, status,
                                               static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "dwa_merge_topk_peers launch");
  return ok();
}

namespace {
// Argument checks shared by the two low-rank entry points; `fn` names the caller.
dwa_status check_lowrank_args(const char* fn, const void* h, int64_t ldh, const float* alpha,
                              const int32_t* gidx, int64_t M, int32_t k, const void* vectors,
                              int64_t row_begin, int64_t row_end, int64_t ldv, int32_t d_A,
                              int32_t d_B, int32_t r, const float* delta) {
  if (M < 0) return fail(DWA_ERR_INVALID_ARG, "%s: negative M", fn);
  if (!h || !alpha || !gidx || !delta)
    return fail(DWA_ERR_INVALID_ARG, "%s: null h/alpha/gidx/delta", fn);
  if (k < 1 || k > DWA_MAX_K)
    return fail(k < 1 ? DWA_ERR_INVALID_ARG : DWA_ERR_UNSUPPORTED_SHAPE,
                "%s: k=%d outside [1, %d]", fn, k, DWA_MAX_K);
  if (d_A < 8 || d_A % 8 != 0 || d_A > 8192 || d_B < 8 || d_B % 8 != 0)
    return fail(DWA_ERR_UNSUPPORTED_SHAPE,
                "%s: d_A=%d (multiple of 8, <= 8192) / d_B=%d (multiple of 8)", fn, d_A, d_B);
  if (r < 1 || r > 32) return fail(DWA_ERR_UNSUPPORTED_SHAPE, "%s: r=%d outside [1, 32]", fn, r);
  if (M > INT32_MAX) return fail(DWA_ERR_UNSUPPORTED_SHAPE, "%s: M too large", fn);
  if (ldh < d_A) return fail(DWA_ERR_INVALID_ARG, "%s: ldh below d_A", fn);
  if (row_begin < 0 || row_end < row_begin || row_end > INT32_MAX)
    return fail(DWA_ERR_INVALID_ARG, "%s: bad owned row range", fn);
  if (row_end > row_begin) {
    const int64_t need = static_cast<int64_t>(d_B) * r + static_cast<int64_t>(r) * d_A + d_B;
    if (!vectors) return fail(DWA_ERR_INVALID_ARG, "%s: null vectors", fn);
    if (ldv < need)
      return fail(DWA_ERR_INVALID_ARG, "%s: ldv=%lld below d_B r + r d_A + d_B = %lld", fn,
                  (long long)ldv, (long long)need);
    if (ldv % 8 != 0 || !aligned(vectors, 16))
      return fail(DWA_ERR_UNSUPPORTED_SHAPE,
                  "%s: vectors need 16-byte aligned rows (ldv %% 8 == 0)", fn);
  }
  return DWA_OK;
}
}  // namespace

dwa_status dwa_lowrank_delta(const void* h, int32_t h_is_bf16, int64_t ldh, const float* alpha,
                             const int32_t* gidx, int64_t M, int32_t k, const void* vectors,
                             int64_t row_begin, int64_t row_end, int64_t ldv, int32_t d_A,
                             int32_t d_B, int32_t r, float* delta, dwa_stream_t stream) {
  if (M == 0) return ok();
  const dwa_status st = check_lowrank_args("dwa_lowrank_delta", h, ldh, alpha, gidx, M, k, vectors,
                                           row_begin, row_end, ldv, d_A, d_B, r, delta);
  if (st != DWA_OK) return st;
  cudaError_t e = dwa::launch_lowrank_delta(h, h_is_bf16 ? 1 : 0, ldh, alpha, gidx, M, k, vectors,
                                            row_begin, row_end, ldv, d_A, d_B, r, delta,
                                            static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "dwa_lowrank_delta launch");
  return ok();
}

size_t dwa_lowrank_delta_rows_workspace(int64_t M, int32_t k, int64_t n_rows, int32_t d_B) {
  if (M < 0 || k < 1 || n_rows < 0 || d_B < 1) return 0;
  return dwa::lowrank_rows_workspace_bytes(M, k, n_rows, d_B);
}

dwa_status dwa_lowrank_delta_rows(const void* h, int32_t h_is_bf16, int64_t ldh,
                                  const float* alpha, const int32_t* gidx, int64_t M, int32_t k,
                                  const void* vectors, int64_t row_begin, int64_t row_end,
                                  int64_t ldv, int32_t d_A, int32_t d_B, int32_t r, float* delta,
                                  void* workspace, size_t workspace_bytes, dwa_stream_t stream) {
  const char* fn = "dwa_lowrank_delta_rows";
  if (M == 0) return ok();
  const dwa_status st = check_lowrank_args(fn, h, ldh, alpha, gidx, M, k, vectors, row_begin,
                                           row_end, ldv, d_A, d_B, r, delta);
  if (st != DWA_OK) return st;
  if (M * static_cast<int64_t>(k) > INT32_MAX)
    return fail(DWA_ERR_UNSUPPORTED_SHAPE, "%s: M k above INT32_MAX", fn);
  if (dwa::lowrank_rows_smem_bytes(d_A, d_B, r) > 200 * 1024)
    return fail(DWA_ERR_UNSUPPORTED_SHAPE,
                "%s: a row's U | V | b (%d bytes) exceeds 200 KB of shared memory", fn,
                dwa::lowrank_rows_smem_bytes(d_A, d_B, r));
  if (!aligned(h, 16) || ldh % (h_is_bf16 ? 8 : 4) != 0)
    return fail(DWA_ERR_UNSUPPORTED_SHAPE, "%s: h rows must be 16-byte aligned", fn);
  if (!aligned(delta, 16)) return fail(DWA_ERR_UNSUPPORTED_SHAPE, "%s: delta not 16-byte aligned", fn);
  const size_t need = dwa::lowrank_rows_workspace_bytes(M, k, row_end - row_begin, d_B);
  if (!workspace || workspace_bytes < need || !aligned(workspace, 256))
    return fail(DWA_ERR_WORKSPACE, "%s: workspace needs %zu bytes, 256-byte aligned (got %zu)", fn,
                need, workspace_bytes);
  cudaError_t e = dwa::launch_lowrank_rows(h, h_is_bf16 ? 1 : 0, ldh, alpha, gidx, M, k, vectors,
                                           row_begin, row_end, ldv, d_A, d_B, r, delta, workspace,
                                           static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "dwa_lowrank_delta_rows launch");
  return ok();
}

dwa_status dwa_assemble_finish(const void* residual, int32_t residual_is_bf16, int64_t ldr,
                               const float* base, const float* delta, int64_t M, int32_t d_B,
                               float gamma, const float* ln_scale, const float* ln_bias, float eps,
                               float* out, dwa_stream_t stream) {
  if (M < 0) return fail(DWA_ERR_INVALID_ARG, "dwa_assemble_finish: negative M");
  if (M == 0) return ok();
  if (!delta || !out) return fail(DWA_ERR_INVALID_ARG, "dwa_assemble_finish: null delta/out");
  if (d_B < 1) return fail(DWA_ERR_INVALID_ARG, "dwa_assemble_finish: d_B=%d", d_B);
  if (residual && ldr < d_B) return fail(DWA_ERR_INVALID_ARG, "dwa_assemble_finish: ldr below d_B");
  if (!(eps >= 0.0f) || !std::isfinite(gamma))
    return fail(DWA_ERR_INVALID_ARG, "dwa_assemble_finish: eps must be >= 0 and gamma finite");
  if (M > (int64_t)INT32_MAX * 8) return fail(DWA_ERR_UNSUPPORTED_SHAPE, "dwa_assemble_finish: M too large");
  cudaError_t e = dwa::launch_assemble_finish(residual, residual_is_bf16 ? 1 : 0, ldr, base, delta,
                                              M, d_B, gamma, ln_scale, ln_bias, eps, out,
                                              static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "dwa_assemble_finish launch");
  return ok();
}

dwa_status dwa_usage_ema(const float* alpha, const int32_t* gidx, int64_t n, int64_t row_begin,
                         int64_t row_end, float weight, float beta, float* ema,
                         dwa_stream_t stream) {
  if (n < 0) return fail(DWA_ERR_INVALID_ARG, "dwa_usage_ema: negative n");
  if (row_begin < 0 || row_end < row_begin || row_end > INT32_MAX)
    return fail(DWA_ERR_INVALID_ARG, "dwa_usage_ema: bad owned row range");
  if (n > 0 && (!alpha || !gidx)) return fail(DWA_ERR_INVALID_ARG, "dwa_usage_ema: null alpha/gidx");
  if (row_end > row_begin && !ema) return fail(DWA_ERR_INVALID_ARG, "dwa_usage_ema: null ema");
  if (!std::isfinite(weight) || !std::isfinite(beta))
    return fail(DWA_ERR_INVALID_ARG, "dwa_usage_ema: weight and beta must be finite");
  if (n > (int64_t)INT32_MAX * 256 || row_end - row_begin > (int64_t)INT32_MAX * 256)
    return fail(DWA_ERR_UNSUPPORTED_SHAPE, "dwa_usage_ema: too many entries");
  cudaError_t e = dwa::launch_usage_ema(alpha, gidx, n, row_begin, row_end, weight, beta, ema,
                                        static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "dwa_usage_ema launch");
  return ok();
}

dwa_status dwa_workspace_status(const void* ws, dwa_stream_t stream, int32_t* out_status) {
  if (!ws || !out_status) return fail(DWA_ERR_INVALID_ARG, "null workspace or output");
  int32_t v = 0;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  cudaError_t e = cudaMemcpyAsync(&v, ws, sizeof(v), cudaMemcpyDeviceToHost, s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  if (e != cudaSuccess) return cuda_fail(e, "dwa_workspace_status");
  *out_status = v;
  return ok();
}

dwa_status dwa_lm_rope_qk(const void* qkv, int64_t B, int64_t S, int32_t H, int32_t dh,
                          int64_t ld_qkv, const void* cos_t, const void* sin_t, int64_t ld_cs,
                          void* q_out, void* k_out, dwa_stream_t stream) {
  if (B < 0 || S < 0 || H < 1 || dh < 8)
    return fail(DWA_ERR_INVALID_ARG, "dwa_lm_rope_qk: bad sizes (B=%lld, S=%lld, H=%d, dh=%d)",
                (long long)B, (long long)S, H, dh);
  if (B == 0 || S == 0) return ok();
  if (!qkv || !cos_t || !sin_t || !q_out || !k_out)
    return fail(DWA_ERR_INVALID_ARG, "dwa_lm_rope_qk: null pointer");
  if (dh % 8 != 0) return fail(DWA_ERR_UNSUPPORTED_SHAPE, "dwa_lm_rope_qk: dh=%d must be a multiple of 8", dh);
  if (ld_qkv < 2ll * H * dh || ld_cs < dh / 2)
    return fail(DWA_ERR_INVALID_ARG, "dwa_lm_rope_qk: a row stride is below its row length");
  if (ld_qkv % 8 != 0 || ld_cs % 4 != 0 || !aligned(qkv, 16) || !aligned(q_out, 16) ||
      !aligned(k_out, 16) || !aligned(cos_t, 8) || !aligned(sin_t, 8))
    return fail(DWA_ERR_UNSUPPORTED_SHAPE, "dwa_lm_rope_qk: alignment (ld_qkv %% 8, ld_cs %% 4, "
                "16-byte qkv / outputs, 8-byte cos / sin)");
  if (2 * B * S * H * (dh / 8) > INT32_MAX * 256ll)
    return fail(DWA_ERR_UNSUPPORTED_SHAPE, "dwa_lm_rope_qk: too many elements");
  cudaError_t e = dwa::launch_rope_qk(qkv, B, S, H, dh, ld_qkv, cos_t, sin_t, ld_cs, q_out, k_out,
                                      static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "dwa_lm_rope_qk launch");
  return ok();
}

dwa_status dwa_lm_aspect_queries(const void* q, int64_t M, int32_t S, int32_t d_k, int64_t ldq,
                                 const float* aspect_logits, const float* tau_param,
                                 float lambda_sharp, float T, int32_t use_sigmoid, void* out,
                                 int64_t ldo, float* w_out, float* params_out,
                                 dwa_stream_t stream) {
  if (M < 0) return fail(DWA_ERR_INVALID_ARG, "dwa_lm_aspect_queries: negative M");
  if (S < 1 || S > dwa::lm_max_aspects())
    return fail(DWA_ERR_UNSUPPORTED_SHAPE, "dwa_lm_aspect_queries: S=%d outside [1, %d]", S,
                dwa::lm_max_aspects());
  if (d_k < 8 || d_k % 8 != 0)
    return fail(DWA_ERR_UNSUPPORTED_SHAPE, "dwa_lm_aspect_queries: d_k=%d must be a positive "
                "multiple of 8", d_k);
  if (!aspect_logits || (use_sigmoid && !tau_param))
    return fail(DWA_ERR_INVALID_ARG, "dwa_lm_aspect_queries: null aspect_logits / tau_param");
  if (M > 0 && (!q || !out)) return fail(DWA_ERR_INVALID_ARG, "dwa_lm_aspect_queries: null q / out");
  if (ldq < static_cast<int64_t>(S) * d_k || ldo < static_cast<int64_t>(S) * d_k)
    return fail(DWA_ERR_INVALID_ARG, "dwa_lm_aspect_queries: a row stride is below S d_k");
  if (ldq % 8 != 0 || ldo % 8 != 0 || (M > 0 && (!aligned(q, 16) || !aligned(out, 16))))
    return fail(DWA_ERR_UNSUPPORTED_SHAPE, "dwa_lm_aspect_queries: 16-byte aligned rows required");
  if (!aligned(aspect_logits, 4) || (tau_param && !aligned(tau_param, 4)) ||
      (w_out && !aligned(w_out, 4)) || (params_out && !aligned(params_out, 4)))
    return fail(DWA_ERR_INVALID_ARG, "dwa_lm_aspect_queries: f32 arrays must be 4-byte aligned");
  if (M * S > INT32_MAX * 256ll)
    return fail(DWA_ERR_UNSUPPORTED_SHAPE, "dwa_lm_aspect_queries: too many rows");
  cudaError_t e = dwa::launch_aspect_queries(q, M, S, d_k, ldq, aspect_logits, tau_param,
                                             lambda_sharp, T, use_sigmoid ? 1 : 0, out, ldo, w_out,
                                             params_out, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "dwa_lm_aspect_queries launch");
  return ok();
}

}  // extern "C"
