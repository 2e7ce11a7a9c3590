/*
 * dwa_lm.h — fused elementwise steps of this library's DWA language model
 * block (the retrieval path's call site: src/model/dwa.py:77-130 and
 * src/model/parts.py:17-83 of the reference).  Not part of the retrieval FFI
 * of dwa_retrieval.h; the same conventions: stream-ordered and asynchronous,
 * arguments validated on the host (non-zero status, nothing launched, when
 * invalid), no allocation, bf16 buffers as uint16 bit patterns.
 */
#ifndef DWA_LM_H_
#define DWA_LM_H_

#include "dwa_retrieval.h"

#ifdef __cplusplus
extern "C" {
#endif

/*
 * Rotary embedding of the attention's queries and keys (parts.py:17-25):
 * for x = the q (columns [0, H dh)) or k (columns [H dh, 2 H dh)) part of
 * row (b, s) of the QKV projection qkv (bf16 [B S, ld_qkv]) and each head,
 * x1 = x[0::2], x2 = x[1::2] (dh / 2 each),
 *   out[b, s, h, 0:dh/2]  = x1 cos[s] - x2 sin[s]
 *   out[b, s, h, dh/2:dh] = x1 sin[s] + x2 cos[s]
 * with every product, sum and difference rounded to bf16 (bit-identical to
 * the same steps as elementwise bf16 tensor operations).  cos / sin: bf16
 * [S, ld_cs] (first dh / 2 columns used); q_out / k_out: bf16 [B, S, H, dh]
 * contiguous (token-major, as the rows of qkv).  dh % 8 == 0; ld_qkv % 8 == 0, ld_cs % 4 == 0; qkv, q_out,
 * k_out 16-byte aligned, cos / sin 8-byte aligned.
 */
DWA_API dwa_status dwa_lm_rope_qk(const void* qkv, int64_t B, int64_t S, int32_t H, int32_t dh,
                                  int64_t ld_qkv, const void* cos_t, const void* sin_t,
                                  int64_t ld_cs, void* q_out, void* k_out, dwa_stream_t stream);

/*
 * Packed aspect queries of the hybrid score (retrieval.py:159-168):
 * w = softmax(aspect_logits) (f32 [S]) and, for every row m and aspect s,
 *   out[m, s d_k + j] = q[m, s d_k + j] sqrt(w_s) / (|q[m, s d_k : (s+1) d_k]| + 1e-8)
 * computed in f32 from the bf16 q (bf16 [M, ldq]) and stored as bf16
 * (out [M, ldo]).  w_out (f32 [S]) and params_out (f32 [3]: lambda_sharp,
 * tau = w . tau_param when use_sigmoid else 0, T: the device scalars of
 * dwa_score_topk_dev) may be NULL; tau_param (f32 [S]) may be NULL when
 * use_sigmoid is 0.  1 <= S <= 64, d_k % 8 == 0, ldq and ldo multiples of 8
 * and >= S d_k, q / out 16-byte aligned.
 */
DWA_API dwa_status dwa_lm_aspect_queries(const void* q, int64_t M, int32_t S, int32_t d_k,
                                         int64_t ldq, const float* aspect_logits,
                                         const float* tau_param, float lambda_sharp, float T,
                                         int32_t use_sigmoid, void* out, int64_t ldo,
                                         float* w_out, float* params_out, dwa_stream_t stream);

#ifdef __cplusplus
}  /* extern "C" */
#endif

#endif /* DWA_LM_H_ */
