/*
 * dwa_retrieval.h — C ABI of the B200 (sm_100a) DWA retrieval hot path.
 *
 * The reference (computd, JAX) runs this path as:
 *   src/kernels/tiled_topk.py:160-176  tiled_topk_fallback: s = q.k^T, gate/exp, lax.top_k
 *   src/kernels/tiled_topk.py:86-153   tiled_topk_fused (same contract, Pallas/TPU, uncalled)
 *   src/model/retrieval.py:285-303     _chip_topk: global index offset, all_gather, merge top_k
 *   src/model/retrieval.py:324-326     alpha = v / (sum(v) + 1e-8)
 *   src/model/assembly.py:104,123-128  vectors[idx] gather and the alpha-weighted sum
 *
 * Every entry point is stream-ordered and asynchronous: it validates its
 * arguments on the host, returns a non-zero status WITHOUT launching anything
 * when they are invalid, and otherwise enqueues kernels on `stream`.
 * The library never allocates device memory: buffers and workspace belong to
 * the caller.  All device pointers are plain CUDA device addresses.
 *
 * Element types: "bf16" buffers hold IEEE bfloat16 (uint16 bit patterns);
 * scores and outputs are fp32; indices are int32.
 */
#ifndef DWA_RETRIEVAL_H_
#define DWA_RETRIEVAL_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(__GNUC__)
#define DWA_API __attribute__((visibility("default")))
#else
#define DWA_API
#endif

/* Opaque CUDA stream handle (cudaStream_t / CUstream). NULL = legacy default stream. */
typedef void* dwa_stream_t;

typedef int32_t dwa_status;
enum {
  DWA_OK = 0,
  DWA_ERR_INVALID_ARG = 1,       /* null pointer, negative size, k > N, misaligned buffer   */
  DWA_ERR_UNSUPPORTED_SHAPE = 2, /* k > DWA_MAX_K, d % 8 != 0, lambda < 0, T <= 0, ...       */
  DWA_ERR_CUDA = 3,              /* a CUDA runtime/driver call failed (message has details) */
  DWA_ERR_TIMEOUT = 4,           /* a bounded device-side wait gave up (kernel returned)    */
  DWA_ERR_DEVICE_CHECK = 5,      /* a device-side argument check failed                     */
  DWA_ERR_WORKSPACE = 6          /* workspace pointer null/misaligned or too small          */
};

/* Largest top-k the fused score kernel keeps per query (its per-row heap
 * lives in shared memory: 128 rows x k x 8 bytes). */
#define DWA_MAX_K 128
#define DWA_ABI_VERSION 2

DWA_API int32_t dwa_abi_version(void);

/* Human-readable name of a status code (static storage). */
DWA_API const char* dwa_status_string(dwa_status s);

/* Detail of the last failing call on this host thread (thread-local storage). */
DWA_API const char* dwa_last_error(void);

/* Bytes of device workspace dwa_score_topk needs for this shape on the current
 * device (0 when the shape is invalid). */
DWA_API size_t dwa_score_topk_workspace(int64_t M, int64_t N_local, int32_t d, int32_t k);

/*
 * Fused score GEMM + streaming top-k over one pool shard.
 * Replaces tiled_topk_fallback / tiled_topk_fused (src/kernels/tiled_topk.py:160-176,
 * :86-153) plus the per-chip global offset of _chip_topk (src/model/retrieval.py:292-293).
 *
 *   s[m, n]  = sum_d q[m, d] * keys[n, d]        (bf16 x bf16, fp32 accumulate, tcgen05)
 *   v(s)     = sigmoid(lambda_sharp * (s - tau)) * exp(s / T)   if use_sigmoid
 *            = exp(s / T)                                       otherwise
 *   out_vals[m, j], out_idx[m, j] = top-k of v over n, sorted by v descending,
 *            equal v ordered by lower index first (the lax.top_k contract);
 *            out_idx = n + idx_offset (int32 global pool row).
 *
 * v is strictly increasing in s for lambda_sharp >= 0 and T > 0, so selection
 * runs on s and v is evaluated for the k survivors only; other parameters
 * return DWA_ERR_UNSUPPORTED_SHAPE.  The [M, N_local] score matrix never
 * reaches device memory.
 *
 * q: bf16 [M, ldq] (row stride ldq elements), keys: bf16 [N_local, ldk].
 * Requirements: d % 8 == 0, ldq % 8 == 0, ldk % 8 == 0, 16-byte aligned bases,
 * 1 <= k <= min(DWA_MAX_K, N_local), N_local + idx_offset <= INT32_MAX.
 * out_vals f32 [M, k], out_idx i32 [M, k] (dense row-major).
 * ws: >= dwa_score_topk_workspace(M, N_local, d, k) bytes, 256-byte aligned.
 */
DWA_API dwa_status dwa_score_topk(const void* q, int64_t M, int64_t ldq,
                          const void* keys, int64_t N_local, int64_t ldk,
                          int32_t d, int32_t k,
                          float lambda_sharp, float tau, float T, int32_t use_sigmoid,
                          int64_t idx_offset,
                          float* out_vals, int32_t* out_idx,
                          void* ws, size_t ws_bytes, dwa_stream_t stream);

/*
 * dwa_score_topk without a caller workspace, for callers that cannot allocate
 * device memory (e.g. a plugin inside a framework whose allocator already owns
 * most of the GPU, or a binding with no scratch-buffer argument).  No
 * counterpart in the reference (its JAX path lets XLA allocate everything).
 *
 * Same arguments, validation, kernels and results as dwa_score_topk; the
 * workspace is a 128 MiB scratch array built into the library, held in device
 * memory by every GPU this entry point runs on until the process exits.
 * Shapes needing more than that return DWA_ERR_UNSUPPORTED_SHAPE (nothing
 * launched).  The first call on a device looks up the scratch address with
 * that device current; make it before any stream capture (a lookup that
 * fails is retried by the next call).  The scratch used is the current
 * device's, so `stream` must belong to the current device (otherwise
 * DWA_ERR_INVALID_ARG).  Every call on a device shares the scratch: calls
 * must be stream-ordered, overlapping calls race.  Allocates nothing.
 */
DWA_API dwa_status dwa_score_topk_noalloc(const void* q, int64_t M, int64_t ldq,
                          const void* keys, int64_t N_local, int64_t ldk,
                          int32_t d, int32_t k,
                          float lambda_sharp, float tau, float T, int32_t use_sigmoid,
                          int64_t idx_offset,
                          float* out_vals, int32_t* out_idx, dwa_stream_t stream);

/*
 * dwa_score_topk with lambda_sharp, tau and T read by the kernels from device
 * memory: params points at three device floats {lambda_sharp, tau, T}.  The
 * reference passes these as (1,)-shaped f32 operands so a learned tau never
 * forces a recompile or a host read (src/kernels/tiled_topk.py:26-29,
 * 112-115); with this form a caller whose scalars live on the device (an XLA
 * FFI handler, a training step computing tau = w . tau_s) enqueues the call
 * without waiting for the host.  Same shapes, workspace and results as
 * dwa_score_topk.  The checks dwa_score_topk makes on the host scalars
 * (T > 0, finite lambda_sharp >= 0 and tau with the gate) run on the device:
 * values that fail them give NaN scores and -1 indices and record
 * DWA_ERR_DEVICE_CHECK in the workspace status word (dwa_workspace_status).
 */
DWA_API dwa_status dwa_score_topk_dev(const void* q, int64_t M, int64_t ldq,
                          const void* keys, int64_t N_local, int64_t ldk,
                          int32_t d, int32_t k, const float* params, int32_t use_sigmoid,
                          int64_t idx_offset, float* out_vals, int32_t* out_idx,
                          void* ws, size_t ws_bytes, dwa_stream_t stream);

/*
 * dwa_score_topk_dev plus, from the same score tiles, the per-sequence mean of
 * the fused scores: the queries are `M / seq` sequences of `seq` consecutive
 * rows, and
 *   fused_mean[b, n] = (1 / seq) sum_{t < seq} v(s[b * seq + t, n])
 * for every key n of the shard (f32 [M / seq, ld_mean], overwritten).  This is
 * hybrid_forward's alpha_raw.mean(axis=1) (src/model/retrieval.py:176-181),
 * which needs every per-position score and so cannot come from the top-k or
 * from a mean query; computing it in the score kernel's epilogue keeps the
 * [M, N] score matrix out of HBM.  seq must divide M; ld_mean >= N_local.
 * The sums use f32 atomics, so their order (and the last bits) may vary from
 * call to call.  Other arguments, workspace and results as dwa_score_topk_dev.
 */
DWA_API dwa_status dwa_score_topk_seqmean(const void* q, int64_t M, int64_t ldq,
                          const void* keys, int64_t N_local, int64_t ldk,
                          int32_t d, int32_t k, const float* params, int32_t use_sigmoid,
                          int64_t idx_offset, int64_t seq, float* fused_mean, int64_t ld_mean,
                          float* out_vals, int32_t* out_idx,
                          void* ws, size_t ws_bytes, dwa_stream_t stream);

/*
 * Sequence-mean auxiliary scores of the retrieval (src/model/retrieval.py:
 * 332-341): for a few query rows q (f32 [B, ldq]; the per-sequence mean
 * queries q_mean_w) against every key of the shard (bf16 [N, ldk]):
 *   sims[b, n]  = <q[b, :d], keys[n, :d]>        (f32 x bf16, fp32 accumulate)
 *   fused[b, n] = sigmoid(lambda_sharp (sims - tau)) * exp(sims / T)   if use_sigmoid
 *               = exp(sims / T)                                        otherwise
 * sims f32 [B, lds], fused f32 [B, ldf] (may be NULL; then params may be
 * NULL too); params: device {lambda_sharp, tau, T}.  HBM-bound: the keys are
 * read once (tensor cores) for B <= 10 when the split query operand fits in
 * shared memory (3 B rounded up to 16 rows x d bf16, about d <= 5100 at
 * B <= 5), otherwise once per 8 query rows.  d % 8 == 0 and d <= 12800, keys 16-byte
 * aligned, ldk % 8 == 0.  status (device int32, may be NULL) receives
 * DWA_ERR_DEVICE_CHECK when the params fail the checks of dwa_score_topk_dev
 * (fused is then NaN).
 */
DWA_API dwa_status dwa_seq_scores(const float* q, int64_t B, int64_t ldq,
                          const void* keys, int64_t N, int64_t ldk, int32_t d,
                          const float* params, int32_t use_sigmoid,
                          float* sims, int64_t lds, float* fused, int64_t ldf,
                          int32_t* status, dwa_stream_t stream);

/*
 * Merge P per-shard candidate lists into the global top-k.
 * Replaces the all_gather transpose/reshape + second top_k + take of
 * _chip_topk (src/model/retrieval.py:295-302).
 *
 * cand_vals f32 / cand_idx i32: [P, M, k] (the all-gather output, list p from
 * shard p).  Output: the k best of the P*k candidates per row, by v descending
 * and lower global index first among equal v.  out_* are [M, k]; they must not
 * alias the inputs.
 */
DWA_API dwa_status dwa_merge_topk(const float* cand_vals, const int32_t* cand_idx,
                          int32_t P, int64_t M, int32_t k,
                          float* out_vals, int32_t* out_idx, dwa_stream_t stream);

/*
 * dwa_merge_topk over candidates at arbitrary element strides: candidate
 * (list l, position p, row r) is cand_vals[l*stride_list + p*stride_pos +
 * r*stride_row] (and likewise cand_idx).  Lets scores and indices travel in
 * one interleaved int32 buffer [P, M, k, 2] — one all-gather instead of two —
 * with cand_idx = cand_vals + 1 element.  Same merge, lists sorted best
 * first, P <= 128.  Replaces the same reference lines as dwa_merge_topk
 * (src/model/retrieval.py:295-302).
 */
DWA_API dwa_status dwa_merge_topk_strided(const float* cand_vals, const int32_t* cand_idx,
                          int32_t P, int64_t M, int32_t k,
                          int64_t stride_list, int64_t stride_pos, int64_t stride_row,
                          float* out_vals, int32_t* out_idx, dwa_stream_t stream);

/*
 * Alpha normalisation + gathered-value weighted sum (owner-computes form).
 * Replaces retrieval.py:326 (alpha = v / (sum v + 1e-8)) and the gather +
 * alpha-weighted sum of WeightAssembler (src/model/assembly.py:104,127):
 *
 *   alpha[m, j] = vals[m, j] / (sum_j vals[m, j] + 1e-8)
 *   out[m, :]   = sum_{j : row_begin <= gidx[m,j] < row_end} alpha[m, j] * values[gidx[m,j] - row_begin, :]
 *
 * values: bf16 rows [row_end - row_begin, ldv] holding global pool rows
 * [row_begin, row_end) (the caller's shard; the whole pool on one GPU).
 * out f32 [M, d] is overwritten (rows owned elsewhere contribute zero, so the
 * partial sums of all shards add up to the full result).  alpha_out f32 [M, k]
 * may be NULL.  With an empty row range (row_begin == row_end) `out` may be
 * NULL and only alpha is computed.  Requirements: d % 8 == 0, ldv % 8 == 0,
 * 16-byte aligned values.
 */
DWA_API dwa_status dwa_weighted_gather(const float* vals, const int32_t* gidx,
                               int64_t M, int32_t k,
                               const void* values, int64_t row_begin, int64_t row_end,
                               int64_t ldv, int32_t d,
                               float* out, float* alpha_out, dwa_stream_t stream);

/* ------------------------------------------------------------------------
 * Backward of the path with the selected indices fixed (the reference trains
 * through the plain-jnp path because its Pallas kernel has no VJP,
 * src/model/retrieval.py:268-271).  With out = sum_j alpha_j V[idx_j],
 * alpha = v / (sum v + 1e-8), v = gate(s) exp(s / T), s_j = <q, K[idx_j]>:
 *   dalpha = dwa_gather_dot(dout, V, idx)        s = dwa_gather_dot(q, K, idx)
 *   ds, dparams = dwa_score_backward(v, s, dalpha)
 *   dq = dwa_gather_rows(ds, idx, K)
 *   dV += dwa_scatter_add_rows(alpha, idx, dout), dK += dwa_scatter_add_rows(ds, idx, q)
 * All four work on an owned pool row range [row_begin, row_end) (rows of
 * `rows`/`grad` are global rows row_begin..): on a sharded pool each rank's
 * partial dalpha / s / dq are summed across ranks, and each rank updates only
 * its own rows.  Row vectors `a` are f32 (a_is_bf16 = 0) or bf16; d % 8 == 0;
 * 16-byte aligned bases, row strides multiples of 8 elements.
 * ------------------------------------------------------------------------ */

/* out[m, j] = <a[m, :], rows[gidx[m, j] - row_begin, :]> (0 for rows owned elsewhere). */
DWA_API dwa_status dwa_gather_dot(const void* a, int32_t a_is_bf16, int64_t lda,
                          const int32_t* gidx, int64_t M, int32_t k,
                          const void* rows, int64_t row_begin, int64_t row_end, int64_t ldr,
                          int32_t d, float* out, dwa_stream_t stream);

/* dscores[m, j] from fused scores v, raw scores s and dalpha; dparams (3
 * floats: dlambda, dtau, dT) is accumulated into (atomically) and may be NULL. */
DWA_API dwa_status dwa_score_backward(const float* vals, const float* scores, const float* dalpha,
                          int64_t M, int32_t k,
                          float lambda_sharp, float tau, float T, int32_t use_sigmoid,
                          float* dscores, float* dparams, dwa_stream_t stream);

/* dwa_score_backward with {lambda_sharp, tau, T} read from the device array
 * params (see dwa_score_topk_dev).  A non-positive or non-finite T, or a
 * non-finite lambda_sharp / tau with the gate on, gives NaN dscores and
 * records DWA_ERR_DEVICE_CHECK in *status (device int32, may be NULL). */
DWA_API dwa_status dwa_score_backward_dev(const float* vals, const float* scores, const float* dalpha,
                          int64_t M, int32_t k, const float* params, int32_t use_sigmoid,
                          float* dscores, float* dparams, int32_t* status, dwa_stream_t stream);

/*
 * The queries-side backward in one launch, for a pool held whole by this GPU
 * (every gidx inside [row_begin, row_end); on a row-sharded pool the partial
 * dot products must be summed across ranks first, so use dwa_gather_dot +
 * dwa_score_backward + dwa_gather_rows there).  Per query m:
 *   s_j = <q[m], keys[gidx_j]>, dalpha_j = <dout[m], values[gidx_j]>,
 *   dscores as dwa_score_backward, dq[m] = sum_j dscores_j keys[gidx_j],
 * each selected key and value row read from HBM once.  Results equal the
 * four-kernel path (same sums in the same order).  q bf16 (q_is_bf16 = 1) or
 * f32; dout f32 [M, ld_dout]; keys / values bf16 rows; vals f32 [M, k] (the
 * forward's fused scores); gidx i32 [M, k]; k <= 128.  dscores f32 [M, k],
 * dq f32 [M, d_k] (16-byte aligned) are written; dparams (3 floats) is
 * accumulated into and may be NULL.  params: NULL (host lambda_sharp / tau /
 * T) or three device floats, checked on the device as in
 * dwa_score_backward_dev (then status, a device int32, may not be NULL).
 * d_k, d_v, ldk, ldv multiples of 8; all row pointers 16-byte aligned.
 */
DWA_API dwa_status dwa_retrieval_backward(const void* q, int32_t q_is_bf16, int64_t ldq,
                          const float* dout, int64_t ld_dout, const void* keys, int64_t ldk,
                          int32_t d_k, const void* values, int64_t ldv, int32_t d_v,
                          const float* vals, const int32_t* gidx, int64_t M, int32_t k,
                          int64_t row_begin, int64_t row_end, float lambda_sharp, float tau,
                          float T, const float* params, int32_t use_sigmoid, float* dscores,
                          float* dq, float* dparams, int32_t* status, dwa_stream_t stream);

/*
 * The dense gradient of the owned pool rows in one write, from the selections:
 *   grad[r, :] = sum over (m, j) with gidx[m, j] == row_begin + r of w[m, j] a[m, :]
 * for every owned row r (zero where no entry selected it), summed in f32 and
 * stored as bf16 (grad_is_bf16 = 1) or f32.  The same values as zero-filling
 * an f32 gradient, dwa_scatter_add_rows into it and converting, without the
 * zero fill, the float atomics or the conversion pass: the (m, j) entries are
 * sorted by row first (a counting sort in the workspace), then one warp per
 * row sums its entries (in an order the sort leaves unspecified, as the
 * atomics do).  w f32 [M, k]; a: [M, lda] bf16 or f32 rows; grad [row_end -
 * row_begin, ldg]; d, lda, ldg multiples of 8; 16-byte aligned rows.
 * workspace: >= dwa_row_gradient_workspace(M, k, row_end - row_begin) bytes,
 * 256-byte aligned.  M k <= INT32_MAX.
 */
DWA_API size_t dwa_row_gradient_workspace(int64_t M, int32_t k, int64_t n_rows);
DWA_API dwa_status dwa_row_gradient(const float* weights, const int32_t* gidx, int64_t M,
                                    int32_t k, const void* a, int32_t a_is_bf16, int64_t lda,
                                    int64_t row_begin, int64_t row_end, void* grad,
                                    int32_t grad_is_bf16, int64_t ldg, int32_t d, void* workspace,
                                    size_t workspace_bytes, dwa_stream_t stream);

/* out[m, :] (= or +=) sum_j w[m, j] rows[gidx[m, j] - row_begin, :] over owned rows. */
DWA_API dwa_status dwa_gather_rows(const float* weights, const int32_t* gidx, int64_t M, int32_t k,
                          const void* rows, int64_t row_begin, int64_t row_end, int64_t ldr,
                          int32_t d, float* out, int32_t accumulate, dwa_stream_t stream);

/* grad[gidx[m, j] - row_begin, :] += w[m, j] * a[m, :] over owned rows (f32 atomics). */
DWA_API dwa_status dwa_scatter_add_rows(const float* weights, const int32_t* gidx,
                          int64_t M, int32_t k, const void* a, int32_t a_is_bf16, int64_t lda,
                          int64_t row_begin, int64_t row_end, float* grad, int64_t ldg,
                          int32_t d, dwa_stream_t stream);

/*
 * Deterministic pool / query initialisation: element (r, c) of a logical
 * [rows_total, cols] matrix is  stddev * N(0,1)  drawn from Philox4x32-10
 * keyed by (seed, row_offset + r, c), rounded to bf16.  A shard
 * [row_offset, row_offset + rows) is therefore identical whichever rank or
 * shard count produces it.  Counterpart of VectorPool's per-shard init
 * (src/model/pool.py:19-40; jax.random.normal per shard with fold_in).
 * out: bf16 [rows, ld], ld % 8 == 0.
 */
DWA_API dwa_status dwa_pool_init_normal(void* out, int64_t rows, int64_t cols, int64_t ld,
                                int64_t row_offset, uint64_t seed, float stddev,
                                dwa_stream_t stream);

/*
 * Pool keys of the retrieval: keys_w[n] = sum_s w[s] k_s / (|k_s| + 1e-8),
 * k_s = W_K[s] vectors[n] (src/model/retrieval.py:241-242, 253, 261: the
 * per-aspect projection, its L2 normalisation and the aspect collapse, one
 * tcgen05 GEMM with the normalisation and collapse in its epilogue; the
 * (S, N, d_k) projection is never materialised).
 * vectors: bf16 [N, ldv] (D used); w_k: bf16 [S * d_k, ldw] (W_K[s, kk, :] at
 * row s * d_k + kk); aspect_w: f32 [S] on the device (softmax of the aspect
 * logits); keys_out: bf16 [N, ldo].  d_k in {32, 64, 128}, D % 8 == 0,
 * 16-byte aligned bases, strides multiples of 8.  status (a device int32,
 * may be NULL) receives DWA_ERR_TIMEOUT if a bounded wait runs out.
 */
DWA_API dwa_status dwa_project_keys(const void* vectors, int64_t N, int64_t ldv, int32_t D,
                            const void* w_k, int64_t ldw, int32_t S, int32_t d_k,
                            const float* aspect_w, void* keys_out, int64_t ldo,
                            int32_t* status, dwa_stream_t stream);

/*
 * The per-aspect keys of hybrid_forward side by side (src/model/retrieval.py:
 * 154-165): keys_out[n, s d_k + j] = sqrt(w[s]) k_s[j] / (|k_s| + 1e-8) with
 * k_s = W_K[s] vectors[n].  Since sum_s w_s <q_s, k_s> = <[sqrt(w_s) q_s]_s,
 * [sqrt(w_s) k_s]_s>, hybrid_forward's aspect-weighted score is one dot
 * product of length S d_k, i.e. dwa_score_topk on these keys and the queries
 * packed the same way.  Same kernel and arguments as dwa_project_keys;
 * keys_out: bf16 [N, ldo], ldo >= S d_k.
 */
DWA_API dwa_status dwa_project_keys_packed(const void* vectors, int64_t N, int64_t ldv, int32_t D,
                            const void* w_k, int64_t ldw, int32_t S, int32_t d_k,
                            const float* aspect_w, void* keys_out, int64_t ldo,
                            int32_t* status, dwa_stream_t stream);

/* ------------------------------------------------------------------------
 * Cross-shard exchange over NVLink peer memory: the all-gather + merge of
 * _chip_topk (src/model/retrieval.py:295-302) as one kernel that reads the
 * other GPUs' candidate lists directly, instead of a collective followed by
 * a merge.  Each rank of a group owns one exchange buffer made by
 * dwa_peer_alloc (set-up time, not per call) and opens the others' with
 * dwa_peer_open; handles travel between processes as DWA_IPC_HANDLE_BYTES
 * opaque bytes (CUDA IPC).
 * ------------------------------------------------------------------------ */
#define DWA_IPC_HANDLE_BYTES 64
#define DWA_MAX_PEERS 16

/* cudaMalloc(bytes), zero-filled, and its IPC handle (out_handle: 64 bytes). */
DWA_API dwa_status dwa_peer_alloc(size_t bytes, void** out_ptr, void* out_handle);
/* Maps another process's dwa_peer_alloc buffer (peer access enabled). */
DWA_API dwa_status dwa_peer_open(const void* handle, void** out_ptr);
DWA_API dwa_status dwa_peer_close(void* ptr);  /* unmaps a dwa_peer_open mapping */
DWA_API dwa_status dwa_peer_free(void* ptr);   /* frees a dwa_peer_alloc buffer */

/*
 * After this stream's earlier work: makes it visible system-wide, then writes
 * `value` to flag word my_rank of every rank's flag array (flag_bases[p] =
 * rank p's flag array as mapped on this GPU; P ranks, P <= DWA_MAX_PEERS).
 */
DWA_API dwa_status dwa_peer_signal(void* const* flag_bases, int32_t P, int32_t my_rank,
                           int32_t value, dwa_stream_t stream);

/*
 * Global top-k of P ranks' candidate lists read over NVLink: packed[p] is
 * rank p's int32 [M, k, 2] list (fused score bits, global index), sorted
 * best first, as mapped on this GPU.  Each warp first waits until
 * flags[p] >= step for every p (this GPU's flag array, written by the
 * ranks' dwa_peer_signal); a wait longer than wait_ns nanoseconds
 * (<= 0: DWA_PEER_WAIT_DEFAULT_NS; capped at DWA_PEER_WAIT_MAX_NS) records
 * DWA_ERR_TIMEOUT in *status, writes -inf / -1 for that row and returns.
 * Choose wait_ns above the longest time a peer can lag (its own score kernel
 * plus host-side stalls).  out_vals f32 / out_idx i32 [M, k] (ties: lower
 * global index first, as lax.top_k).  k must be even and the lists 16-byte
 * aligned (each row is staged in shared memory with 16-byte loads).
 */
#define DWA_PEER_WAIT_DEFAULT_NS 30000000000LL
#define DWA_PEER_WAIT_MAX_NS 600000000000LL
DWA_API dwa_status dwa_merge_topk_peers(const void* const* packed, int32_t P, int64_t M, int32_t k,
                                const int32_t* flags, int32_t step, int64_t wait_ns,
                                float* out_vals, int32_t* out_idx, int32_t* status,
                                dwa_stream_t stream);

/*
 * Owner-computes value sum with the cross-rank sum over NVLink (the
 * reference's gather + einsum, assembly.py:104-127, on a row-sharded pool,
 * where the partial sums of the shards must be added).  Row block o of the
 * output, rows [o * block_rows, (o + 1) * block_rows), belongs to rank o.
 *  1. dwa_weighted_gather_peers: alpha (all rows, local) and this shard's
 *     partial sum of every row m, stored into the inbox of the rank owning m,
 *     at inboxes[o] + ((rank * block_rows) + m - o * block_rows) * d (f32);
 *     then dwa_peer_signal on the "partials ready" flag arrays.
 *  2. dwa_reduce_broadcast_peers: waits (bounded) until every rank's partials
 *     flag >= step, sums its block's P partials (inbox [P][block_rows][d])
 *     and writes the sums into every rank's output (outs[p]: f32 [M, d]);
 *     then dwa_peer_signal on the "block done" flag arrays.
 *  3. dwa_peer_wait on the "block done" flags before the output is read.
 * d % 8 == 0; P <= DWA_MAX_PEERS.  The waits give up after wait_ns (as in
 * dwa_merge_topk_peers) and record DWA_ERR_TIMEOUT in *status.
 */
DWA_API dwa_status dwa_weighted_gather_peers(const float* vals, const int32_t* gidx, int64_t M,
                                     int32_t k, const void* values, int64_t row_begin,
                                     int64_t row_end, int64_t ldv, int32_t d,
                                     void* const* inboxes, int32_t P, int32_t rank,
                                     int64_t block_rows, float* alpha_out, dwa_stream_t stream);
DWA_API dwa_status dwa_reduce_broadcast_peers(const float* inbox, int32_t P, int32_t rank,
                                      int64_t block_rows, int64_t M, int32_t d,
                                      void* const* outs, const int32_t* flags, int32_t step,
                                      int64_t wait_ns, int32_t* status, dwa_stream_t stream);
DWA_API dwa_status dwa_peer_wait(const int32_t* flags, int32_t P, int32_t step, int64_t wait_ns,
                         int32_t* status, dwa_stream_t stream);

/* ------------------------------------------------------------------------
 * Low-rank weight assembly: the consumer of the retrieved rows in a DWA
 * block, WeightAssembler.__call__ with per-position idx
 * (src/model/assembly.py:75-128).  Pool row layout (assembly.py:10-14):
 * [U (d_B x r) | V (r x d_A) | b (d_B) | unused], row-major blocks.
 * ------------------------------------------------------------------------ */

/*
 * delta[m, :] = sum_j alpha[m, j] (U_j (V_j h[m]) + b_j), j over the entries of
 * gidx[m, :] owned by this shard, U_j, V_j, b_j the blocks of pool row
 * vectors[gidx[m, j] - row_begin] (assembly.py:104, 123-127: the reference's
 * vectors[idx] gather + the three einsums, without materialising the gather).
 * h: [M, ldh] bf16 (h_is_bf16 = 1) or f32.  alpha f32 [M, k], gidx i32 [M, k].
 * vectors: bf16 [row_end - row_begin, ldv], ldv >= d_B r + r d_A + d_B.
 * delta f32 [M, d_B] is overwritten; shards' partial deltas add up.
 * Requirements: d_A and d_B multiples of 8 with d_A <= 8192, 1 <= r <= 32,
 * ldv % 8 == 0, 16-byte aligned vectors.
 */
DWA_API dwa_status dwa_lowrank_delta(const void* h, int32_t h_is_bf16, int64_t ldh,
                             const float* alpha, const int32_t* gidx, int64_t M, int32_t k,
                             const void* vectors, int64_t row_begin, int64_t row_end,
                             int64_t ldv, int32_t d_A, int32_t d_B, int32_t r,
                             float* delta, dwa_stream_t stream);

/*
 * The same delta as dwa_lowrank_delta, organised by pool row: the (token,
 * entry) pairs are sorted by owned row, each selected row's U | V | b is read
 * from HBM about once and applied to every token that selected it, each pair
 * writes alpha (U_j (V_j h[m]) + b_j) to its own slot of the workspace, and a
 * final pass sums each token's slots in entry order (no float atomics: the
 * result is the same on every run).  Reads ~1.2x the selected rows instead of
 * one row per (token, entry), at the cost of M k d_B floats written and read
 * back.  Sums may differ from dwa_lowrank_delta's in the last bits (another
 * order of the V_j h[m] dot products).
 * Extra requirements: M k <= INT32_MAX; the row's U | V | b
 * ((d_B r + r d_A + d_B) bf16) at most 200 KB; h rows 16-byte aligned (ldh a
 * multiple of 8 for bf16, 4 for f32); delta 16-byte aligned.
 * workspace: >= dwa_lowrank_delta_rows_workspace(M, k, row_end - row_begin,
 * d_B) bytes, 256-byte aligned, not shared with a concurrent call.
 */
DWA_API size_t dwa_lowrank_delta_rows_workspace(int64_t M, int32_t k, int64_t n_rows,
                                                int32_t d_B);
DWA_API dwa_status dwa_lowrank_delta_rows(const void* h, int32_t h_is_bf16, int64_t ldh,
                                          const float* alpha, const int32_t* gidx, int64_t M,
                                          int32_t k, const void* vectors, int64_t row_begin,
                                          int64_t row_end, int64_t ldv, int32_t d_A,
                                          int32_t d_B, int32_t r, float* delta, void* workspace,
                                          size_t workspace_bytes, dwa_stream_t stream);

/*
 * out[m, :] = LayerNorm(residual[m, :] + gamma * (base[m, :] + delta[m, :]))
 * (assembly.py:128: residual = h_A when d_A == d_B, base = h_A W_base^T +
 * b_base, computed by the caller's GEMM).  residual (bf16 or f32, stride
 * ldr) and base (f32 [M, d_B]) may be NULL (zero); ln_scale / ln_bias
 * (f32 [d_B]) may be NULL (1 / 0).  Mean and variance over the row, then
 * (x - mean) / sqrt(var + eps) * scale + bias; out f32 [M, d_B].
 */
DWA_API dwa_status dwa_assemble_finish(const void* residual, int32_t residual_is_bf16, int64_t ldr,
                               const float* base, const float* delta, int64_t M, int32_t d_B,
                               float gamma, const float* ln_scale, const float* ln_bias,
                               float eps, float* out, dwa_stream_t stream);

/*
 * Pool-usage EMA (src/training/trainer.py:227-233, src/model/pool.py:52-55):
 * ema *= beta, then ema[gidx[e] - row_begin] += weight * alpha[e] for the n
 * entries whose row this shard owns (f32 atomics).  For the reference's
 * update pass weight = (1 - beta) / n_total; to fold several blocks' entries
 * into one update call once with beta and then with beta = 1.
 * ema: f32 [row_end - row_begin].
 */
DWA_API dwa_status dwa_usage_ema(const float* alpha, const int32_t* gidx, int64_t n,
                         int64_t row_begin, int64_t row_end, float weight, float beta,
                         float* ema, dwa_stream_t stream);

/*
 * Device-side status word of a workspace: DWA_OK, or the first error a
 * kernel recorded there (DWA_ERR_TIMEOUT from a bounded wait).  Copies 4
 * bytes device->host on `stream` and synchronises that stream.
 */
DWA_API dwa_status dwa_workspace_status(const void* ws, dwa_stream_t stream, int32_t* out_status);

#ifdef __cplusplus
}  /* extern "C" */
#endif

#endif /* DWA_RETRIEVAL_H_ */
