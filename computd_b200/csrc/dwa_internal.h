// dwa_internal.h — launch plans and launchers shared by the kernel files and
// the C ABI (capi.cu).  Nothing here is exported from the shared library.
#pragma once

#include <cstddef>
#include <cstdint>
#include <cuda.h>
#include <cuda_runtime.h>

namespace dwa {

// Tile shape of the fused score + top-k kernel: a CTA pair (cta_group::2)
// computes 2 x kTileM query rows against kTileN keys per MMA.
constexpr int kTileM = 128;   // query rows per CTA   (TMEM lanes)
constexpr int kTileN = 256;   // pool keys per tile   (UMMA N, TMEM columns)
constexpr int kTileK = 64;    // bf16 elements per 128-byte swizzled row
constexpr size_t kStatusBytes = 256;  // status word block at the head of the workspace
constexpr int kMaxSplits = 128;       // most lists one merge handles (key splits or shards)
#define DWA_MERGE_MAX_K 128           // most entries a merged list keeps

// How one dwa_score_topk call is cut into work units.
// A unit is (query tile, contiguous range of key tiles); each unit leaves one
// partial top-k list per query row in the workspace, merged afterwards.
struct ScoreTopkPlan {
  int64_t M = 0, N = 0;
  int d = 0, k = 0;
  int n_qt = 0;        // pair query tiles = ceil(M / 256)
  int64_t n_kt = 0;    // key tiles    = ceil(N / 256)
  int n_split = 0;     // key-range splits per query tile
  int group = 0;       // query tiles per unit group (0: plain split-major order)
  int num_kb = 0;      // k-blocks of 64 along d
  int kcap = 0;        // heap capacity variant (16, 32, 64, 128)
  int nwg = 1;         // epilogue warpgroups (1 or 2), one partial list each per unit
  int64_t m_pad = 0;   // n_qt * 256
  size_t ws_bytes = 0; // status block + per-row bounds + partial lists
};

// Sets the thread-local message dwa_last_error() returns; returns `s`.
int32_t record_error(int32_t s, const char* msg);

// Returns false when the shape is outside what the kernel supports.
bool plan_score_topk(int64_t M, int64_t N, int d, int k, int num_sms, ScoreTopkPlan* plan);

// Number of SMs of the current device (cached per device).
int device_sm_count();

// Optional output of the fused kernel: out[g * ld + n] = mean over the rows m
// of group g (rows [g * group_rows, (g + 1) * group_rows)) of v(s[m, n]).
struct SeqMeanOut {
  float* out;
  int64_t ld;
  int64_t group_rows;  // divides M
};

// Launches the fused kernel + split merge.  Arguments were validated by the caller.
// `params` (device {lambda, tau, T}, may be null) overrides the host scalars.
cudaError_t launch_score_topk(const ScoreTopkPlan& plan, const void* q, int64_t ldq,
                              const void* keys, int64_t ldk, float lambda_sharp, float tau,
                              float T, int use_sigmoid, int64_t idx_offset, float* out_vals,
                              int32_t* out_idx, void* ws, cudaStream_t stream,
                              const char** err_detail, const float* params = nullptr,
                              const SeqMeanOut* seq_mean = nullptr);

// Generic candidate merge.  Candidate (list l, position p, row r) lives at
// offset l*stride_list + p*stride_pos + r*stride_row.  When `transform` is
// set, candidate scores are raw dot products s and the output holds
// v(s) = [sigmoid(lambda (s - tau))] * exp(s / T); otherwise the scores are
// copied.  Indices get `idx_offset` added.  `params` (device {lambda, tau,
// T}, may be null) overrides the host scalars; scalars that fail the device
// check record DWA_ERR_DEVICE_CHECK in `status` (may be null).
cudaError_t launch_merge_topk(const float* cand_vals, const int32_t* cand_idx, int n_lists,
                              int k_in, int64_t stride_list, int64_t stride_pos,
                              int64_t stride_row, int64_t M, int k, int transform,
                              float lambda_sharp, float tau, float T, int use_sigmoid,
                              int64_t idx_offset, float* out_vals, int32_t* out_idx,
                              cudaStream_t stream, const float* params = nullptr,
                              int* status = nullptr);

cudaError_t launch_weighted_gather(const float* vals, const int32_t* gidx, int64_t M, int k,
                                   const void* values, int64_t row_begin, int64_t row_end,
                                   int64_t ldv, int d, float* out, float* alpha_out,
                                   cudaStream_t stream);

cudaError_t launch_gather_dot(const void* a, int a_bf16, int64_t lda, const int32_t* idx, int64_t M,
                              int k, const void* rows, int64_t row_begin, int64_t row_end,
                              int64_t ldr, int d, float* out, cudaStream_t stream);
cudaError_t launch_score_backward(const float* v, const float* s, const float* dalpha, int64_t M,
                                  int k, float lambda_sharp, float tau, float T, int use_sigmoid,
                                  float* ds, float* dparams, cudaStream_t stream,
                                  const float* params = nullptr, int* status = nullptr);

// seq_scores.cu: sims[b, n] = <q[b], keys[n]> (f32 x bf16, fp32 accumulate)
// and fused[b, n] = v(sims[b, n]) for a few (<= 64) query rows against a
// whole key shard.  Arguments validated by the caller.
cudaError_t launch_seq_scores(const float* q, int64_t B, int64_t ldq, const void* keys, int64_t N,
                              int64_t ldk, int d, const float* params, int use_sigmoid,
                              float* sims, int64_t lds, float* fused, int64_t ldf, int* status,
                              cudaStream_t stream);
int seq_scores_max_d();  // largest d launch_seq_scores accepts

// lm_ops.cu: the LM block's fused elementwise steps (dwa_lm.h)
cudaError_t launch_rope_qk(const void* qkv, int64_t B, int64_t S, int H, int dh, int64_t ld_qkv,
                           const void* cosv, const void* sinv, int64_t ld_cs, void* q_out,
                           void* k_out, cudaStream_t stream);
cudaError_t launch_aspect_queries(const void* q, int64_t M, int S, int d_k, int64_t ldq,
                                  const float* logits, const float* tau_param, float lambda_sharp,
                                  float T, int use_sigmoid, void* out, int64_t ldo, float* w_out,
                                  float* params_out, cudaStream_t stream);
int lm_max_aspects();
cudaError_t launch_gather_rows(const float* wts, const int32_t* idx, int64_t M, int k,
                               const void* rows, int64_t row_begin, int64_t row_end, int64_t ldr,
                               int d, float* out, int accumulate, cudaStream_t stream);
cudaError_t launch_scatter_add_rows(const float* wts, const int32_t* idx, int64_t M, int k,
                                    const void* a, int a_bf16, int64_t lda, int64_t row_begin,
                                    int64_t row_end, float* grad, int64_t ldg, int d,
                                    cudaStream_t stream);

// score_topk.cu: 2-D bf16 tensor map, 128-byte swizzle, box (box_inner x box_rows)
bool make_bf16_tile_map(CUtensorMap* map, const void* ptr, uint64_t inner, uint64_t rows,
                        uint64_t ld_elems, uint32_t box_inner, uint32_t box_rows);

// weighted_gather.cu: NVLink owner-computes reduction
cudaError_t launch_weighted_gather_peers(const float* vals, const int32_t* gidx, int64_t M, int k,
                                         const void* values, int64_t row_begin, int64_t row_end,
                                         int64_t ldv, int d, float* const* inboxes, int P, int rank,
                                         int64_t block_rows, float* alpha_out, cudaStream_t stream);
cudaError_t launch_reduce_broadcast_peers(const float* inbox, int P, int rank, int64_t block_rows,
                                          int64_t M, int d, float* const* outs, const int32_t* flags,
                                          int step, uint64_t wait_ns, int* status,
                                          cudaStream_t stream);
cudaError_t launch_peer_wait(const int32_t* flags, int P, int step, uint64_t wait_ns, int* status,
                             cudaStream_t stream);

// Limits of the waits for other ranks' flags (the peer merge, reduce and wait):
// a caller's wait_ns <= 0 takes the default; larger values are capped.
constexpr uint64_t kPeerWaitDefaultNs = 30ull * 1000000000ull;
constexpr uint64_t kPeerWaitMaxNs = 600ull * 1000000000ull;

// key_projection.cu
// packed = false: the collapsed keys [N, d_k]; true: [sqrt(w_s) k_s / (|k_s| + 1e-8)]_s [N, S d_k].
cudaError_t launch_project_keys(const void* vectors, int64_t N, int64_t ldv, int D, const void* w_k,
                                int64_t ldw, int S, int d_k, const float* aspect_w, void* keys_out,
                                int64_t ldo, int* status, cudaStream_t stream, bool packed = false);

// merge_topk.cu: NVLink peer exchange
int max_peers();
cudaError_t launch_peer_signal(int32_t* const* flag_bases, int n, int my_rank, int value,
                               cudaStream_t stream);
cudaError_t launch_merge_topk_peers(const int32_t* const* packed, int n, int64_t M, int k,
                                    const int32_t* flags, int step, uint64_t wait_ns,
                                    float* out_vals, int32_t* out_idx, int* status,
                                    cudaStream_t stream);

// assembly.cu
size_t lowrank_delta_smem_bytes(int d_A, int k, int r);
cudaError_t launch_lowrank_delta(const void* h, int h_bf16, int64_t ldh, const float* alpha,
                                 const int32_t* gidx, int64_t M, int k, const void* vectors,
                                 int64_t row_begin, int64_t row_end, int64_t ldv, int d_A, int d_B,
                                 int r, float* delta, cudaStream_t stream);
// backward.cu: the queries-side backward of a one-GPU pool in one launch
cudaError_t launch_retrieval_backward(const void* q, int q_bf16, int64_t ldq, const float* dout,
                                      int64_t ld_dout, const void* keys, int64_t ldk, int d_k,
                                      const void* values, int64_t ldv, int d_v, const float* v,
                                      const int32_t* idx, int64_t M, int k, int64_t row_begin,
                                      int64_t row_end, float lambda_sharp, float tau, float T,
                                      const float* params, int use_sigmoid, float* ds, float* dq,
                                      float* dparams, int* status, cudaStream_t stream);
// pair_sort.cu: (query, entry) pairs of an index array sorted by owned row
struct PairSort {
  int32_t* offsets;  // [n_rows + 1]: pairs of owned row r at pairs[offsets[r] .. offsets[r + 1])
  int32_t* pairs;    // pair ids (indices into gidx)
};
size_t pair_sort_workspace_bytes(int64_t n_pairs, int64_t n_rows);
cudaError_t launch_sort_pairs_by_row(const int32_t* gidx, int64_t n_pairs, int64_t row_begin,
                                     int64_t row_end, void* ws, PairSort* out,
                                     cudaStream_t stream);
// backward.cu: dense row gradients from the row-sorted pairs (pair_sort workspace)
size_t row_gradient_workspace_bytes(int64_t M, int k, int64_t n_rows);
cudaError_t launch_row_gradient(const float* w, const int32_t* idx, int64_t M, int k, const void* a,
                                int a_bf16, int64_t lda, int64_t row_begin, int64_t row_end,
                                void* grad, int grad_bf16, int64_t ldg, int d, void* ws,
                                cudaStream_t stream);
// lowrank_rows.cu: the same delta, row-stationary (rows read once), with a caller workspace
size_t lowrank_rows_workspace_bytes(int64_t M, int k, int64_t n_rows, int d_B);
int lowrank_rows_smem_bytes(int d_A, int d_B, int r);
cudaError_t launch_lowrank_rows(const void* h, int h_bf16, int64_t ldh, const float* alpha,
                                const int32_t* gidx, int64_t M, int k, const void* vectors,
                                int64_t row_begin, int64_t row_end, int64_t ldv, int d_A, int d_B,
                                int r, float* delta, void* ws, cudaStream_t stream);
cudaError_t launch_assemble_finish(const void* residual, int res_bf16, int64_t ldr,
                                   const float* base, const float* delta, int64_t M, int d_B,
                                   float gamma, const float* ln_scale, const float* ln_bias,
                                   float eps, float* out, cudaStream_t stream);
cudaError_t launch_usage_ema(const float* alpha, const int32_t* gidx, int64_t n, int64_t row_begin,
                             int64_t row_end, float weight, float beta, float* ema,
                             cudaStream_t stream);

cudaError_t launch_pool_init_normal(void* out, int64_t rows, int64_t cols, int64_t ld,
                                    int64_t row_offset, uint64_t seed, float stddev,
                                    cudaStream_t stream);

}  // namespace dwa
