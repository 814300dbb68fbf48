/*
 * msa_b200.h - C ABI of the B200 (sm_100a) MiniMax-M3 sparse attention library.
 *
 * Drop-in boundary for the three-stage hot path of yeyeyeping/msa_triton:
 *   index score  ->  top-k block selection  ->  block-sparse GQA attention
 * The reference is a pure-Python package (Triton kernels + torch ops); it has no
 * foreign-function interface of its own, so each entry point below names the
 * reference function / kernel it replaces (paths inside the reference project).
 * A ctypes binding of every symbol lives in msa_triton_b200/_lib.py.
 *
 * Conventions shared by every entry point
 *   - Plain device pointers, element counts and a CUDA stream (cudaStream_t
 *     passed as void*; NULL = legacy default stream). No torch types.
 *   - Tensors are dense, row-major ("TND"): q[T][Hq][D], k/v[T][G][D],
 *     index_q[T][G][Di], index_k[T][1][Di], scores[T][G][NB], indices[T][G][K].
 *   - cu_seqlens: int32[nseq+1] on the device, cu[0]=0, cu[nseq]=T,
 *     nondecreasing (validated by the caller; the reference validates on the
 *     host: layout.py:18-30).
 *   - Blocks are numbered from the start of each packed sequence; the query
 *     heads g*(Hq/G) .. (g+1)*(Hq/G)-1 share group g's selection.
 *   - dtype codes: MSA_F32 = 0, MSA_F16 = 1, MSA_BF16 = 2.
 *   - Return 0 on success, otherwise an MSA_ERR_* code; msa_last_error()
 *     returns the calling thread's last message. Launches are asynchronous.
 *   - Workspace: where an entry point needs scratch memory the caller passes
 *     it; the matching *_workspace_size() returns the byte count.
 */
#ifndef MSA_B200_H_
#define MSA_B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum {
  MSA_OK = 0,
  MSA_ERR_INVALID_ARGUMENT = 1,
  MSA_ERR_UNSUPPORTED = 2,
  MSA_ERR_CUDA = 3,
  MSA_ERR_TIMEOUT = 4,
};

enum { MSA_F32 = 0, MSA_F16 = 1, MSA_BF16 = 2 };

/* Library version string and the calling thread's last error message. */
const char* msa_version(void);
const char* msa_last_error(void);

/* Number of CUDA kernels this library has launched in the process so far
 * (all entry points, all threads). Benchmarks difference it around a timed
 * region. No counterpart in the reference (it has no native code). */
uint64_t msa_kernel_launches(void);

/* Per-kernel device timing, for benchmarks (no counterpart in the reference).
 * While enabled, the tensor-core attention entry points record a CUDA event
 * pair on their stream around their main kernel ("attn_fwd_tc",
 * "attn_bwd_tc" for the fused backward, "attn_dkdv_tc" / "attn_dq_tc" when only
 * one side is requested). msa_timing_read waits for the recorded pairs
 * of `kernel`, returns their summed milliseconds and count, and forgets them. */
int msa_timing_enable(int on);
int msa_timing_read(const char* kernel, double* total_ms, int64_t* launches);

/* Small device -> host int32 read (cu_seqlens and the like) that uses no copy
 * engine: a kernel on `stream` writes the values into mapped pinned memory,
 * the call waits for it (and so for the stream's earlier work, as a
 * synchronous copy would) and copies them to `dst`. Unlike a cudaMemcpy it
 * does not queue behind bulk transfers on other streams. The reference reads
 * cu_seqlens to the host with a synchronous copy (layout.py:18-30). */
int msa_read_i32(const int32_t* src, int64_t n, int32_t* dst, void* stream);

/* cu_block_lens (exclusive prefix of per-sequence block counts) computed on
 * the device from cu_seqlens (K2QCSR.cu_block_lens, triton/k2q.py:39-128). */
int msa_block_prefix(const int32_t* cu_seqlens, int32_t nseq, int32_t block_size, int32_t* cu_block_lens,
                     void* stream);

/* ---------------------------------------------------------------- stage 1
 * Index score, precise path (float64 dot products).
 * Replaces triton/index_score.py:93-136 (_index_score_forward) as launched by
 * _IndexScore.forward (:237-265). scores[t][g][b] = max over keys j of block b
 * (sequence-local, j <= t) of scale * index_q[t][g] . index_k[j]; -inf for
 * future / out-of-sequence blocks. When max_val and tie_info are non-NULL the
 * backward state is written: max_val = the float64 maximum, tie_info = winner
 * offset + 1 when unique, else -(number of tied maxima) (0 for masked blocks).
 * scores may be NULL when only the state is wanted.
 */
int msa_index_score_fwd(const void* index_q, const void* index_k, int dtype,
                        const int32_t* cu_seqlens, int32_t nseq, int64_t total_tokens,
                        int32_t groups, int32_t index_dim, int32_t num_blocks,
                        int32_t block_size, double scale,
                        float* scores, double* max_val, int32_t* tie_info, void* stream);

/* Index score backward (ties split equally, torch.amax semantics).
 * Replaces _index_score_backward_q (index_score.py:139-178) and
 * _index_score_backward_k_group + _index_score_reduce_k (:181-232).
 * dscores: float32 [T][G][NB]. d_index_q [T][G][Di] and d_index_k [T][1][Di]
 * are written in `dtype` (either may be NULL to skip it).
 */
int msa_index_score_bwd(const void* index_q, const void* index_k, int dtype,
                        const int32_t* cu_seqlens, int32_t nseq, int64_t total_tokens,
                        int32_t groups, int32_t index_dim, int32_t num_blocks,
                        int32_t block_size, double scale,
                        const double* max_val, const int32_t* tie_info, const float* dscores,
                        void* d_index_q, void* d_index_k, void* stream);

/* Index score, tensor-core path: tcgen05 GEMM index_q . index_k^T fed by TMA
 * (rows of query tokens [q_lo, q_hi) only; other rows of `scores` are left
 * untouched -- a context-parallel rank scores its own queries against all keys)
 * with the causal mask and the per-block maximum fused in the TMEM epilogue
 * (the T x T logits never reach memory). bf16/f16 inputs, index_dim in
 * {64, 128}, block_size == 128, groups a power of two <= 128. Dot products
 * accumulate the exact products in float32. Scores only (no backward state).
 * Same output contract as msa_index_score_fwd; a kernel wait that gives up
 * leaves NaN in every score. Replaces _index_score_forward
 * (triton/index_score.py:93-136). */
int msa_index_score_fwd_tc(const void* index_q, const void* index_k, int dtype,
                           const int32_t* cu_seqlens, int32_t nseq, int64_t total_tokens,
                           int32_t groups, int32_t index_dim, int32_t num_blocks,
                           int32_t block_size, float scale, int64_t q_lo, int64_t q_hi,
                           float* scores, void* stream);

/* Tensor-core score forward with the backward's winner state (when index_q or
 * index_k needs a gradient). Same scores as msa_index_score_fwd_tc over all
 * tokens; tie_info [T][G][NB] int32 = winning key offset + 1, or -(number of
 * keys tied at the block's float64 maximum, which goes to max_val [T][G][NB]
 * float64; other max_val entries are not written), 0 for future blocks. A
 * winner is taken from the float32 tensor-core scores only when no other key
 * comes within twice a float32 accumulation error bound of it; those entries
 * are decided by float64 recomputation, so the state equals the float64
 * definition (the state _IndexScore.forward saves, triton/index_score.py:
 * 237-265). workspace: msa_index_score_state_workspace_size() bytes. */
size_t msa_index_score_state_workspace_size(int64_t total_tokens, int32_t groups);
int msa_index_score_fwd_tc_state(const void* index_q, const void* index_k, int dtype, const int32_t* cu_seqlens,
                                 int32_t nseq, int64_t total_tokens, int32_t groups, int32_t index_dim,
                                 int32_t num_blocks, int32_t block_size, float scale, float* scores,
                                 int32_t* tie_info, double* max_val, void* workspace, size_t workspace_bytes,
                                 void* stream);

/* Score backward from that state (bf16/f16, Di 64 or 128, block_size 128):
 * dq / dk (either may be NULL) in the input dtype, float64 sums rounded once.
 * dIK is transposed through per-(key block, query chunk) partial sums added in
 * a fixed order (no atomics). Replaces _index_score_backward_q / _k
 * (triton/index_score.py:139-232). workspace:
 * msa_index_score_bwd_tc_workspace_size() bytes. */
size_t msa_index_score_bwd_tc_workspace_size(int64_t total_tokens, int32_t nseq, int32_t groups, int32_t index_dim,
                                             int32_t num_blocks);
int msa_index_score_bwd_tc(const void* index_q, const void* index_k, int dtype, const int32_t* cu_seqlens,
                           int32_t nseq, int64_t total_tokens, int32_t groups, int32_t index_dim, int32_t num_blocks,
                           int32_t block_size, double scale, const double* max_val, const int32_t* tie_info,
                           const float* dscores, void* dq, void* dk, void* workspace, size_t workspace_bytes,
                           void* stream);

/* ---------------------------------------------------------------- stage 2
 * Top-k block selection. Replaces triton/topk.py:11-47 (masked_fill + torch.topk).
 * Future blocks rank -inf, the local_blocks most recent causal blocks rank
 * +inf, the top min(K, NB) are written in descending rank order (equal ranks
 * in ascending block id), -inf picks and the tail are -1.
 */
int msa_topk(const float* scores, const int32_t* cu_seqlens, int32_t nseq, int64_t total_tokens,
             int32_t groups, int32_t num_blocks, int32_t block_size, int32_t topk_blocks,
             int32_t local_blocks, int32_t* indices, void* stream);

/* ---------------------------------------------------------------- k2q CSR
 * Block -> query transpose of indices[T][G][K]. Replaces triton/k2q.py:39-128.
 * Three integer stages: per-tile histogram, exclusive scans, stable scatter.
 * Outputs: row_ptr int32[rows+1] (rows = total_blocks * G), query_indices and
 * slot_indices int32[T*G*K] (ordered by query then slot inside each row, -1
 * tail). cu_block_lens (int32[nseq+1], prefix sum of per-sequence block
 * counts) is an input computed by the caller from the host-side lengths.
 */
size_t msa_k2q_workspace_size(const int32_t* host_cu_seqlens, int32_t nseq, int32_t groups,
                              int32_t block_size);
int msa_k2q_build(const int32_t* indices, const int32_t* cu_seqlens, const int32_t* host_cu_seqlens,
                  const int32_t* cu_block_lens, int32_t nseq, int64_t total_tokens, int32_t groups,
                  int32_t topk_blocks, int32_t block_size, int32_t* row_ptr, int32_t* query_indices,
                  int32_t* slot_indices, void* workspace, size_t workspace_bytes, void* stream);
/* msa_k2q_build that allocates nothing (no counterpart in the reference): its
 * scratch is a fixed 4 MiB device array inside the library, so a caller with
 * no device allocator of its own (a plain C / cgo / JNI host reusing
 * caller-owned row_ptr / query_indices / slot_indices buffers) needs no
 * workspace and makes no allocation per call. Same inputs, outputs and order
 * as msa_k2q_build. Problems whose scratch would exceed 4 MiB (about T = 32K
 * tokens at G = 8, B = 128) are rejected with MSA_ERR_INVALID_ARGUMENT. The
 * scratch needs no zeroing (each call writes every word it reads); row_ptr is
 * zeroed by the call. The first call on each device sets up (looks up the
 * array's device address with that device current): make that first call
 * before any stream capture. The looked-up address is kept for the life of
 * the process: do not call it again on a device after cudaDeviceReset (or any
 * teardown of that device's primary context). All calls on a device share the
 * array: calls that may execute at the same time (other streams, unordered
 * threads) race. */
int msa_k2q_build_noalloc(const int32_t* indices, const int32_t* cu_seqlens, const int32_t* host_cu_seqlens,
                          const int32_t* cu_block_lens, int32_t nseq, int64_t total_tokens, int32_t groups,
                          int32_t topk_blocks, int32_t block_size, int32_t* row_ptr, int32_t* query_indices,
                          int32_t* slot_indices, void* stream);

/* ---------------------------------------------------------------- stage 3
 * Sparse attention forward, precise path (float64 arithmetic, one rounding).
 * Replaces _forward_kernel (triton/sparse_attention.py:35-84) as launched by
 * _SparseAttention.forward (:334-359). out [T][Hq][D] in `dtype`, lse float32
 * [T][Hq] (natural log, -inf for empty rows), lse64 float64 [T][Hq] is the
 * backward state. Duplicate block ids in a row select their block once.
 */
int msa_attn_fwd(const void* q, const void* k, const void* v, int dtype, const int32_t* indices,
                 const int32_t* cu_seqlens, int32_t nseq, int64_t total_tokens, int32_t q_heads,
                 int32_t groups, int32_t head_dim, int32_t topk_blocks, int32_t block_size,
                 double scale, void* out, float* lse, double* lse64, void* stream);

/* Sparse attention forward, tensor-core path (bf16/f16, head_dim 128,
 * block_size 128, Hq/G in {4, 8, 16}, Hq >= 8). Key-block stationary: walks the k2q CSR
 * (row_ptr / query_indices from msa_k2q_build, num_rows = total_blocks * G),
 * gathers the selecting tokens' query heads into 128-row tiles with TMA,
 * computes S = Q K^T and O += P V with tcgen05 (TMEM accumulators), exponent
 * against a per-row upper bound |scale||q| max|k| over the row's selected key
 * blocks. Rows whose bound sits so far above their logits that the row's mass
 * l < 2^-88 are re-run through the same tensor-core kernel, re-centred on
 * their exact logit maximum (rows still short after that would go to the
 * float64 row kernel), so any input scale stays on the tensor cores. Same
 * contract as
 * msa_attn_fwd for out and lse. workspace: msa_attn_fwd_tc_workspace_size()
 * bytes (float32 O accumulator [T][Hq][128], row sums and bounds, schedule).
 * Replaces _forward_kernel (triton/sparse_attention.py:35-84). */
size_t msa_attn_fwd_tc_workspace_size(int64_t total_tokens, int32_t q_heads, int32_t num_rows, int32_t groups,
                                      int32_t topk_blocks);
int msa_attn_fwd_tc(const void* q, const void* k, const void* v, int dtype, const int32_t* indices,
                    const int32_t* cu_seqlens, const int32_t* cu_block_lens, const int32_t* row_ptr,
                    const int32_t* query_indices, int32_t nseq, int64_t total_tokens, int32_t q_heads,
                    int32_t groups, int32_t head_dim, int32_t topk_blocks, int32_t block_size, double scale,
                    int32_t num_rows, void* out, float* lse, void* workspace, size_t workspace_bytes,
                    void* stream);
/* msa_attn_fwd_tc for the query tokens [q_lo, q_hi) only: out and lse rows
 * outside the range are not written, and the per-row passes (bounds,
 * accumulator zeroing, finalize) cover the range alone. Tokens outside the
 * range must select no block (indices -1). A context-parallel rank uses it on
 * full-length buffers that hold its own query slice (no counterpart in the
 * reference, which has no multi-GPU path). */
int msa_attn_fwd_tc_range(const void* q, const void* k, const void* v, int dtype, const int32_t* indices,
                          const int32_t* cu_seqlens, const int32_t* cu_block_lens, const int32_t* row_ptr,
                          const int32_t* query_indices, int32_t nseq, int64_t total_tokens, int32_t q_heads,
                          int32_t groups, int32_t head_dim, int32_t topk_blocks, int32_t block_size, double scale,
                          int32_t num_rows, int64_t q_lo, int64_t q_hi, void* out, float* lse, void* workspace,
                          size_t workspace_bytes, void* stream);
/* Synchronously reads the error word a previous msa_attn_fwd_tc left in
 * `workspace` (0 = ok, else the code of the bounded wait that gave up). */
int msa_attn_fwd_tc_error(const void* workspace, int64_t total_tokens, int32_t q_heads, int32_t num_rows,
                          int32_t* host_err);
/* Synchronously reads how many rows of the last msa_attn_fwd_tc on `workspace`
 * needed the re-centred tensor-core re-run (`rerun_rows`: their bound sat so
 * far above their logits that l < 2^-88) and how many of those still went to
 * the float64 row kernel (`f64_rows`). Diagnostics of the row bound; the
 * reference's online-softmax kernel (sparse_attention.py:35-84) has no such
 * state. */
int msa_attn_fwd_tc_rerun_counts(const void* workspace, int64_t total_tokens, int32_t q_heads, int32_t num_rows,
                                 int32_t* rerun_rows, int32_t* f64_rows);

/* Query-owned backward: dQ (if dq != NULL) and the per-(token, head) softmax
 * derivative centre delta64 = sum_j P_j dP_j (if delta64 != NULL).
 * Replaces _backward_kernel (sparse_attention.py:87-198) without atomics. */
int msa_attn_bwd_q(const void* q, const void* k, const void* v, const void* dout, int dtype,
                   const int32_t* indices, const int32_t* cu_seqlens, int32_t nseq,
                   int64_t total_tokens, int32_t q_heads, int32_t groups, int32_t head_dim,
                   int32_t topk_blocks, int32_t block_size, double scale, const double* lse64,
                   void* dq, double* delta64, void* stream);

/* Key-owned backward: dK / dV (either may be NULL) by walking the k2q CSR,
 * fixed-order float64 sums, no floating-point atomics.
 * Replaces _backward_kv_kernel (sparse_attention.py:223-295). */
int msa_attn_bwd_kv(const void* q, const void* k, const void* v, const void* dout, int dtype,
                    const int32_t* indices, const int32_t* cu_seqlens, const int32_t* cu_block_lens,
                    const int32_t* row_ptr, const int32_t* query_indices, const int32_t* slot_indices,
                    int32_t nseq, int64_t total_tokens, int32_t q_heads, int32_t groups,
                    int32_t head_dim, int32_t topk_blocks, int32_t block_size, double scale,
                    const double* lse64, const double* delta64, void* dk, void* dv, void* stream);

/* Tensor-core backward (tcgen05/TMA; bf16/f16, head_dim 128, block_size 128,
 * Hq/G in {4, 8, 16}, Hq >= 8). out / lse are the forward's outputs.
 * dK/dV (either may be NULL) are key-block stationary over the k2q CSR with
 * TMEM accumulators: deterministic, no floating-point atomics (replaces
 * _backward_kv_kernel, triton/sparse_attention.py:223-296). dQ (may be NULL)
 * accumulates per-(key block, query tile) products in a float32 buffer
 * inside `workspace` (the role of the dQ of _backward_kernel,
 * sparse_attention.py:87-199); with dK or dV it comes out of the same pass
 * (dS computed once). kv_dtype: dtype of dk / dv, `dtype` or MSA_F32
 * (float32 partial sums, e.g. for a context-parallel reduce-scatter).
 * workspace: msa_attn_bwd_tc_workspace_size() bytes. A bounded wait that
 * gives up leaves a code in the workspace's error word and NaN in every
 * requested gradient. */
size_t msa_attn_bwd_tc_workspace_size(int64_t total_tokens, int32_t q_heads, int32_t num_rows, int32_t groups,
                                      int32_t topk_blocks);
int msa_attn_bwd_tc(const void* q, const void* k, const void* v, const void* out, const void* dout,
                    const float* lse, int dtype, const int32_t* cu_seqlens, const int32_t* cu_block_lens,
                    const int32_t* row_ptr, const int32_t* query_indices, int32_t nseq, int64_t total_tokens,
                    int32_t q_heads, int32_t groups, int32_t head_dim, int32_t topk_blocks, int32_t block_size,
                    double scale, int32_t num_rows, void* dq, void* dk, void* dv, int kv_dtype,
                    void* workspace, size_t workspace_bytes, void* stream);
/* msa_attn_bwd_tc for the query tokens [q_lo, q_hi) only (the forward's range):
 * dq rows outside it are not written; dk / dv cover every key as above. Tokens
 * outside the range must select no block. */
int msa_attn_bwd_tc_range(const void* q, const void* k, const void* v, const void* out, const void* dout,
                          const float* lse, int dtype, const int32_t* cu_seqlens, const int32_t* cu_block_lens,
                          const int32_t* row_ptr, const int32_t* query_indices, int32_t nseq, int64_t total_tokens,
                          int32_t q_heads, int32_t groups, int32_t head_dim, int32_t topk_blocks,
                          int32_t block_size, double scale, int32_t num_rows, int64_t q_lo, int64_t q_hi, void* dq,
                          void* dk, void* dv, int kv_dtype, void* workspace, size_t workspace_bytes, void* stream);
/* Synchronously reads the error word of a previous msa_attn_bwd_tc's workspace. */
int msa_attn_bwd_tc_error(const void* workspace, int32_t* host_err);

/* Private regression path: query-owned backward with float64 atomics for
 * dK/dV. Replaces _SparseAttentionAtomicReference.backward
 * (sparse_attention.py:398-426). dk_acc / dv_acc: float64 [T][G][D] scratch,
 * zeroed by this call; dk / dv written in `dtype`. */
int msa_attn_bwd_atomic(const void* q, const void* k, const void* v, const void* dout, int dtype,
                        const int32_t* indices, const int32_t* cu_seqlens, int32_t nseq,
                        int64_t total_tokens, int32_t q_heads, int32_t groups, int32_t head_dim,
                        int32_t topk_blocks, int32_t block_size, double scale, const double* lse64,
                        void* dq, double* dk_acc, double* dv_acc, void* dk, void* dv, void* stream);

/* ---------------------------------------------------------------- decode over a paged KV cache
 * One new query token per request against a paged cache: page p of the cache
 * holds page_size consecutive key tokens of one request, block_table[b][i] the
 * physical page of request b's logical page i, seq_lens[b] the request's key
 * count including the new token (at position seq_lens[b] - 1). Caches:
 * index_k_cache [num_pages][page_size][1][Di], k_cache / v_cache
 * [num_pages][page_size][G][D]. Selection semantics as in prefill (block b of
 * the request is valid iff b <= (seq_lens[b] - 1) / block_size; causal keys;
 * repeated ids count once; -1 pads). The reference describes the serving
 * layouts (docs/vllm_ascend_k2q.md:22-40) but implements no decode path. */

/* scores [B][G][num_blocks] float32: block maxima of scale * iq[b][g] . ik[j]
 * (float32 sums), -inf for blocks past the query; groups * index_dim <= 4096. */
int msa_decode_index_score(const void* index_q, const void* index_k_cache, int dtype, const int32_t* block_table,
                           const int32_t* seq_lens, int32_t batch, int32_t groups, int32_t index_dim,
                           int32_t page_size, int32_t max_pages, int32_t num_blocks, int32_t block_size,
                           double scale, float* scores, void* stream);

/* Top-k of score rows whose query positions are given directly (positions[t],
 * within the query's sequence; decode: seq_lens - 1): the rule of msa_topk. */
int msa_topk_positions(const float* scores, const int32_t* positions, int64_t total_tokens, int32_t groups,
                       int32_t num_blocks, int32_t block_size, int32_t topk_blocks, int32_t local_blocks,
                       int32_t* indices, void* stream);

/* out [B][Hq][D] (dtype), lse [B][Hq] float32 (natural log, -inf without keys):
 * split over the selected blocks, then a combine. h = Hq / G <= 16, D <= 256.
 * workspace: msa_decode_attn_workspace_size() bytes (per-slot partials). */
size_t msa_decode_attn_workspace_size(int32_t batch, int32_t q_heads, int32_t head_dim, int32_t topk_blocks);
int msa_decode_attn(const void* q, const void* k_cache, const void* v_cache, int dtype, const int32_t* block_table,
                    const int32_t* seq_lens, const int32_t* indices, int32_t batch, int32_t q_heads, int32_t groups,
                    int32_t head_dim, int32_t page_size, int32_t max_pages, int32_t topk_blocks, int32_t block_size,
                    double scale, void* out, float* lse, void* workspace, size_t workspace_bytes, void* stream);

/* ---------------------------------------------------------------- index KL loss
 * The indexer's sparse-stage KL objective. The reference specifies it but has
 * no kernel (docs/msa_training_flow.md:92-138, docs/implementation_plan.md:
 * 66-69); these entry points have no counterpart to replace. On the selected
 * causal keys J(t, g) of each (token, group) pair (the attention's key set):
 *   student p_s = softmax_J(index_scale * index_q[t,g] . index_k[j]),
 *   teacher p_T = mean over the group's query heads of softmax_J(scale * q[t,h] . k[j,g]),
 *   loss = sum over pairs of KL(p_T || p_s) / (T * G);  dL/ds_j = (p_s - p_T) / (T * G).
 * pt [T*G][K][block_size] holds p_T per (pair, selection slot, key) after the
 * teacher step, and index_scale * dL/ds_j after a student step with need_grad
 * (zero for keys past the query; invalid or repeated slots are left unwritten). */

/* Teacher, tensor-core path (shapes of msa_attn_fwd_tc): the attention forward's
 * S = Q K^T tiles over the k2q CSR (row_ptr / query_indices / slot_indices of
 * msa_k2q_build), P = exp(S - lse) with lse the main attention's float32 LSE
 * [T][Hq] (from msa_attn_fwd_tc), head mean written to float32 pt.
 * workspace: msa_index_kl_teacher_tc_workspace_size() bytes. */
size_t msa_index_kl_teacher_tc_workspace_size(int64_t total_tokens, int32_t q_heads, int32_t num_rows,
                                              int32_t groups, int32_t topk_blocks);
int msa_index_kl_teacher_tc(const void* q, const void* k, int dtype, const float* lse, const int32_t* cu_seqlens,
                            const int32_t* cu_block_lens, const int32_t* row_ptr, const int32_t* query_indices,
                            const int32_t* slot_indices, int32_t nseq, int64_t total_tokens, int32_t q_heads,
                            int32_t groups, int32_t head_dim, int32_t topk_blocks, int32_t block_size,
                            double scale, int32_t num_rows, float* pt, void* workspace, size_t workspace_bytes,
                            void* stream);

/* Student logits, key-block stationary (16-bit index tensors, index_dim 64,
 * block_size 128): one CTA per (key block, group) walks the group's k2q CSR row,
 * the block's index_k rows in registers (thread = key), and writes
 * sbuf[(pair, slot)][key] = index_scale * index_q[t,g] . index_k[key] (float32,
 * pt's layout) for every edge. */
int msa_index_kl_logits_tc(const void* index_q, const void* index_k, int dtype, const int32_t* cu_seqlens,
                           const int32_t* cu_block_lens, const int32_t* row_ptr, const int32_t* query_indices,
                           const int32_t* slot_indices, int32_t nseq, int64_t total_tokens, int32_t groups,
                           int32_t topk_blocks, int32_t total_blocks, double index_scale, float* sbuf, void* stream);

/* Student step after the tensor-core teacher and msa_index_kl_logits_tc:
 * streams pt and sbuf once per pair (no index_k reads): loss (one device
 * float64, fixed-order sum) and, with need_grad, pt overwritten with
 * index_scale * dL/ds_j. block_size 128. workspace:
 * msa_index_kl_student_workspace_size() bytes. */
int msa_index_kl_student_tc(const float* sbuf, float* pt, const int32_t* indices, const int32_t* cu_seqlens,
                            int32_t nseq, int64_t total_tokens, int32_t groups, int32_t topk_blocks,
                            double index_scale, int need_grad, double* loss, void* workspace,
                            size_t workspace_bytes, void* stream);

/* Gradients after msa_index_kl_student_tc (16-bit index tensors, index_dim 64,
 * block_size 128): one key-block-stationary walk of the k2q CSR per (block,
 * group) on tcgen05, 128 edges per step: d_index_k [T][64] float32 (sum over
 * selecting pairs of g * index_q, accumulated in TMEM over the row) and, per
 * edge, the products of its g row with the block's index_k rows, summed per pair
 * over its selection slots in order into d_index_q [T][G][64] float32. g enters
 * the tensor cores as 16-bit values scaled by a power of two chosen from
 * index_scale and T * G (|g| <= |index_scale| / (T * G)). No atomics.
 * workspace: msa_index_kl_grad_tc_workspace_size() bytes. */
size_t msa_index_kl_grad_tc_workspace_size(int64_t total_tokens, int32_t groups, int32_t topk_blocks);
int msa_index_kl_grad_tc(const void* index_q, const void* index_k, int dtype, const int32_t* indices,
                         const int32_t* cu_seqlens, const int32_t* cu_block_lens, const int32_t* row_ptr,
                         const int32_t* query_indices, const int32_t* slot_indices, int32_t nseq,
                         int64_t total_tokens, int32_t groups, int32_t topk_blocks, int32_t total_blocks,
                         double index_scale, const float* g_pt, float* d_index_q, float* d_index_k,
                         void* workspace, size_t workspace_bytes, void* stream);

/* Teacher, precise path (any shape, float64): pt is float64. */
int msa_index_kl_teacher(const void* q, const void* k, int dtype, const int32_t* indices,
                         const int32_t* cu_seqlens, int32_t nseq, int64_t total_tokens, int32_t q_heads,
                         int32_t groups, int32_t head_dim, int32_t topk_blocks, int32_t block_size,
                         double scale, double* pt, void* stream);

/* Student step: loss (one device float64, fixed-order sum) and, with need_grad,
 * d_index_q_acc [T][G][Di] (index_scale * dL/dindex_q, float32 for pt_f64 = 0,
 * float64 for pt_f64 = 1) plus pt overwritten with index_scale * dL/ds_j.
 * index_dim <= 256. workspace: msa_index_kl_student_workspace_size() bytes. */
size_t msa_index_kl_student_workspace_size(int64_t total_tokens, int32_t groups);
int msa_index_kl_student(const void* index_q, const void* index_k, int dtype, const int32_t* indices,
                         const int32_t* cu_seqlens, int32_t nseq, int64_t total_tokens, int32_t groups,
                         int32_t index_dim, int32_t topk_blocks, int32_t block_size, double index_scale, void* pt,
                         int pt_f64, int need_grad, double* loss, void* d_index_q_acc, void* workspace,
                         size_t workspace_bytes, void* stream);

/* dIK: d_index_k_acc [T][Di] (float32 / float64 as pt) = sum over the pairs that
 * selected key j's block (every group's k2q CSR row, in edge order, the groups'
 * sums added in order; no atomics) of the student step's pt value times
 * index_q[t,g]. total_blocks = the CSR's blocks (cu_block_lens[nseq]).
 * workspace: msa_index_kl_dik_workspace_size() bytes (per-group sums). */
size_t msa_index_kl_dik_workspace_size(int64_t total_tokens, int32_t groups, int32_t index_dim, int pt_f64);
int msa_index_kl_dik(const void* index_q, int dtype, const int32_t* cu_seqlens, const int32_t* cu_block_lens,
                     const int32_t* row_ptr, const int32_t* query_indices, const int32_t* slot_indices,
                     int32_t nseq, int64_t total_tokens, int32_t groups, int32_t index_dim, int32_t topk_blocks,
                     int32_t block_size, int32_t total_blocks, const void* g_pt, int pt_f64,
                     void* d_index_k_acc, void* workspace, size_t workspace_bytes, void* stream);

/* ---------------------------------------------------------------- diagnostics
 * Self-test of the tensor-core building blocks (no counterpart in the
 * reference): one 128 x nw tile per CTA of C = A B. layout bit 0: B stored
 * [K][N] (MN-major), else [N][K]; bit 1: A stored [K][M] (MN-major), else
 * [M][K]; bit 2: nw = 64 (N = 64 per instruction), else 128. bf16/f16 in, f32
 * out; M = 128 m_tiles, N = nw n_tiles, k in {64, 128}. err: device int32, 0
 * on success (nonzero = a bounded wait timed out). */
int msa_selftest_umma(const void* a, const void* b, int dtype, int32_t m_tiles, int32_t n_tiles, int32_t k,
                      int32_t layout, float* c, int32_t* err, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* MSA_B200_H_ */
