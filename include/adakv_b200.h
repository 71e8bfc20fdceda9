/*
 * adakv_b200.h -- C ABI of the B200 (sm_100a) AdaKV decode hot path.
 *
 * One decode step of AdaKV (query-aware, per-head-adaptive block-sparse
 * attention) runs as hand-written CUDA kernels behind these entry points:
 *
 *   adakv_centroid_build   per-block key centroids after prefill        (a)
 *   adakv_kv_append        in-place KV append + trailing-centroid refresh (a)
 *   adakv_centroid_refresh trailing-centroid refresh of a caller-grown cache (a)
 *   adakv_plan             q.centroid estimator, entropy budget, top-k  (b)(c)
 *   adakv_attend           ragged block-sparse split-KV flash decode    (d)
 *   adakv_decode_step      adakv_plan followed by adakv_attend          (b)-(d)
 *   adakv_minmax_build / adakv_minmax_refresh / adakv_estimate_minmax
 *                          the minmax (Quest) estimator                 (b')
 *   adakv_estimate / adakv_select / adakv_attend_partial / adakv_combine
 *                          the same step split for a sequence sharded over GPUs (e)
 *   adakv_shard_prep / adakv_shard_clamp / adakv_shard_finish
 *                          its selection from exchanged statistics (e)
 *   adakv_peer_*           all-gather through peer-mapped memory (e)
 *
 * Conventions
 *   - Every function returns ADAKV_OK (0) or an error code; the message of
 *     the last error on the calling thread is returned by adakv_last_error().
 *     Arguments are validated on the host before anything is launched.
 *   - Pointers are device pointers unless stated otherwise.  No call
 *     allocates device memory: scratch lives in a caller-provided workspace
 *     (size from adakv_*_workspace_bytes, zero-filled once before first use;
 *     it keeps no state a later call depends on beyond call counters).
 *     Calls that share a workspace must be ordered on one stream.  The
 *     exceptions: adakv_attend_noalloc's scratch, a fixed 4 MiB __device__
 *     array of the library, present on every device the library's device
 *     code is loaded on (4 MiB of device memory each), whether or not that
 *     entry point is ever called; and adakv_peer_alloc, the one-time
 *     set-up of a multi-GPU exchange buffer, which calls cudaMalloc.
 *   - Inputs (q, K/V, centroids, seq_lens, tables) must be complete when the
 *     call is enqueued: the decode kernels use programmatic dependent launch
 *     and some of them read their inputs before waiting for the previous
 *     kernel on the stream to finish, so a producer of those inputs must not
 *     itself be a kernel that triggers its dependents early (before its last
 *     write).  The one-kernel adakv_decode_step reads nothing before that wait.
 *   - All work is enqueued on `stream` (a cudaStream_t passed as void*); no
 *     function synchronises the host except adakv_read_status.
 *   - Tensors are [batch, heads, tokens, head_dim] views described by
 *     adakv_view; head_dim must be contiguous and each row 16-byte aligned.
 *   - q/K/V/out share one element type (adakv_geometry.dtype); centroids and
 *     scores are float32.
 *
 * Reference interfaces replaced (paths inside the adakv project):
 *   adakv/attention.py:119-139  AdaKVCache.append_prefill   -> adakv_centroid_build
 *   adakv/runtime.py:43-60      update_cache_decode         -> adakv_kv_append
 *   adakv/baselines_rt.py:43-81 h2o/snapkv_key_importance_torch -> adakv_key_importance
 *   adakv/attention.py:141-146  AdaKVCache.append_decode    -> adakv_kv_append
 *   adakv/attention.py:149-247  plan_selection              -> adakv_plan
 *   adakv/kernels/block_sparse_decode.py:103-135 block_sparse_decode -> adakv_attend
 *   adakv/attention.py:250-268  adakv_decode_attention      -> adakv_decode_step
 *   adakv/runtime.py:85-112     adakv_decode_step           -> adakv_decode_step
 */
#ifndef ADAKV_B200_H_
#define ADAKV_B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define ADAKV_B200_ABI_VERSION 2

/* element types of q / K / V / out */
#define ADAKV_DTYPE_F32 0
#define ADAKV_DTYPE_F16 1
#define ADAKV_DTYPE_BF16 2

/* budget policies (adakv/budget.py:45-86) */
#define ADAKV_POLICY_FIXED 0    /* every head gets round(target) blocks           */
#define ADAKV_POLICY_ADAPTIVE 1 /* surplus split by normalised score entropy       */
#define ADAKV_POLICY_NUCLEUS 2  /* surplus split by the blocks holding nucleus_p of
                                   the softmax mass (budget.py:38-41)              */

/* return codes */
#define ADAKV_OK 0
#define ADAKV_ERR_INVALID 1     /* bad argument (reference: ValueError / assert)   */
#define ADAKV_ERR_UNSUPPORTED 2 /* valid but not built (e.g. head_dim 96)          */
#define ADAKV_ERR_CUDA 3        /* a CUDA runtime call failed                      */

/* device status bits (adakv_read_status) */
#define ADAKV_ST_WAIT_TIMEOUT 1u /* a bounded device wait gave up                   */
#define ADAKV_ST_BAD_BLOCK_ID 2u /* a block table entry was outside [0, nb)        */
#define ADAKV_ST_BAD_SEL_LEN 4u  /* sel_lens[h] exceeded the table width          */
#define ADAKV_ST_BAD_SEQ_LEN 8u  /* seq_lens[b] outside [1, max_seq_len]           */

/* Problem geometry.  One decode query token per sequence. */
typedef struct adakv_geometry {
  int32_t batch;       /* B sequences                                        */
  int32_t n_q_heads;   /* Hq                                                 */
  int32_t n_kv_heads;  /* Hkv; Hq % Hkv == 0, Hq / Hkv <= 16                 */
  int32_t head_dim;    /* D: 64 or 128                                       */
  int32_t block_size;  /* tokens per block: 16 or 32                         */
  int32_t max_seq_len; /* host-side bound of every seq_lens[b]               */
  int32_t nb_cap;      /* block capacity of the centroid table, >= ceil(max_seq_len / block_size) */
  int32_t dtype;       /* ADAKV_DTYPE_*                                      */
} adakv_geometry;

/* A [B, H, S, D] tensor view (element strides; the D stride is 1). */
typedef struct adakv_view {
  void* data;
  int64_t stride_b;
  int64_t stride_h;
  int64_t stride_s; /* ignored for q and out */
} adakv_view;

/* Selection knobs, named and defaulted as plan_selection
 * (adakv/attention.py:149-162): avg_budget, k_min=2, k_max=64,
 * n_sink_blocks=1, n_local_blocks=4, c_min=1, temperature=1.0,
 * policy=ADAKV_POLICY_ADAPTIVE, nucleus_p=0.9. */
typedef struct adakv_select_params {
  double avg_budget;
  double temperature;
  int32_t k_min;
  int32_t k_max;
  int32_t n_sink_blocks;
  int32_t n_local_blocks;
  int32_t c_min;
  int32_t policy;
  double nucleus_p; /* ADAKV_POLICY_NUCLEUS: cumulative mass target (0.9)   */
} adakv_select_params;

/* ABI version of the loaded library (ADAKV_B200_ABI_VERSION). */
int adakv_abi_version(void);

/* Message of the last failed call on this thread ("" if none). */
const char* adakv_last_error(void);

/* Width of the block table adakv_plan writes: the largest per-head count
 * this geometry and these knobs can produce (plan_selection's max_sel without
 * the host sync of adakv/attention.py:242). */
int32_t adakv_plan_table_width(const adakv_geometry* geo, const adakv_select_params* sp);

/* Workspace bytes for adakv_plan / adakv_decode_step. */
size_t adakv_plan_workspace_bytes(const adakv_geometry* geo, const adakv_select_params* sp);

/* Workspace bytes for a stand-alone adakv_attend over a table of `table_width`. */
size_t adakv_attend_workspace_bytes(const adakv_geometry* geo, int32_t table_width);

/* Centroid table from a prefilled cache (adakv/attention.py:119-139,
 * oracle adakv/estimator.py:27-48): centroid[b, h, j, :] = mean of the keys of
 * block j over its real tokens, float32, summed in token order.
 * k: [B, Hkv, S, D]; centroid: [B, Hkv, nb_cap, D] float32 contiguous;
 * seq_lens: [B] int32 device array or NULL (every sequence max_seq_len). */
int adakv_centroid_build(const adakv_geometry* geo, const adakv_view* k, const int32_t* seq_lens,
                         float* centroid, void* stream);

/* Append n_new tokens per sequence in place and refresh the centroids of every
 * block they touch (adakv/runtime.py:43-60, without the full-cache torch.cat).
 * seq_lens[b] is the length AFTER the append; the new tokens land at
 * [seq_lens[b] - n_new, seq_lens[b]).  k_new/v_new: [B, Hkv, n_new, D]. */
int adakv_kv_append(const adakv_geometry* geo, const adakv_view* k_cache, const adakv_view* v_cache,
                    const adakv_view* k_new, const adakv_view* v_new, int32_t n_new,
                    const int32_t* seq_lens, float* centroid, void* stream);

/* Recompute the centroids of every block touched by the last n_new tokens of
 * each sequence, reading the cache only (the tokens were already written by
 * the caller, e.g. a HuggingFace DynamicCache).  Same numerics as
 * adakv_centroid_build on those blocks. */
int adakv_centroid_refresh(const adakv_geometry* geo, const adakv_view* k, int32_t n_new,
                           const int32_t* seq_lens, float* centroid, void* stream);

/* Block selection for one decode query per sequence (adakv/attention.py:149-247):
 * scores = q . centroid (GQA folded, unscaled), per-head budget from the
 * normalised entropy of softmax(scores / T) with the mean pinned to
 * avg_budget, sink/local blocks forced, top-k of the rest (ties -> lowest
 * block index).  Writes block_table[(b*Hq + h) * table_width + i] for
 * i < sel_lens[b*Hq + h] in ascending block order.  scores_out (nullable):
 * [B, Hq, nb_cap] float32 copy of the block scores. */
int adakv_plan(const adakv_geometry* geo, const adakv_select_params* sp, const adakv_view* q,
               const float* centroid, const int32_t* seq_lens, int32_t* block_table,
               int32_t table_width, int32_t* sel_lens, float* scores_out, void* workspace,
               size_t workspace_bytes, void* stream);

/* Ragged block-sparse decode attention over a given table
 * (adakv/kernels/block_sparse_decode.py:103-135): out[b, h] = softmax over the
 * tokens of the listed blocks of (q . k) * sm_scale, times V; tokens at or past
 * seq_lens[b] are masked.  Rows with sel_lens 0 produce zeros. */
int adakv_attend(const adakv_geometry* geo, const adakv_view* q, const adakv_view* k,
                 const adakv_view* v, const int32_t* block_table, int32_t table_width,
                 const int32_t* sel_lens, const int32_t* seq_lens, float sm_scale,
                 const adakv_view* out, void* workspace, size_t workspace_bytes, void* stream);

/* ---- minmax (Quest) estimator (adakv/estimator.py:50-57, 76-79;
 *      adakv/attention.py:134-138, 190-198) ----
 * kmin / kmax: [B, Hkv, nb_cap, D] float32 per-block per-dimension key minima
 * and maxima over the real tokens.  Scores
 * sum_d max(q_d, 0) kmax_d + min(q_d, 0) kmin_d go to a caller buffer; the
 * selection then runs through adakv_select and the attention through
 * adakv_attend. */
int adakv_minmax_build(const adakv_geometry* geo, const adakv_view* k, const int32_t* seq_lens,
                       float* kmin, float* kmax, void* stream);

/* Recompute the tables of the blocks touched by the last n_new tokens. */
int adakv_minmax_refresh(const adakv_geometry* geo, const adakv_view* k, int32_t n_new,
                         const int32_t* seq_lens, float* kmin, float* kmax, void* stream);

/* scores[(b * Hq + h) * score_stride + j] for every block j of every sequence. */
int adakv_estimate_minmax(const adakv_geometry* geo, const adakv_view* q, const float* kmin,
                          const float* kmax, const int32_t* seq_lens, float* scores,
                          int32_t score_stride, void* stream);

/* adakv_attend without a workspace: no counterpart in the reference.
 *
 * For callers that cannot hand over device memory: a serving engine that has
 * given all free memory to its KV-cache pool, or a host language with no
 * device allocator at hand.  The scratch (status word, selection bitmaps,
 * split-KV partials, arrival counters) is a fixed 4 MiB array inside this
 * library, one per device; a call needs exactly
 * adakv_attend_workspace_bytes(geo, table_width) bytes of it, and a geometry
 * needing more than 4 MiB is rejected with ADAKV_ERR_INVALID (batch 1 at 128K
 * tokens, 32 q / 8 KV heads, D 128, needs about 0.33 MiB).  Nothing is
 * allocated on the device by the call.  The first call on each device looks the array up (and may load
 * the library's device code): make that first call before any stream capture.
 * The scratch is shared, so two calls in flight at once on one device (other
 * streams, other threads) race and corrupt each other; order them on one
 * stream.  `status` (optional device word, may be NULL) receives this call's
 * ADAKV_ST_* bits, overwritten each call.  Same inputs and output as
 * adakv_attend. */
int adakv_attend_noalloc(const adakv_geometry* geo, const adakv_view* q, const adakv_view* k,
                         const adakv_view* v, const int32_t* block_table, int32_t table_width,
                         const int32_t* sel_lens, const int32_t* seq_lens, float sm_scale,
                         const adakv_view* out, uint32_t* status, void* stream);

/* One full decode step with no host synchronisation anywhere
 * (adakv/attention.py:250-268, adakv/runtime.py:85-112, adakv/runtime.py:43-60):
 * optionally append n_new tokens per sequence (k_new / v_new [B, Hkv, n_new, D];
 * n_new = 0 and NULL views to skip; seq_lens[b] is the length AFTER the append)
 * into k / v in place with the touched centroids refreshed, then adakv_plan,
 * then attention of every query head over its selection, written to out.
 * The workspace is sized by adakv_plan_workspace_bytes.  By default the step
 * is three PDL-chained kernels (estimator, plan, attend); with ADAKV_FUSED=1
 * in the environment (read once) it is one persistent kernel where that
 * kernel applies (adaptive or fixed policy, B * Hq <= 128, head_dim 128,
 * g = 4 or 8, block 16); both give the same selection. */
int adakv_decode_step(const adakv_geometry* geo, const adakv_select_params* sp,
                      const adakv_view* q, const adakv_view* k, const adakv_view* v,
                      const adakv_view* k_new, const adakv_view* v_new, int32_t n_new,
                      float* centroid, const int32_t* seq_lens, float sm_scale,
                      int32_t* block_table, int32_t table_width, int32_t* sel_lens,
                      const adakv_view* out, void* workspace, size_t workspace_bytes,
                      void* stream);

/* Per-key attention importance of the H2O / SnapKV eviction baselines
 * (adakv/baselines.py:69-117, adakv/baselines_rt.py:43-81): the last n_query
 * prompt query rows (n_query = S: H2O's accumulated attention; the
 * observation window: SnapKV, before its max-pool) attend causally to the S
 * keys with scale sm_scale, and
 *   importance[(b * Hq + h) * imp_stride + j] = sum over those rows i >= j of
 *   softmax_i(j), float32, j < S = max_seq_len.
 * q: [B, Hq, S, D] views; k: [B, Hkv, S, D] (read per KV head, not expanded);
 * the workspace holds the rows' softmax maxima and sums
 * (adakv_importance_workspace_bytes).  O(S * n_query * D) work, run once per
 * prompt; deterministic (no atomics). */
size_t adakv_importance_workspace_bytes(const adakv_geometry* geo, int32_t n_query);
int adakv_key_importance(const adakv_geometry* geo, const adakv_view* q, const adakv_view* k,
                         int32_t n_query, float sm_scale, float* importance, int32_t imp_stride,
                         void* workspace, size_t workspace_bytes, void* stream);

/* Synchronise `stream`, copy the workspace's device status word (ADAKV_ST_*
 * bits) to *status and clear it. */
int adakv_read_status(void* workspace, uint32_t* status, void* stream);

/* Let the kernels that use `workspace` also write their ADAKV_ST_* bits to
 * `host_word`, a page-locked host word mapped into the device address space
 * (cudaHostAlloc / cudaHostRegister with mapping; NULL detaches).  A host
 * can then notice a failed step without synchronising: the word stays 0
 * until some kernel reports.  Synchronises `stream` once (set-up call).
 * No counterpart in the reference (its errors are host exceptions). */
int adakv_set_status_sink(void* workspace, uint32_t* host_word, void* stream);

/* Copy `bytes` from `src` (device memory, or page-locked host memory mapped
 * into the device's address space) to device memory `dst` on `stream`, with a
 * kernel that reads the source directly.  Meant for a decode step's few KB of
 * inputs (q and the new K / V rows) arriving from the host: for transfers this
 * small a copy-engine transfer's fixed cost dominates (about 11 us for a 12 KB
 * row on B200), while the kernel finishes in a few us.  Both addresses 16-byte
 * aligned.  No counterpart in the reference (its inputs are torch tensors). */
int adakv_stage(void* dst, const void* src, size_t bytes, void* stream);

/* Block scores (q . centroid, float32, unscaled) of the last adakv_plan or
 * adakv_decode_step enqueued on `workspace`, into
 * scores_out[(b * Hq + h) * score_stride + j] for j < ceil(max_seq_len / block_size).
 * The scores the reference's plan_selection computes
 * (adakv/attention.py:187-189), for inspection and tests. */
int adakv_read_scores(const adakv_geometry* geo, void* workspace, size_t workspace_bytes,
                      float* scores_out, int32_t score_stride, void* stream);

/* How the last adakv_plan / adakv_decode_step enqueued on `workspace` ran:
 * 0 nothing yet, 1 as the estimator / plan / attend kernel chain (three
 * launches; adakv_plan: two), 2 as the one-kernel decode step.  Host-side
 * bookkeeping, no device access. */
int adakv_last_path(const void* workspace);

/* Test-only knobs, process-wide, all off (0) by default.  No counterpart in
 * the reference.
 *   ADAKV_KNOB_WAIT_NS    bound of every bounded device wait, in ns (0: 200 ms)
 *   ADAKV_KNOB_FLAGS      bit 0: the entropy of query head 0 of sequence 0 is
 *                         never published, so the per-sequence exchange of the
 *                         budget waits out its bound (failure-detection tests)
 *   ADAKV_KNOB_STEP_PATH  adakv_decode_step: 0 runs the three-kernel chain
 *                         (or the one-kernel step where it applies when the
 *                         environment has ADAKV_FUSED=1), 1 forces the chain,
 *                         2 picks the one-kernel step wherever it applies
 *   ADAKV_KNOB_STEP_CLUSTER  largest thread-block cluster (1, 2, 4 or 8 CTAs)
 *                         one query head's selection may span in the one-kernel
 *                         step (0: 8) */
#define ADAKV_KNOB_WAIT_NS 1
#define ADAKV_KNOB_FLAGS 2
#define ADAKV_KNOB_STEP_PATH 3
#define ADAKV_KNOB_STEP_CLUSTER 4
int adakv_debug_knob(int32_t knob, int64_t value);

/* Test-only: with ADAKV_KNOB_FLAGS bit 1 set, the one-kernel step records per
 * CTA 24 words, globaltimer stamps (ns; 0 where the CTA has no such phase).
 * Word: 0 start, 1 estimator done, 2 score slice and row statistics ready,
 * 3 budget weights known, 4 bitmap and table published, 5 group bitmaps
 * read, 6 attention partial published, 7 end, 8 / 9 first / last estimator
 * stage arrived, 10 every estimator CTA arrived, 11 entropy published,
 * 12 cluster candidates visible, 13 gather and MMA done, 14 candidates
 * ranked, 15 unused, 16 histogram and clamp pass done, 17 cluster
 * histograms visible, 18 cluster counts visible, 19 estimator records
 * folded, 20 threshold bucket found, 21 bitmap words marked, 22 union list
 * built, 23 warp partials combined.  adakv_b200.step_timeline prints them.
 * Synchronises `stream`, copies max_ctas * 24 words of the last step on
 * `workspace` to the host array `out`.  No counterpart in the
 * reference. */
int adakv_debug_timeline(const adakv_geometry* geo, void* workspace, size_t workspace_bytes,
                         uint64_t* out, int32_t max_ctas, void* stream);

/* ---- sequence-sharded decode (one sequence's blocks split over GPUs) ----
 * The reference decodes one sequence on one device; these four calls split
 * its steps so that a long sequence can be sharded by contiguous blocks:
 * each rank scores its shard (adakv_estimate, the block scoring of
 * adakv/estimator.py:62-74), the ranks all-gather the score rows, every rank
 * selects on the full rows (adakv_select, adakv/budget.py:45-86 +
 * adakv/selector.py:18-60; identical tables everywhere), attends over the
 * blocks it holds (adakv_attend_partial) and the per-rank outputs are merged
 * by their log-sum-exp (adakv_combine).  Collectives are the caller's. */

/* Block scores q . centroid of every block of the cache described by `geo`
 * into scores[(b * Hq + h) * score_stride + j] (float32, unscaled).
 * Workspace: adakv_plan_workspace_bytes(geo, any params). */
int adakv_estimate(const adakv_geometry* geo, const adakv_view* q, const float* centroid,
                   const int32_t* seq_lens, float* scores, int32_t score_stride, void* workspace,
                   size_t workspace_bytes, void* stream);

/* Entropy budget + top-k over caller-given score rows (the layout written by
 * adakv_estimate; `geo` describes the whole sequence).  Outputs as adakv_plan. */
int adakv_select(const adakv_geometry* geo, const adakv_select_params* sp, const float* scores,
                 int32_t score_stride, const int32_t* seq_lens, int32_t* block_table,
                 int32_t table_width, int32_t* sel_lens, void* workspace, size_t workspace_bytes,
                 void* stream);

/* Attention of every query head over the selected blocks that this cache
 * holds: `block_table` lists global block ids, the cache (`geo`, k, v,
 * seq_lens) holds global blocks [block_offset, block_offset + nb); other ids
 * are skipped.  Writes the normalised output out_f32[b * Hq + h][D] (float32)
 * and lse[b * Hq + h] = log sum over the attended tokens of
 * exp(q . k * sm_scale) (-inf when the head attends to nothing here).
 * Workspace: adakv_attend_workspace_bytes(geo, table_width). */
int adakv_attend_partial(const adakv_geometry* geo, const adakv_view* q, const adakv_view* k,
                         const adakv_view* v, const int32_t* block_table, int32_t table_width,
                         const int32_t* sel_lens, int32_t block_offset, const int32_t* seq_lens,
                         float sm_scale, float* out_f32, float* lse, void* workspace,
                         size_t workspace_bytes, void* stream);

/* out[b, h] = sum_n exp(lse[n][r] - LSE) parts[n][r][:] with r = b * Hq + h
 * and LSE = log sum_n exp(lse[n][r]); rows with every lse = -inf get zeros.
 * parts: [n_parts, batch * n_q_heads, head_dim] float32; lse: [n_parts, rows]. */
int adakv_combine(int32_t n_parts, int32_t batch, int32_t n_q_heads, int32_t head_dim,
                  int32_t dtype, const float* parts, const float* lse, const adakv_view* out,
                  void* stream);

/* adakv_combine over parts packed the way adakv_attend_partial's outputs
 * travel in one collective: part n at packed + n * part_stride holds
 * out_f32 [batch * Hq][D] followed by lse [batch * Hq] (part_stride >=
 * batch * Hq * (D + 1) floats). */
int adakv_combine_packed(int32_t n_parts, int32_t batch, int32_t n_q_heads, int32_t head_dim,
                         int32_t dtype, const float* packed, int64_t part_stride,
                         const adakv_view* out, void* stream);

/* ---- sequence-sharded selection from exchanged statistics ----
 * Replaces the score-row all-gather + adakv_select above for the fixed and
 * adaptive policies (adakv/budget.py:45-86, adakv/selector.py:18-60 over the
 * whole row), exchanging per head only softmax statistics, a sorted list of
 * the shard's top content candidates and one clamp term:
 *   1. adakv_shard_prep     this shard's record (statistics + candidates);
 *   2. all-gather the records (rank order);
 *   3. adakv_shard_clamp    this shard's clamp terms (adaptive policy only);
 *   4. all-gather the clamp terms (float64 [world][Hq]);
 *   5. adakv_shard_finish   every head's budget and this rank's table rows:
 *      the global ids of the selected blocks this shard holds.
 * The union of the ranks' rows is the head's selection; every rank derives
 * the same budgets.  `geo` describes the whole sequence (batch 1, no
 * seq_lens: max_seq_len tokens); shard blocks are [block_lo,
 * block_lo + n_local) and `scores` this shard's rows [Hq][score_stride]
 * (adakv_estimate's layout).  Collectives are the caller's. */

/* Bytes of one rank's record; 0 when the path does not apply (batch != 1,
 * nucleus policy, more than 4096 candidates per head). */
size_t adakv_shard_record_bytes(const adakv_geometry* geo, const adakv_select_params* sp);

int adakv_shard_prep(const adakv_geometry* geo, const adakv_select_params* sp, const float* scores,
                     int32_t score_stride, int32_t block_lo, int32_t n_local, void* record,
                     void* stream);

/* cc[Hq] float64; `records`: world records, record_stride bytes apart. */
int adakv_shard_clamp(const adakv_geometry* geo, const adakv_select_params* sp, const float* scores,
                      int32_t score_stride, int32_t block_lo, int32_t n_local, const void* records,
                      size_t record_stride, int32_t world, double* cc, void* stream);

/* block_table [Hq][table_width] (table_width >= adakv_plan_table_width),
 * sel_lens [Hq]; cc_all may be NULL for the fixed policy; status: optional
 * device word for ADAKV_ST_* bits. */
int adakv_shard_finish(const adakv_geometry* geo, const adakv_select_params* sp,
                       const void* records, size_t record_stride, const double* cc_all,
                       int32_t world, int32_t rank, int32_t block_lo, int32_t n_local,
                       int32_t* block_table, int32_t table_width, int32_t* sel_lens,
                       uint32_t* status, void* stream);

/* ---- all-gather of small payloads through peer-mapped memory ----
 * The sharded step's exchanges (records, clamp terms, partial outputs) are
 * 0.5 KB - 0.5 MB; an NCCL all-gather of that size costs about 11 us inside
 * a CUDA graph on two B200s.  These calls move them with NVLink stores into
 * every rank's buffer instead (no counterpart in the reference, which runs
 * on one device).  Set-up, once per buffer and process (these synchronise
 * and allocate; do it before any stream capture):
 *   adakv_peer_alloc   cudaMalloc of adakv_peer_buffer_bytes(world,
 *                      slot_bytes), zeroed, and its 64-byte IPC handle;
 *   share the handles between the ranks (the caller's collective);
 *   adakv_peer_open    map another rank's buffer here (its own: use ptr);
 *   adakv_peer_close / adakv_peer_free at the end.
 * adakv_peer_exchange then copies `bytes` of `src` into slot `rank` of every
 * rank's buffer (dsts: device array [world] of the mapped pointers, own
 * included) and waits, bounded, until every rank's payload has arrived in
 * `local`; slot r of `local` then holds rank r's payload.  Every rank calls
 * it the same number of times on the same buffer; a payload must have been
 * consumed everywhere before the next exchange on that buffer starts (the
 * sharded step's order guarantees this).  On an expired wait the status word
 * gets ADAKV_ST_WAIT_TIMEOUT and the call returns. */
size_t adakv_peer_buffer_bytes(int32_t world, size_t slot_bytes);
int adakv_peer_alloc(size_t bytes, void** ptr, void* handle);
int adakv_peer_free(void* ptr);
int adakv_peer_open(const void* handle, void** ptr);
int adakv_peer_close(void* ptr);
int adakv_peer_exchange(const void* src, size_t bytes, void* const* dsts, int32_t world,
                        int32_t rank, size_t slot_bytes, void* local, uint32_t* status,
                        void* stream);

#ifdef __cplusplus
}
#endif

#endif /* ADAKV_B200_H_ */
