/*
 * aoakv.h — C ABI of libaoakv.so, the B200 (sm_100a) sparse-decode path of
 * AOA-KV / Quest: page-metadata append, page-score estimate, top-k page
 * filter and split-KV sparse paged decode.
 *
 * Conventions shared by every entry point
 *   - Pointers are device pointers unless stated otherwise. No torch types.
 *   - KV data and metadata are fp16 and use the reference's NHD paged layout,
 *     one layer slice per call:
 *         kv_data       [kv_capacity_pages, 2, page_size, num_heads, head_dim]
 *         metadata_data [metadata_capacity_pages, 2, page_size, num_heads, head_dim]
 *     Entry j of metadata page m describes KV page m*page_size + j; its K slot
 *     holds the per-channel key maximum, its V slot the per-channel minimum.
 *         v_log_norm    [kv_capacity_pages, num_heads] fp16,
 *                       log(||mean_t V[page, t, head, :]||_2 + 1e-6), written
 *                       when a page becomes full.
 *   - Page ids are int32 physical page ids; every id is range-checked against
 *     the capacity argument. A bad id found on the device does not fault: the
 *     kernel skips it and records AOAKV_DEV_ERR_BAD_PAGE, which
 *     aoakv_get_device_error() returns.
 *   - `stream` is a cudaStream_t (NULL = legacy default stream). Work is
 *     stream-ordered; no entry point synchronises the device or allocates
 *     device memory. Callers own every buffer, including workspaces.
 *   - Return value: AOAKV_OK or an AOAKV_ERR_* code; aoakv_last_error()
 *     returns a message for the calling thread's last failure.
 *   - head_dim must be 64 or 128; layout must be AOAKV_LAYOUT_NHD.
 */
#ifndef AOAKV_H_
#define AOAKV_H_

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define AOAKV_API __attribute__((visibility("default")))
#else
#define AOAKV_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

enum {
  AOAKV_OK = 0,
  AOAKV_ERR_INVALID_ARG = 1,   /* bad shape, size, pointer or flag */
  AOAKV_ERR_UNSUPPORTED = 2,   /* valid but not built (e.g. HND layout) */
  AOAKV_ERR_CUDA = 3,          /* a CUDA runtime call failed */
  AOAKV_ERR_WORKSPACE = 4,     /* workspace missing or too small */
};

/* Device-side error codes (aoakv_get_device_error). */
enum {
  AOAKV_DEV_OK = 0,
  AOAKV_DEV_ERR_BAD_PAGE = 1,  /* a page id outside [0, capacity) was skipped */
  AOAKV_DEV_ERR_TIMEOUT = 2,   /* a bounded device-side wait gave up */
  AOAKV_DEV_ERR_NO_PAGES = 3,  /* a page-table append found no room; the sequence is unchanged */
};

enum { AOAKV_DTYPE_F16 = 0, AOAKV_DTYPE_F32 = 1 };
enum { AOAKV_LAYOUT_NHD = 0, AOAKV_LAYOUT_HND = 1 };
/* score_mode: QUEST = sum_i max(q_i*kmax_i, q_i*kmin_i);
 *             AOAKV = 2*QUEST/sqrt(head_dim) + 2*v_log_norm[page, head]. */
enum { AOAKV_SCORE_QUEST = 0, AOAKV_SCORE_AOAKV = 1 };

/* Message for the calling thread's last non-OK return ("" if none). */
AOAKV_API const char* aoakv_last_error(void);

/* ABI version (major*10000 + minor*100 + patch). */
AOAKV_API int aoakv_version(void);

/* Reads (and with clear != 0 resets) the device-side error word of the
 * current device. Synchronises the current device. */
AOAKV_API int aoakv_get_device_error(int32_t* code_out, int32_t clear);

/* Failure-path check (no reference counterpart): launches one CTA that
 * waits until *flag >= target, bounded by limit_us microseconds, with the
 * same bounded wait the fused step kernels use between phases. If the flag
 * is never raised the wait expires, the kernel records
 * AOAKV_DEV_ERR_TIMEOUT in the device error word and returns; the context
 * stays usable. flag is device memory. */
AOAKV_API int aoakv_debug_wait_flag(const uint32_t* flag, uint32_t target, int32_t limit_us,
                                    void* stream);

/* RoPE — replaces apply_rope_in_place (bsk_ops.h:23-27, page.cu:224-264,
 * kernel decode_page.cuh:786-869). In place on q and k, NHD
 * [seq_len, num_heads, head_dim] fp16: token t at position past_kv_len + t,
 * channel i rotated with its partner i +- head_dim/2 by the angle
 * position * (1/rope_scale) * (1/rope_theta)^(2 (i mod head_dim/2) / head_dim)
 * (rotate-half convention). Angles are evaluated in fp32 with an accurate
 * sine/cosine. */
AOAKV_API int aoakv_apply_rope_in_place(void* q, void* k, int32_t seq_len, int32_t past_kv_len,
                                        int32_t num_heads, int32_t head_dim, float rope_scale,
                                        float rope_theta, void* stream);

/* RMSNorm — replaces rms_norm_forward (bsk_ops.h, ops/csrc/rms_norm.cu;
 * py utils/__init__.py:54-67). Per row of `columns` fp16 values (a
 * multiple of 8): out = x * rsqrt(mean(x^2) + epsilon) * weight, computed
 * in fp32. input, out [rows, columns]; weight [columns]; 16-byte aligned. */
AOAKV_API int aoakv_rms_norm(const void* input, const void* weight, void* out, int32_t rows,
                             int32_t columns, float epsilon, void* stream);

/* a1 — replaces append_kv_cache_decode
 *   (kernels/aoa_kv/quest/ops/csrc/bsk_ops.h:71-86, page.cu:6-105,
 *    kernel decode_page.cuh:392-506).
 * Appends one token k,v [1, num_heads, head_dim] at position
 * (num_kv_pages-1)*page_size + kv_last_page_len - 1, i.e. after the caller
 * has reserved the slot. Updates the last page's running key max/min
 * (initialised to -/+65504 when the token opens a page) and, when the token
 * fills the page, writes v_log_norm[kv_indices[num_kv_pages-1], :].
 * metadata_last_page_len must equal ((num_kv_pages-1) % page_size) + 1 and
 * num_metadata_pages must equal ceil(num_kv_pages / page_size). */
AOAKV_API int aoakv_append_kv_cache_decode(
    const void* k, const void* v,
    void* kv_data, const int32_t* kv_indices, int32_t num_kv_pages,
    int32_t kv_last_page_len, int32_t kv_capacity_pages,
    void* metadata_data, const int32_t* metadata_indices,
    int32_t num_metadata_pages, int32_t metadata_last_page_len,
    int32_t metadata_capacity_pages,
    void* v_log_norm,
    int32_t num_heads, int32_t head_dim, int32_t page_size, int32_t layout,
    void* stream);

/* a2 — replaces append_kv_cache_prefill
 *   (bsk_ops.h:55-69, page.cu:107-222, kernel decode_page.cuh:522-692).
 * Appends seq_len tokens k,v [seq_len, num_heads, head_dim]; they occupy the
 * last seq_len positions of the sequence described by the page table.
 * Every page the tokens touch gets its key max/min merged; every page that
 * ends up full gets its v_log_norm. */
AOAKV_API int aoakv_append_kv_cache_prefill(
    const void* k, const void* v, int32_t seq_len,
    void* kv_data, const int32_t* kv_indices, int32_t num_kv_pages,
    int32_t kv_last_page_len, int32_t kv_capacity_pages,
    void* metadata_data, const int32_t* metadata_indices,
    int32_t num_metadata_pages, int32_t metadata_last_page_len,
    int32_t metadata_capacity_pages,
    void* v_log_norm,
    int32_t num_heads, int32_t head_dim, int32_t page_size, int32_t layout,
    void* stream);

/* a3 — replaces estimate_attn_score
 *   (bsk_ops.h:43-53, estimate.cu:6-90, kernel decode_attn.cuh:263-443 with
 *    compute_max_possible :143-199).
 * Scores the N-1 complete pages (N = (num_metadata_pages-1)*page_size +
 * metadata_last_page_len; the last KV page is excluded) for every head:
 *   out[h * out_row_stride + p], p in [0, N-1), dtype out_dtype.
 * AOAKV mode reads v_log_norm[kv_indices[p], h] (the page's own norm; the
 * reference reads the norm of page kv_indices-of-metadata-page p/page_size,
 * decode_attn.cuh:185-190, which this library does not reproduce).
 * kv_indices NULL means physical page id == logical page id (a fresh
 * reference KvPool allocates pages in that order); QUEST mode ignores it. */
AOAKV_API int aoakv_estimate_attn_score(
    const void* q, void* out, int32_t out_dtype, int64_t out_row_stride,
    const void* metadata_data, const int32_t* metadata_indices,
    int32_t num_metadata_pages, int32_t metadata_last_page_len,
    int32_t metadata_capacity_pages,
    const int32_t* kv_indices, int32_t kv_capacity_pages,
    const void* v_log_norm,
    int32_t num_heads, int32_t head_dim, int32_t page_size, int32_t layout,
    int32_t score_mode, void* stream);

/* a4 — replaces topk_filtering
 *   (bsk_ops.h:35-41, topk.cu:7-46, decode_select_k.cuh:25-61 which runs
 *    RAFT radix_topk_one_block_kernel).
 * For each of num_rows rows selects the k largest of num_pages scores
 * (scores_dtype f16 or f32). Ties break toward the lower position; NaN
 * ranks below every number; -0 equals +0. With sink_first_page != 0
 * position 0 is always selected (the simulation's fixed sink page) and the
 * other k-1 come from positions 1..num_pages-1. Output order: descending
 * score (ties: lower position first) for k <= 256, ascending position for
 * larger k (the reference's order is unspecified):
 *   out_indices[r*out_indices_row_stride + i] = in_indices[r*in_row_stride + pos]
 *   (pos itself when in_indices is NULL; in_row_stride may be 0 to share
 *    one index row), out_values likewise (may be NULL; same dtype as
 *    scores). Requires 1 <= k <= num_pages <= 49152. No scratch buffer. */
AOAKV_API int aoakv_topk_filtering(
    const void* scores, int32_t scores_dtype, int64_t scores_row_stride,
    const int32_t* in_indices, int64_t in_indices_row_stride,
    int32_t num_rows, int32_t num_pages, int32_t k,
    void* out_values, int64_t out_values_row_stride,
    int32_t* out_indices, int64_t out_indices_row_stride,
    int32_t sink_first_page, void* stream);

/* a5 — workspace for aoakv_sparse_decode (replaces the temporary buffers of
 * BatchDecodeHandler::BeginForward, decode_handler.cuh:73-121). The caller
 * allocates it once, zero-fills it once, and may reuse it for every call on
 * one stream; calls keep it zeroed. */
AOAKV_API int aoakv_decode_workspace_size(int32_t num_heads, int32_t head_dim,
                                int32_t max_pages_per_head, size_t* bytes);

/* a5 — replaces BatchDecodeWithPagedKVCachePyTorchWrapper::Forward
 *   (bsk_ops.h:96-125, approx_attn.cu:69-151, kernels decode_attn.cuh:469-688
 *    and :937-1047 plus FlashInfer VariableLengthMergeStates).
 * o[h] = softmax(q[h].K^T * sm_scale) V over head h's num_selected pages
 * indices[h*indices_row_stride + i] (stride 0 shares one row) plus the last
 * page last_page_idx holding last_page_len tokens. q, o: [num_heads,
 * head_dim] fp16. sm_scale <= 0 means 1/sqrt(head_dim). Pages are gathered
 * with TMA; partial softmax states of page chunks merge by log-sum-exp
 * inside the same kernel. */
AOAKV_API int aoakv_sparse_decode(
    const void* q, void* o,
    const void* kv_data, int32_t kv_capacity_pages,
    const int32_t* indices, int64_t indices_row_stride, int32_t num_selected,
    int32_t last_page_idx, int32_t last_page_len,
    int32_t num_heads, int32_t head_dim, int32_t page_size, int32_t layout,
    float sm_scale, void* workspace, size_t workspace_bytes, void* stream);

/* Sparse decode for callers that cannot allocate device memory — no
 * counterpart in the reference. Same inputs, outputs and results as
 * aoakv_sparse_decode, but the partial softmax states of the page chunks go
 * to a fixed 1 MiB array inside the library (one per GPU that loads it, kept
 * until the process exits) instead of a caller workspace. It calls no
 * cudaMalloc/cudaFree. For callers that cannot allocate: a runtime that
 * pre-reserves all device memory for its own pool, a host that gives its
 * plugins no allocator, or a caller that cannot accept the device
 * synchronisation an allocation may cause.
 *   - The first call on each device resolves the array's address
 *     (cudaGetSymbolAddress); make that first call before any stream capture.
 *   - Every call shares the array: calls that overlap on the GPU race, so
 *     serialise them (one stream per device). Each call zeroes the chunk
 *     tickets it needs on its own stream first.
 *   - The partial states, num_heads x chunks x (8 + 4 * head_dim) bytes (a
 *     chunk holds up to 8 pages), must fit 1 MiB: for 32 heads of head_dim
 *     128 that allows num_selected <= 503 pages (about 8,000 tokens at page
 *     size 16). Larger problems return AOAKV_ERR_UNSUPPORTED; use
 *     aoakv_sparse_decode with a workspace. */
AOAKV_API int aoakv_sparse_decode_noalloc(
    const void* q, void* o,
    const void* kv_data, int32_t kv_capacity_pages,
    const int32_t* indices, int64_t indices_row_stride, int32_t num_selected,
    int32_t last_page_idx, int32_t last_page_len,
    int32_t num_heads, int32_t head_dim, int32_t page_size, int32_t layout,
    float sm_scale, void* stream);

/* a5 split across GPUs — the per-GPU half of the reference's split-KV decode
 * (decode_attn.cuh:469-688 writes per-chunk (o, lse) before
 * VariableLengthMergeStates, :1035-1043), for a sequence whose pages are
 * spread over several GPUs by page range. Same inputs as
 * aoakv_sparse_decode, but:
 *   - an index of -1 means "not on this GPU" and is skipped;
 *   - last_page_idx may be -1 when another GPU owns the last page;
 *   - outputs are this GPU's partial state: o_partial [num_heads, head_dim]
 *     fp32 (normalised over this GPU's tokens) and lse [num_heads] fp32
 *     (natural log of the sum of exp(scaled scores)); a head with no tokens
 *     here gets o_partial = 0 and lse = -inf.
 * Combine the parts with aoakv_merge_states. */
AOAKV_API int aoakv_sparse_decode_partial(
    const void* q, float* o_partial, float* lse,
    const void* kv_data, int32_t kv_capacity_pages,
    const int32_t* indices, int64_t indices_row_stride, int32_t num_selected,
    int32_t last_page_idx, int32_t last_page_len,
    int32_t num_heads, int32_t head_dim, int32_t page_size, int32_t layout,
    float sm_scale, void* workspace, size_t workspace_bytes, void* stream);

/* Log-sum-exp merge of num_parts partial states (the math of FlashInfer's
 * VariableLengthMergeStates, call site decode_attn.cuh:1035-1043):
 * o_parts [num_parts, num_heads, head_dim] fp32 and lse_parts
 * [num_parts, num_heads] fp32 -> o [num_heads, head_dim] fp16 and, if
 * lse_out is not NULL, the merged lse [num_heads] fp32. */
AOAKV_API int aoakv_merge_states(const float* o_parts, const float* lse_parts,
                                 int32_t num_parts, int32_t num_heads, int32_t head_dim,
                                 void* o, float* lse_out, void* stream);

/* Page-range sharding helper (no reference counterpart: the reference runs
 * on one GPU): out[i] = local_kv_indices[global_ids[i] - page_lo] when the
 * global page id lies in [page_lo, page_lo + n_local), else -1 (the page is
 * on another GPU), for count ids. */
AOAKV_API int aoakv_map_pages(const int32_t* global_ids, int64_t count, int32_t page_lo,
                              int32_t n_local, const int32_t* local_kv_indices, int32_t* out,
                              void* stream);

/* Whole per-layer decode step for one request: a1 append of (k_new, v_new),
 * a3 estimate, a4 top-k and a5 sparse decode, as the reference's
 * QuestAttention.forward decode branch issues them
 * (kernels/aoa_kv/quest/models/QuestAttention.py:99-157).
 * num_kv_pages / kv_last_page_len describe the sequence INCLUDING the new
 * token. page_budget counts pages including the always-attended last page:
 *   sink_first_page == 0 (kernel-tree rule, controller.py:124, utils:237):
 *       k = min(page_budget, N); top-(k-1) of pages 0..N-2, plus page N-1.
 *   sink_first_page != 0 (simulation rule, filter_util.py:226-231,373-377):
 *       k = min(max(3, page_budget), N); page 0, top-(k-2) of 1..N-2, N-1.
 *   If N <= k every page is attended and no scoring runs.
 * selected_out (optional, [num_heads, B] with B = page_budget, or
 * max(3, page_budget) with the sink) receives the attended page ids per head:
 * slot 0 the sink page (with the sink), then the selected pages (descending
 * score when one kernel runs the step, ascending page otherwise), slot k-1
 * the last page; unused slots are -1.
 * The workspace (used only when the step runs as a chain of kernels, see
 * aoakv_step_plan_info) is sized by aoakv_step_workspace_size, zero-filled
 * once by the caller, and kept zeroed by every call. */
AOAKV_API int aoakv_step_workspace_size(int32_t num_heads, int32_t head_dim,
                              int32_t max_pages, int32_t max_page_budget,
                              size_t* bytes);

/* The step planned once per layer — replaces BatchDecodeHandler's
 * BeginForward / Forward / EndForward (decode_handler.cuh:73-136,
 * approx_attn.cu:27-151), which re-plan with a device synchronisation and an
 * allocation on every step. aoakv_step_plan_create binds one layer's
 * kv_data / metadata_data / v_log_norm and the step's parameters, chooses how
 * the step runs on the current device (one launch of thread-block clusters
 * when head_dim is 64 or 128 and page_size <= 16, else the four-kernel chain)
 * and encodes its tensor maps; it allocates host memory only.
 *   max_pages  the largest num_kv_pages the plan will run (0 = capacity);
 *              shared memory is sized for it.
 *   max_ctas   0 = the whole GPU, else at most this many CTAs per step (so
 *              several requests' steps can share the GPU).
 *   flags      AOAKV_PLAN_CHAIN forces the four-kernel chain;
 *              AOAKV_PLAN_SHARD sizes the plan for aoakv_shard_* (a page
 *              range of a longer sequence: up to page_budget attended
 *              pages even when max_pages is smaller).
 * aoakv_step_plan_run runs one step (arguments as aoakv_decode_step) on the
 * device the plan was created on; it does not synchronise, allocate or
 * re-plan. Plans are immutable: one plan may serve several streams. */
enum { AOAKV_PLAN_CHAIN = 1, AOAKV_PLAN_SHARD = 2 };
typedef struct aoakv_step_plan_s* aoakv_step_plan;

AOAKV_API int aoakv_step_plan_create(aoakv_step_plan* plan_out, void* kv_data,
                                     int32_t kv_capacity_pages, void* metadata_data,
                                     int32_t metadata_capacity_pages, void* v_log_norm,
                                     int32_t num_heads, int32_t head_dim, int32_t page_size,
                                     int32_t page_budget, int32_t score_mode,
                                     int32_t sink_first_page, int32_t max_pages,
                                     int32_t max_ctas, int32_t flags);
AOAKV_API int aoakv_step_plan_run(aoakv_step_plan plan, const void* q, const void* k_new,
                                  const void* v_new, void* o, const int32_t* kv_indices,
                                  int32_t num_kv_pages, int32_t kv_last_page_len,
                                  const int32_t* metadata_indices, int32_t* selected_out,
                                  void* workspace, size_t workspace_bytes, void* stream);
/* *kernels_out: launches per step for num_kv_pages pages (1 = one cluster
 * launch; 2 append + decode or 4 append, estimate, top-k, decode for the
 * chain, plus 1 with selected_out); *cluster_out: CTAs per head of the
 * cluster launch (0 = chain). Either may be NULL. */
AOAKV_API int aoakv_step_plan_info(aoakv_step_plan plan, int32_t num_kv_pages,
                                   int32_t want_selected, int32_t* kernels_out,
                                   int32_t* cluster_out);
AOAKV_API int aoakv_step_plan_destroy(aoakv_step_plan plan);
/* RoPE fused into the plan's step (the reference applies it as its own op
 * just before the append, utils/__init__.py:25-52 / decode_page.cuh:786-869):
 * with rope_scale > 0, aoakv_step_plan_run takes q and k_new unrotated,
 * rotates both at the new token's position ((num_kv_pages - 1) * page_size +
 * kv_last_page_len - 1) exactly as aoakv_apply_rope_in_place does (same
 * bits), uses them, and leaves the rotated q and k_new in place.
 * rope_scale <= 0 turns it off (the default). Not used by the shard passes
 * or the batched step. Call it between steps, not while one runs. */
AOAKV_API int aoakv_step_plan_set_rope(aoakv_step_plan plan, float rope_scale,
                                       float rope_theta);

/* One sequence split over GPUs by page range (config 5's 128K-token decode;
 * the reference runs it on one GPU only). GPU g holds global pages
 * [page_lo, page_lo + num_local_pages) through its own layer pools and page
 * tables (page_lo a multiple of page_size, so metadata pages are never
 * split); the GPU holding page num_total_pages - 1 owns the last page. Per
 * layer and token every GPU runs, with its own plan (created with
 * AOAKV_PLAN_SHARD, max_pages >= num_local_pages + 1 and the whole
 * sequence's page_budget):
 *   1 aoakv_shard_propose: scores its pages and writes its best k-1
 *     (k = min(budget, num_total_pages), the budget rule of
 *     aoakv_decode_step) to cand_out [num_heads, k-1] as {uint32 order key,
 *     uint32 global page id}, best first (ties: lower page), unused entries
 *     {0, 0xffffffff}. Only when num_total_pages > k > 1.
 *   2 an all_gather of cand_out into cand_all [world, num_heads, k-1]
 *     (rank order);
 *   3 aoakv_shard_finish: ranks its entries against the other GPUs', decodes
 *     the winners it holds and, on the owner, the last page after appending
 *     k_new, v_new to it (the append and metadata update of
 *     aoakv_append_kv_cache_decode); writes its partial state
 *     state_out [num_heads, head_dim + 1] fp32 = {o normalised over its
 *     tokens, lse = ln(sum exp(scaled scores))}, {0, -inf} for no tokens.
 *     cand_all may be NULL when no selection runs (every page attended, or
 *     only the last). selected_out (optional, [num_heads, k-1]) receives the
 *     whole selection's global page ids, best first;
 *   4 an all_gather of state_out into states [world, num_heads, head_dim+1];
 *   5 aoakv_merge_packed_states: the log-sum-exp merge into o [num_heads,
 *     head_dim] fp16 (the same output on every GPU).
 * The global selection equals the one-GPU step's: each GPU's k-1 best
 * contain its share of the global k-1 best. Limits: world <= 8,
 * world * (k-1) <= 2048. The plan must run the cluster kernel
 * (AOAKV_ERR_UNSUPPORTED otherwise). */
AOAKV_API int aoakv_shard_propose(aoakv_step_plan plan, const void* q,
                                  const int32_t* kv_indices, int32_t num_local_pages,
                                  int32_t num_total_pages, int32_t page_lo,
                                  const int32_t* metadata_indices, void* cand_out,
                                  void* stream);
AOAKV_API int aoakv_shard_finish(aoakv_step_plan plan, const void* q, const void* k_new,
                                 const void* v_new, const int32_t* kv_indices,
                                 int32_t num_local_pages, int32_t num_total_pages,
                                 int32_t page_lo, int32_t kv_last_page_len,
                                 const int32_t* metadata_indices, const void* cand_all,
                                 int32_t world, int32_t rank, float* state_out,
                                 int32_t* selected_out, void* stream);
AOAKV_API int aoakv_merge_packed_states(const float* states, int32_t num_parts,
                                        int32_t num_heads, int32_t head_dim, void* o,
                                        void* stream);

/* The same three passes with the two exchanges done by the kernels
 * themselves (no collective library): each GPU owns a mailbox in its own
 * memory, mapped into every other GPU's address space (CUDA IPC, NVLink
 * peer access). The propose pass stores each head's list straight into every
 * GPU's mailbox; the finish pass reads every GPU's lists from its own
 * mailbox, ranks, decodes and stores its partial state into every mailbox the
 * same way; the merge reads the states and writes o. Every 64-bit word
 * travels with the number of the exchange it belongs to (a single-copy-
 * atomic store of {value, epoch}), and a reader waits on the words it needs
 * until they carry the current number, so no fence or flag is needed; the
 * wait is bounded (AOAKV_DEV_ERR_TIMEOUT, never a hang). Per layer and token:
 *   aoakv_shard_propose_p2p (only when a selection runs, as above),
 *   aoakv_shard_finish_p2p, aoakv_shard_merge_p2p(with_proposals = whether
 *   the propose pass ran).
 * Every GPU must run the same passes in the same order. One mailbox serves
 * all layers of a sequence (each pass completes its exchange before the
 * next layer's can start on another GPU).
 * Setup, once per process group: aoakv_shard_mailbox_create allocates and
 * zero-fills this GPU's mailbox (it synchronises the device) and writes its
 * 64-byte IPC handle; the caller all-gathers the handles (rank order) and
 * passes them to aoakv_shard_mailbox_connect. Destroy only after every GPU
 * has finished its last pass (a host barrier). max_proposals bounds k-1. */
typedef struct aoakv_shard_mailbox_s* aoakv_shard_mailbox;
AOAKV_API int aoakv_shard_mailbox_create(aoakv_shard_mailbox* mb_out, int32_t world,
                                         int32_t rank, int32_t num_heads, int32_t head_dim,
                                         int32_t max_proposals, void* ipc_handle_out);
AOAKV_API int aoakv_shard_mailbox_connect(aoakv_shard_mailbox mb, const void* ipc_handles);
AOAKV_API int aoakv_shard_mailbox_destroy(aoakv_shard_mailbox mb);
AOAKV_API int aoakv_shard_propose_p2p(aoakv_step_plan plan, aoakv_shard_mailbox mb,
                                      const void* q, const int32_t* kv_indices,
                                      int32_t num_local_pages, int32_t num_total_pages,
                                      int32_t page_lo, const int32_t* metadata_indices,
                                      void* stream);
AOAKV_API int aoakv_shard_finish_p2p(aoakv_step_plan plan, aoakv_shard_mailbox mb,
                                     const void* q, const void* k_new, const void* v_new,
                                     const int32_t* kv_indices, int32_t num_local_pages,
                                     int32_t num_total_pages, int32_t page_lo,
                                     int32_t kv_last_page_len, const int32_t* metadata_indices,
                                     int32_t* selected_out, void* stream);
AOAKV_API int aoakv_shard_merge_p2p(aoakv_shard_mailbox mb, int32_t with_proposals, void* o,
                                    void* stream);

/* aoakv_step_plan_info for a problem without a plan (the default plan). */
AOAKV_API int aoakv_step_launches(int32_t num_heads, int32_t head_dim, int32_t page_size,
                                  int32_t num_kv_pages, int32_t page_budget,
                                  int32_t sink_first_page, int32_t want_selected,
                                  int32_t* kernels_out);

/* One step without a plan (plans it on every call). */
AOAKV_API int aoakv_decode_step(
    const void* q, const void* k_new, const void* v_new, void* o,
    void* kv_data, const int32_t* kv_indices, int32_t num_kv_pages,
    int32_t kv_last_page_len, int32_t kv_capacity_pages,
    void* metadata_data, const int32_t* metadata_indices,
    int32_t metadata_capacity_pages,
    void* v_log_norm,
    int32_t num_heads, int32_t head_dim, int32_t page_size,
    int32_t page_budget, int32_t score_mode, int32_t sink_first_page,
    int32_t* selected_out, void* workspace, size_t workspace_bytes,
    void* stream);

/* aoakv_decode_step on at most max_ctas CTAs (0 = the whole GPU; no
 * reference counterpart): several independent requests' steps can run
 * concurrently on separate streams; results are the same. */
AOAKV_API int aoakv_decode_step_grid(
    const void* q, const void* k_new, const void* v_new, void* o, void* kv_data,
    const int32_t* kv_indices, int32_t num_kv_pages, int32_t kv_last_page_len,
    int32_t kv_capacity_pages, void* metadata_data, const int32_t* metadata_indices,
    int32_t metadata_capacity_pages, void* v_log_norm, int32_t num_heads,
    int32_t head_dim, int32_t page_size, int32_t page_budget, int32_t score_mode,
    int32_t sink_first_page, int32_t* selected_out, void* workspace,
    size_t workspace_bytes, int32_t max_ctas, void* stream);

/* Paged prefill attention (ops/csrc/batch_prefill.cu:27-116,
 * prefill_with_paged_kv_cache; kernel include/prefill/prefill.cuh:688-1119):
 * one sequence of qo_len new tokens, q and o [qo_len, num_qo_heads,
 * head_dim] fp16, attending the layer's paged KV (NHD pages
 * [kv_capacity_pages, 2, page_size, num_kv_heads, head_dim]) of kv_len =
 * (num_kv_pages - 1) * page_size + kv_last_page_len tokens, whose K/V
 * already include the new tokens. Query i sits at position kv_len - qo_len +
 * i; causal != 0 lets it attend KV tokens j <= i + kv_len - qo_len (needs
 * qo_len <= kv_len). Query head h reads KV head h / (num_qo_heads /
 * num_kv_heads). sm_scale <= 0 means 1/sqrt(head_dim). lse (optional,
 * [qo_len, num_qo_heads] fp32) receives each row's natural-log
 * log-sum-exp of the scaled scores. head_dim 64 or 128; page_size 8, 16,
 * 32, 64 or 128. One launch on the tcgen05 tensor cores (accumulators in
 * tensor memory); no workspace, no allocation, no synchronisation. The
 * reference's rope_scale / rope_theta arguments are not taken: it runs this
 * kernel with RoPE off (RotaryMode::kNone, batch_prefill.cu:96). */
AOAKV_API int aoakv_prefill_paged(
    const void* q, void* o, float* lse, const void* kv_data, int32_t kv_capacity_pages,
    const int32_t* kv_indices, int32_t num_kv_pages, int32_t kv_last_page_len, int32_t qo_len,
    int32_t num_qo_heads, int32_t num_kv_heads, int32_t head_dim, int32_t page_size,
    int32_t layout, int32_t causal, float sm_scale, void* stream);

/* Grouped-query attention (GQA; the reference's CUDA tree is MHA only,
 * docs/KERNEL_DIFF.md:66-76): the step of aoakv_decode_step for
 * num_qo_heads query heads sharing num_kv_heads KV heads (num_qo_heads a
 * multiple of num_kv_heads, at most 16 query heads per KV head; query head h
 * reads KV head h / (num_qo_heads / num_kv_heads)). Group-consistent
 * selection as in filtering/filter_util.py: each KV head scores its pages
 * once for its whole group — QUEST sums the group's page bounds (:219-221),
 * AOAKV takes the logsumexp over the group of 2*bound/sqrt(head_dim) and
 * adds 2*v_log_norm (:352-361, :367) — and every query head of the group
 * attends the same pages. q, o: [num_qo_heads, head_dim]; k_new, v_new,
 * the caches and v_log_norm use num_kv_heads; selected_out (optional) is
 * [num_kv_heads, B] as for aoakv_decode_step. Runs as four launches
 * (append, group scoring, top-k, decode); the workspace is
 * aoakv_step_workspace_size(num_qo_heads, ...). */
AOAKV_API int aoakv_decode_step_gqa(
    const void* q, const void* k_new, const void* v_new, void* o, void* kv_data,
    const int32_t* kv_indices, int32_t num_kv_pages, int32_t kv_last_page_len,
    int32_t kv_capacity_pages, void* metadata_data, const int32_t* metadata_indices,
    int32_t metadata_capacity_pages, void* v_log_norm, int32_t num_qo_heads,
    int32_t num_kv_heads, int32_t head_dim, int32_t page_size, int32_t page_budget,
    int32_t score_mode, int32_t sink_first_page, int32_t* selected_out, void* workspace,
    size_t workspace_bytes, void* stream);

/* Batched decode step (config 4's single launch; no reference counterpart:
 * the reference hard-wires batch 1, decode_attn.cuh:504-509): the step of
 * aoakv_decode_step for num_requests requests whose pages live in ONE layer
 * pool, as one launch over (request, head). Request r's KV pages are
 * kv_indices[kv_indptr[r] .. kv_indptr[r+1]) (the reference's paged_kv_t
 * indptr convention, decode_page.cuh:79-352), its metadata pages start at
 * metadata_indices[metadata_indptr[r]], its last page holds
 * kv_last_page_len[r] tokens (all device arrays, the new token included).
 * q, k_new, v_new, o are [num_requests, num_heads, head_dim]; selected_out
 * (optional) is [num_requests, num_heads, B] as for aoakv_decode_step.
 * max_pages bounds every request's page count (shared memory is sized for
 * it); a request with no pages, more than max_pages pages or a last page
 * length outside [1, page_size] is skipped and AOAKV_DEV_ERR_BAD_PAGE is
 * recorded. Needs head_dim 64/128 and page_size <= 16; no workspace. */
AOAKV_API int aoakv_decode_step_batched(
    const void* q, const void* k_new, const void* v_new, void* o, void* kv_data,
    int32_t kv_capacity_pages, const int32_t* kv_indptr, const int32_t* kv_indices,
    const int32_t* kv_last_page_len, void* metadata_data, int32_t metadata_capacity_pages,
    const int32_t* metadata_indptr, const int32_t* metadata_indices, void* v_log_norm,
    int32_t num_requests, int32_t max_pages, int32_t num_heads, int32_t head_dim,
    int32_t page_size, int32_t page_budget, int32_t score_mode, int32_t sink_first_page,
    int32_t* selected_out, void* stream);

/* ------------------------------------------------ device-resident page table
 * The reference keeps the page table on the host (quest/utils/kv_cache.py:
 * 7-133 KvPool / KvCache, controller.py:82-141 rebuilding index tensors from
 * Python lists every step). Here one device buffer holds, for num_seqs
 * sequences, each sequence's KV page list (room for max_pages_per_seq) and
 * metadata page list (room for ceil(max_pages_per_seq / page_size)), its
 * page count, last-page length and token count, and the free stacks of the
 * KV pool (kv_capacity_pages) and metadata pool (metadata_capacity_pages).
 * Pages are allocated on the device, so a whole decode token (append +
 * every layer's step) can be captured as one CUDA graph and replayed. The
 * caller owns the buffer (aoakv_page_table_bytes bytes, 16-byte aligned). */
typedef struct aoakv_page_table_s* aoakv_page_table;

AOAKV_API int aoakv_page_table_bytes(int32_t num_seqs, int32_t max_pages_per_seq,
                                     int32_t kv_capacity_pages, int32_t metadata_capacity_pages,
                                     int32_t page_size, size_t* bytes);
/* Initialises the buffer on `stream` (every sequence empty, both pools
 * free; a fresh pool hands out page ids 0, 1, 2, ... like the reference's
 * fresh set) and returns a host handle. */
AOAKV_API int aoakv_page_table_create(aoakv_page_table* table_out, int32_t num_seqs,
                                      int32_t max_pages_per_seq, int32_t kv_capacity_pages,
                                      int32_t metadata_capacity_pages, int32_t page_size,
                                      void* device_buffer, size_t buffer_bytes, void* stream);
AOAKV_API int aoakv_page_table_destroy(aoakv_page_table table);
/* KvCache.append_seq (kv_cache.py:115-126) + the metadata append of
 * controller.py:82-87 on the device, one launch: num_tokens more tokens for
 * sequence seq (-1: every sequence, in order). A new KV page when the last
 * page is full or the sequence is empty; a new metadata page every
 * page_size KV pages. A sequence that would exceed its room or a pool is
 * left unchanged and AOAKV_DEV_ERR_NO_PAGES is recorded. */
AOAKV_API int aoakv_page_table_append(aoakv_page_table table, int32_t seq, int32_t num_tokens,
                                      void* stream);
/* KvCache.release (kv_cache.py:128-133): the sequence's pages (seq -1:
 * every sequence) go back to the pools, last page first, so they are handed
 * out again in their old order. */
AOAKV_API int aoakv_page_table_release(aoakv_page_table table, int32_t seq, void* stream);
/* Word offsets (int32) of the buffer's regions: [0] KV free-stack height,
 * [1] metadata free-stack height, [2] kv_start[R], [3] kv_end[R] (sequence
 * r's KV pages are kv_indices[kv_start[r] .. kv_end[r])), [4] last_len[R],
 * [5] seq_len[R], [6] meta_start[R], [7] meta_count[R], [8] kv_indices,
 * [9] metadata_indices, [10] KV free stack, [11] metadata free stack,
 * [12] total words, [13] R, [14] max_pages_per_seq, [15] metadata pages per
 * sequence. */
AOAKV_API int aoakv_page_table_layout(aoakv_page_table table, int64_t* words);
/* aoakv_decode_step_batched over the table's sequences: sequence r's page
 * count, last-page length and page lists are read on the device, so the
 * call can be captured in a CUDA graph and replayed after
 * aoakv_page_table_append(table, -1, 1) for every token. q, k_new, v_new, o
 * are [num_seqs, num_heads, head_dim] (the new token already counted by the
 * append); an empty sequence is skipped. Same limits as the batched step.
 * rope_scale > 0 fuses RoPE as aoakv_step_plan_set_rope does: q and k_new
 * arrive unrotated, each sequence's pair is rotated at that sequence's
 * new-token position (read on the device) and left rotated in place;
 * rope_scale <= 0: no RoPE. */
AOAKV_API int aoakv_decode_step_table(
    aoakv_page_table table, const void* q, const void* k_new, const void* v_new, void* o,
    void* kv_data, int32_t kv_capacity_pages, void* metadata_data,
    int32_t metadata_capacity_pages, void* v_log_norm, int32_t num_heads, int32_t head_dim,
    int32_t page_budget, int32_t score_mode, int32_t sink_first_page, int32_t* selected_out,
    float rope_scale, float rope_theta, void* stream);

#ifdef __cplusplus
}  /* extern "C" */
#endif

#endif  /* AOAKV_H_ */
