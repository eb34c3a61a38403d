// Per-layer decode step for one request: append -> estimate -> top-k ->
// sparse decode, stream-ordered, with no host synchronisation and no
// allocation; planned once per layer (aoakv_step_plan_*), run per token.
//
// Reference call order: kernels/aoa_kv/quest/models/QuestAttention.py:99-157
// (append_kv, then need_estimate() ? estimate + topk + sparse decode : decode
// over every page), with the page budget of controller.py:118-127 and
// utils/__init__.py:237 (top-(k-1) plus the last page) or, with the sink,
// filtering/filter_util.py:226-231 and :373-377 (page 0 and the last page
// forced, k = min(max(3, budget), N)). The plan replaces the reference's
// BatchDecodeHandler begin/forward/end (decode_handler.cuh:73-136,
// approx_attn.cu:27-151), which re-plans with a device synchronisation and
// an allocation on every step.
//
// Two ways to run a step:
//   cluster  one launch of step_cluster.cu (the default whenever the shape
//            fits: head_dim 64/128, page_size <= 16);
//   chain    append, estimate, top-k and decode as four launches with
//            programmatic dependent launch (other shapes, or on request).
#include <cmath>
#include <cstring>
#include <new>

#include "decode.cuh"
#include "estimate.cuh"
#include "page_table.h"
#include "plan.h"
#include "step_cluster.h"
#include "topk.cuh"

// The opaque plan behind aoakv_step_plan.
struct aoakv_step_plan_s {
  int device;
  int H, D, P;
  void* kv;
  int kv_cap;
  void* meta;
  int meta_cap;
  void* vlog;
  int budget, mode, sink, max_pages;
  bool cluster_ok;               // the cluster kernel runs this layer
  aoakv::ClusterPlan cp;
  CUtensorMap kv_sw;             // cluster: K/V tiles, 128-byte swizzle
  CUtensorMap meta_map;          // cluster: metadata tiles
  CUtensorMap kv_plain;          // chain: the decode kernel's K/V boxes
  bool rope;                     // RoPE fused into the step (aoakv_step_plan_set_rope)
  float rope_scale, rope_theta;
};

namespace aoakv {
namespace {

// selected_out[h, i]: slot i's page id, the last page after the selected
// ones, -1 beyond.
__global__ void fill_selected_kernel(int32_t* out, int budget, const int32_t* idx,
                                     int64_t idx_stride, int n_sel,
                                     const int32_t* last_ptr, int H) {
  pdl_wait();
  const int h = blockIdx.x;
  for (int i = threadIdx.x; i < budget; i += blockDim.x) {
    int v = -1;
    if (i < n_sel)
      v = __ldcg(idx + static_cast<size_t>(h) * idx_stride + i);
    else if (i == n_sel)
      v = __ldcg(last_ptr);
    out[static_cast<size_t>(h) * budget + i] = v;
  }
}

// Chain workspace: [decode partials][fp32 scores][selected ids]. The decode
// tickets must be zero between calls (zeroed once; the kernels re-arm them).
struct StepWs {
  size_t dec_off, scores_off, idx_off, total;
};

StepWs step_ws_layout(int H, int D, int max_pages, int max_budget) {
  auto up = [](size_t x) { return (x + 255) / 256 * 256; };
  const int max_slots = max_budget < 3 ? 3 : max_budget;
  StepWs w;
  size_t off = 0;
  w.dec_off = off;
  off += up(decode_ws_bytes(H, D, max_slots));
  w.scores_off = off;
  off += up(static_cast<size_t>(H) * max_pages * 4);
  w.idx_off = off;
  off += up(static_cast<size_t>(H) * max_slots * 4);
  w.total = off;
  return w;
}

// Pages attended per head: k_pages from the budget rule, k = min(k_pages, N).
void step_budget(int N, int budget, int sink, int* k_pages, int* k) {
  *k_pages = sink ? (budget < 3 ? 3 : budget) : budget;
  *k = *k_pages < N ? *k_pages : N;
}

int check_plan_args(int H, int D, int P, int kv_cap, int meta_cap, int budget, int mode) {
  int rc = check_decode_shape(H, D, P, kv_cap, AOAKV_LAYOUT_NHD);
  if (rc) return rc;
  AOAKV_CHECK_ARG(budget >= 1, "step: page_budget must be >= 1");
  AOAKV_CHECK_ARG(mode == AOAKV_SCORE_QUEST || mode == AOAKV_SCORE_AOAKV,
                  "step: score_mode must be QUEST or AOAKV");
  AOAKV_CHECK_ARG(meta_cap >= (kv_cap + P - 1) / P,
                  "step: metadata capacity below ceil(kv_capacity_pages / page_size)");
  return AOAKV_OK;
}

// Fills *p (no allocation): the launch shape, kernel attributes and tensor
// maps of one layer.
int plan_init(aoakv_step_plan_s* p, void* kv, int kv_cap, void* meta, int meta_cap, void* vlog,
              int H, int D, int P, int budget, int mode, int sink, int max_pages, int max_ctas,
              int flags) {
  AOAKV_CHECK_ARG(kv && meta && vlog, "step plan: NULL buffer");
  int rc = check_plan_args(H, D, P, kv_cap, meta_cap, budget, mode);
  if (rc) return rc;
  AOAKV_CHECK_ARG(max_pages >= 0 && max_pages <= kv_cap,
                  "step plan: max_pages must be in [0, kv_capacity_pages]");
  AOAKV_CHECK_ARG(max_ctas >= 0, "step plan: max_ctas must be >= 0");
  AOAKV_CHECK_ARG((flags & ~(AOAKV_PLAN_CHAIN | AOAKV_PLAN_SHARD)) == 0,
                  "step plan: unknown flag");
  AOAKV_CUDA_TRY(cudaGetDevice(&p->device), "step plan: cudaGetDevice");
  p->H = H;
  p->D = D;
  p->P = P;
  p->kv = kv;
  p->kv_cap = kv_cap;
  p->meta = meta;
  p->meta_cap = meta_cap;
  p->vlog = vlog;
  p->budget = budget;
  p->mode = mode;
  p->sink = sink != 0;
  p->max_pages = max_pages ? max_pages : kv_cap;
  int k_pages, k;
  step_budget(p->max_pages, budget, p->sink, &k_pages, &k);
  p->cluster_ok = !(flags & AOAKV_PLAN_CHAIN) &&
                  cluster_step_plan(H, D, P, p->max_pages, k_pages, max_ctas, &p->cp,
                                    (flags & AOAKV_PLAN_SHARD) != 0);
  if (p->cluster_ok) {
    rc = make_kv_tmap_sw128(&p->kv_sw, kv, H, D, P, kv_cap);
    if (rc) return rc;
    rc = make_kv_tmap(&p->meta_map, meta, H, D, P, meta_cap);
    if (rc) return rc;
  }
  return make_kv_tmap(&p->kv_plain, kv, H, D, P, kv_cap);
}

int run_cluster(const aoakv_step_plan_s* p, const void* q, const void* k_new, const void* v_new,
                void* o, const int32_t* kv_indices, int N, int last_len,
                const int32_t* meta_indices, int32_t* selected_out, int k_pages, int k,
                cudaStream_t s) {
  ClusterStepArgs a = {};
  a.q = static_cast<const __half*>(q);
  a.k_new = static_cast<const __half*>(k_new);
  a.v_new = static_cast<const __half*>(v_new);
  a.o = static_cast<__half*>(o);
  a.kv = static_cast<__half*>(p->kv);
  a.kv_indices = kv_indices;
  a.n_pages = N;
  a.last_len = last_len;
  a.kv_cap = p->kv_cap;
  a.meta = static_cast<__half*>(p->meta);
  a.meta_indices = meta_indices;
  a.meta_cap = p->meta_cap;
  a.vlog = static_cast<__half*>(p->vlog);
  a.H = p->H;
  a.P = p->P;
  a.k_slots = k;
  a.sink = p->sink;
  a.mode = p->mode;
  a.two_rsqrt_d = 2.f / std::sqrt(static_cast<float>(p->D));
  a.scale_log2 = (1.f / std::sqrt(static_cast<float>(p->D))) * 1.4426950408889634f;
  a.selected_out = selected_out;
  a.sel_cols = k_pages;
  a.err = dev_error_ptr();
  if (p->rope) {
    a.rope = 1;
    a.rope_pos = (N - 1) * p->P + last_len - 1;
    a.rope_rcp_scale = 1.f / p->rope_scale;
    a.rope_log2_rcp_theta = std::log2(1.f / p->rope_theta);
  }
  return launch_cluster_step(a, p->kv_sw, p->meta_map, p->D, p->cp, s);
}

int run_chain(const aoakv_step_plan_s* p, const void* q, const void* k_new, const void* v_new,
              void* o, const int32_t* kv_indices, int N, int last_len,
              const int32_t* meta_indices, int32_t* selected_out, void* workspace,
              size_t workspace_bytes, int k_pages, int k, cudaStream_t s) {
  const int H = p->H, D = p->D, P = p->P;
  const bool sparse = N > k && k > 1;  // k == 1 keeps only the last page: nothing to score
  AOAKV_CHECK_ARG(!sparse || N - 1 <= kTopkMaxN, "step: more than 49153 pages");
  const StepWs lay = step_ws_layout(H, D, N, k_pages);
  AOAKV_CHECK_ARG(workspace != nullptr, "step: workspace is NULL");
  if (workspace_bytes < lay.total)
    return set_error(AOAKV_ERR_WORKSPACE,
                     "step: workspace smaller than aoakv_step_workspace_size(...) = " +
                         std::to_string(lay.total));
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  const int n_meta = (N + P - 1) / P;
  if (p->rope) {  // q and k_new rotated in place at the new token's position first
    const int rc0 = aoakv_apply_rope_in_place(const_cast<void*>(q), const_cast<void*>(k_new), 1,
                                              (N - 1) * P + last_len - 1, H, D, p->rope_scale,
                                              p->rope_theta, s);
    if (rc0) return rc0;
  }
  int rc = aoakv_append_kv_cache_decode(k_new, v_new, p->kv, kv_indices, N, last_len, p->kv_cap,
                                        p->meta, meta_indices, n_meta, (N - 1) % P + 1,
                                        p->meta_cap, p->vlog, H, D, P, AOAKV_LAYOUT_NHD, s);
  if (rc) return rc;
  DecodeArgs da = {};
  da.q = static_cast<const __half*>(q);
  da.o = static_cast<__half*>(o);
  da.last_len = last_len;
  da.last_page_ptr = kv_indices + (N - 1);
  da.H = H;
  da.P = P;
  da.kv_cap = p->kv_cap;
  da.scale_log2 = (1.f / std::sqrt(static_cast<float>(D))) * 1.4426950408889634f;
  da.err = dev_error_ptr();
  int32_t* sel_idx = reinterpret_cast<int32_t*>(ws + lay.idx_off);
  if (sparse) {
    EstimateArgs ea;
    ea.q = static_cast<const __half*>(q);
    ea.meta = static_cast<const __half*>(p->meta);
    ea.meta_indices = meta_indices;
    ea.kv_indices = kv_indices;
    ea.vlog = static_cast<const __half*>(p->vlog);
    ea.out = ws + lay.scores_off;
    ea.out_stride = N;
    ea.out_f32 = 1;
    ea.n_score = N - 1;
    ea.H = H;
    ea.P = P;
    ea.meta_cap = p->meta_cap;
    ea.kv_cap = p->kv_cap;
    ea.mode = p->mode;
    ea.two_rsqrt_d = 2.f / std::sqrt(static_cast<float>(D));
    ea.err = da.err;
    rc = launch_estimate(ea, D, s);
    if (rc) return rc;
    TopkArgs ta;
    ta.scores = ws + lay.scores_off;
    ta.s_stride = N;
    ta.in_idx = kv_indices;
    ta.in_stride = 0;
    ta.out_vals = nullptr;
    ta.ov_stride = 0;
    ta.out_idx = sel_idx;
    ta.oi_stride = k - 1;
    ta.f32 = 1;
    ta.n = N - 1;
    ta.k = k - 1;
    ta.sink = p->sink;
    rc = launch_topk(ta, H, s, true);
    if (rc) return rc;
    da.indices = sel_idx;
    da.idx_stride = k - 1;
    da.n_sel = k - 1;
  } else {
    da.indices = kv_indices;
    da.idx_stride = 0;
    da.n_sel = N > k ? 0 : N - 1;  // k == 1: last page only; else every page
  }
  const DecodePlan pl = plan_decode(H, da.n_sel + 1, D, P);
  da.chunk_pages = pl.chunk_pages;
  da.n_chunks = pl.n_chunks;
  carve_decode_ws(ws + lay.dec_off, H, D, da.n_sel + 1, da);
  rc = launch_decode(da, p->kv_plain, D, pl, s, sparse);
  if (rc) return rc;
  if (selected_out) {
    fill_selected_kernel<<<H, 128, 0, s>>>(selected_out, k_pages, da.indices, da.idx_stride,
                                           da.n_sel, da.last_page_ptr, H);
    AOAKV_CUDA_TRY(cudaGetLastError(), "fill_selected launch");
  }
  return AOAKV_OK;
}

int plan_run(const aoakv_step_plan_s* p, const void* q, const void* k_new, const void* v_new,
             void* o, const int32_t* kv_indices, int N, int last_len,
             const int32_t* meta_indices, int32_t* selected_out, void* workspace,
             size_t workspace_bytes, void* stream) {
  AOAKV_NVTX("aoakv_decode_step");
  AOAKV_CHECK_ARG(q && k_new && v_new && o && kv_indices && meta_indices,
                  "step: NULL pointer argument");
  AOAKV_CHECK_ARG(N >= 1 && N <= p->max_pages,
                  "step: num_kv_pages must be in [1, the plan's max_pages]");
  AOAKV_CHECK_ARG(last_len >= 1 && last_len <= p->P,
                  "step: kv_last_page_len must be in [1, page_size]");
  int k_pages, k;
  step_budget(N, p->budget, p->sink, &k_pages, &k);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (p->cluster_ok)
    return run_cluster(p, q, k_new, v_new, o, kv_indices, N, last_len, meta_indices,
                       selected_out, k_pages, k, s);
  return run_chain(p, q, k_new, v_new, o, kv_indices, N, last_len, meta_indices, selected_out,
                   workspace, workspace_bytes, k_pages, k, s);
}

// Kernels one step launches: 1 (cluster), else the chain's count.
int plan_kernels(const aoakv_step_plan_s* p, int N, bool want_selected) {
  if (p->cluster_ok) return 1;
  int k_pages, k;
  step_budget(N, p->budget, p->sink, &k_pages, &k);
  const bool sparse = N > k && k > 1;
  return (sparse ? 4 : 2) + (want_selected ? 1 : 0);
}

}  // namespace
}  // namespace aoakv

using namespace aoakv;

namespace aoakv {
namespace {

// The GQA step: append (KV heads), group scoring, top-k per KV head, decode
// per query head from its KV head's pages; stream-ordered with programmatic
// dependent launch like the chain.
int run_gqa(const void* q, const void* k_new, const void* v_new, void* o, void* kv,
            const int32_t* kv_indices, int N, int last_len, int kv_cap, void* meta,
            const int32_t* meta_indices, int meta_cap, void* vlog, int Hq, int Hk, int D,
            int P, int budget, int mode, int sink, int32_t* selected_out, void* workspace,
            size_t workspace_bytes, cudaStream_t s) {
  AOAKV_CHECK_ARG(q && k_new && v_new && o && kv && kv_indices && meta && meta_indices && vlog,
                  "step_gqa: NULL pointer argument");
  AOAKV_CHECK_ARG(Hk >= 1 && Hq >= Hk && Hq % Hk == 0 && Hq / Hk <= 16,
                  "step_gqa: num_qo_heads must be a multiple (1 to 16) of num_kv_heads");
  int rc = check_plan_args(Hk, D, P, kv_cap, meta_cap, budget, mode);
  if (rc) return rc;
  AOAKV_CHECK_ARG(N >= 1 && N <= kv_cap && last_len >= 1 && last_len <= P,
                  "step_gqa: bad num_kv_pages or kv_last_page_len");
  const int group = Hq / Hk;
  int k_pages, k;
  step_budget(N, budget, sink, &k_pages, &k);
  const bool sparse = N > k && k > 1;
  AOAKV_CHECK_ARG(!sparse || N - 1 <= kTopkMaxN, "step_gqa: more than 49153 pages");
  const StepWs lay = step_ws_layout(Hq, D, N, k_pages);
  AOAKV_CHECK_ARG(workspace != nullptr, "step_gqa: workspace is NULL");
  if (workspace_bytes < lay.total)
    return set_error(AOAKV_ERR_WORKSPACE,
                     "step_gqa: workspace smaller than aoakv_step_workspace_size(num_qo_heads, "
                     "...) = " + std::to_string(lay.total));
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  rc = aoakv_append_kv_cache_decode(k_new, v_new, kv, kv_indices, N, last_len, kv_cap, meta,
                                    meta_indices, (N + P - 1) / P, (N - 1) % P + 1, meta_cap,
                                    vlog, Hk, D, P, AOAKV_LAYOUT_NHD, s);
  if (rc) return rc;
  DecodeArgs da = {};
  da.q = static_cast<const __half*>(q);
  da.o = static_cast<__half*>(o);
  da.last_len = last_len;
  da.last_page_ptr = kv_indices + (N - 1);
  da.H = Hq;
  da.P = P;
  da.kv_cap = kv_cap;
  da.group = group;
  da.scale_log2 = (1.f / std::sqrt(static_cast<float>(D))) * 1.4426950408889634f;
  da.err = dev_error_ptr();
  int32_t* sel_idx = reinterpret_cast<int32_t*>(ws + lay.idx_off);
  if (sparse) {
    EstimateArgs ea = {};
    ea.q = static_cast<const __half*>(q);
    ea.meta = static_cast<const __half*>(meta);
    ea.meta_indices = meta_indices;
    ea.kv_indices = kv_indices;
    ea.vlog = static_cast<const __half*>(vlog);
    ea.out = ws + lay.scores_off;
    ea.out_stride = N;
    ea.out_f32 = 1;
    ea.n_score = N - 1;
    ea.H = Hk;
    ea.P = P;
    ea.meta_cap = meta_cap;
    ea.kv_cap = kv_cap;
    ea.mode = mode;
    ea.two_rsqrt_d = 2.f / std::sqrt(static_cast<float>(D));
    ea.err = da.err;
    rc = launch_gqa_estimate(ea, D, group, s);
    if (rc) return rc;
    TopkArgs ta;
    ta.scores = ws + lay.scores_off;
    ta.s_stride = N;
    ta.in_idx = kv_indices;
    ta.in_stride = 0;
    ta.out_vals = nullptr;
    ta.ov_stride = 0;
    ta.out_idx = sel_idx;
    ta.oi_stride = k - 1;
    ta.f32 = 1;
    ta.n = N - 1;
    ta.k = k - 1;
    ta.sink = sink;
    rc = launch_topk(ta, Hk, s, true);
    if (rc) return rc;
    da.indices = sel_idx;
    da.idx_stride = k - 1;
    da.n_sel = k - 1;
  } else {
    da.indices = kv_indices;
    da.idx_stride = 0;
    da.n_sel = N > k ? 0 : N - 1;
  }
  CUtensorMap tmap;
  rc = make_kv_tmap(&tmap, kv, Hk, D, P, kv_cap);
  if (rc) return rc;
  const DecodePlan pl = plan_decode(Hq, da.n_sel + 1, D, P);
  da.chunk_pages = pl.chunk_pages;
  da.n_chunks = pl.n_chunks;
  carve_decode_ws(ws + lay.dec_off, Hq, D, da.n_sel + 1, da);
  rc = launch_decode(da, tmap, D, pl, s, sparse);
  if (rc) return rc;
  if (selected_out) {
    fill_selected_kernel<<<Hk, 128, 0, s>>>(selected_out, k_pages, da.indices, da.idx_stride,
                                            da.n_sel, da.last_page_ptr, Hk);
    AOAKV_CUDA_TRY(cudaGetLastError(), "fill_selected launch");
  }
  return AOAKV_OK;
}

}  // namespace
}  // namespace aoakv

extern "C" int aoakv_decode_step_gqa(
    const void* q, const void* k_new, const void* v_new, void* o, void* kv_data,
    const int32_t* kv_indices, int32_t num_kv_pages, int32_t kv_last_page_len,
    int32_t kv_capacity_pages, void* metadata_data, const int32_t* metadata_indices,
    int32_t metadata_capacity_pages, void* v_log_norm, int32_t num_qo_heads,
    int32_t num_kv_heads, int32_t head_dim, int32_t page_size, int32_t page_budget,
    int32_t score_mode, int32_t sink_first_page, int32_t* selected_out, void* workspace,
    size_t workspace_bytes, void* stream) {
  AOAKV_NVTX("aoakv_decode_step_gqa");
  return run_gqa(q, k_new, v_new, o, kv_data, kv_indices, num_kv_pages, kv_last_page_len,
                 kv_capacity_pages, metadata_data, metadata_indices, metadata_capacity_pages,
                 v_log_norm, num_qo_heads, num_kv_heads, head_dim, page_size, page_budget,
                 score_mode, sink_first_page != 0, selected_out, workspace, workspace_bytes,
                 static_cast<cudaStream_t>(stream));
}

extern "C" int aoakv_step_workspace_size(int32_t num_heads, int32_t head_dim,
                                         int32_t max_pages, int32_t max_page_budget,
                                         size_t* bytes) {
  AOAKV_CHECK_ARG(bytes != nullptr, "step_workspace_size: bytes is NULL");
  AOAKV_CHECK_ARG(num_heads >= 1 && (head_dim == 64 || head_dim == 128) &&
                      max_pages >= 1 && max_page_budget >= 1,
                  "step_workspace_size: bad arguments");
  *bytes = step_ws_layout(num_heads, head_dim, max_pages, max_page_budget).total;
  return AOAKV_OK;
}

extern "C" int aoakv_step_plan_create(aoakv_step_plan* plan_out, void* kv_data,
                                      int32_t kv_capacity_pages, void* metadata_data,
                                      int32_t metadata_capacity_pages, void* v_log_norm,
                                      int32_t num_heads, int32_t head_dim, int32_t page_size,
                                      int32_t page_budget, int32_t score_mode,
                                      int32_t sink_first_page, int32_t max_pages,
                                      int32_t max_ctas, int32_t flags) {
  AOAKV_CHECK_ARG(plan_out != nullptr, "step plan: plan_out is NULL");
  *plan_out = nullptr;
  aoakv_step_plan_s* p = new (std::nothrow) aoakv_step_plan_s();
  if (!p) return set_error(AOAKV_ERR_INVALID_ARG, "step plan: out of host memory");
  const int rc = plan_init(p, kv_data, kv_capacity_pages, metadata_data, metadata_capacity_pages,
                           v_log_norm, num_heads, head_dim, page_size, page_budget, score_mode,
                           sink_first_page, max_pages, max_ctas, flags);
  if (rc) {
    delete p;
    return rc;
  }
  *plan_out = p;
  return AOAKV_OK;
}

extern "C" int aoakv_step_plan_run(aoakv_step_plan plan, const void* q, const void* k_new,
                                   const void* v_new, void* o, const int32_t* kv_indices,
                                   int32_t num_kv_pages, int32_t kv_last_page_len,
                                   const int32_t* metadata_indices, int32_t* selected_out,
                                   void* workspace, size_t workspace_bytes, void* stream) {
  AOAKV_CHECK_ARG(plan != nullptr, "step plan: plan is NULL");
  return plan_run(plan, q, k_new, v_new, o, kv_indices, num_kv_pages, kv_last_page_len,
                  metadata_indices, selected_out, workspace, workspace_bytes, stream);
}

extern "C" int aoakv_step_plan_info(aoakv_step_plan plan, int32_t num_kv_pages,
                                    int32_t want_selected, int32_t* kernels_out,
                                    int32_t* cluster_out) {
  AOAKV_CHECK_ARG(plan != nullptr, "step plan: plan is NULL");
  AOAKV_CHECK_ARG(num_kv_pages >= 1, "step plan: num_kv_pages must be >= 1");
  if (kernels_out) *kernels_out = plan_kernels(plan, num_kv_pages, want_selected != 0);
  if (cluster_out) *cluster_out = plan->cluster_ok ? plan->cp.cluster : 0;
  return AOAKV_OK;
}

extern "C" int aoakv_step_plan_set_rope(aoakv_step_plan plan, float rope_scale,
                                        float rope_theta) {
  AOAKV_CHECK_ARG(plan != nullptr, "step_plan_set_rope: plan is NULL");
  AOAKV_CHECK_ARG(rope_scale <= 0.f || rope_theta > 0.f,
                  "step_plan_set_rope: rope_theta must be > 0");
  plan->rope = rope_scale > 0.f;
  plan->rope_scale = rope_scale;
  plan->rope_theta = rope_theta;
  return AOAKV_OK;
}

extern "C" int aoakv_step_plan_destroy(aoakv_step_plan plan) {
  delete plan;
  return AOAKV_OK;
}

// ---------------------------------------------------- page-range sharding
namespace aoakv {
namespace {

constexpr int kShardMaxProp = 1024;  // entries per (rank, head): k - 1

// A selection runs (proposals travel) when the sequence has more pages than
// k and k > 1.
bool num_total_ok(int n_total, int k) { return n_total > k && k > 1; }

// Arguments shared by both shard passes; fills the whole-sequence k.
int shard_args(const aoakv_step_plan_s* p, ClusterStepArgs* a, const void* q,
               const int32_t* kv_indices, int n_local, int n_total, int page_lo,
               const int32_t* meta_indices, int* k_out) {
  AOAKV_CHECK_ARG(p != nullptr, "shard: plan is NULL");
  if (!p->cluster_ok)
    return set_error(AOAKV_ERR_UNSUPPORTED,
                     "shard: the plan runs the four-kernel chain (needs head_dim 64/128, "
                     "page_size <= 16 and a page count that fits the cluster kernel)");
  AOAKV_CHECK_ARG(q && kv_indices && meta_indices, "shard: NULL pointer argument");
  AOAKV_CHECK_ARG(n_local >= 1 && page_lo >= 0 && page_lo % p->P == 0 &&
                      page_lo + n_local <= n_total,
                  "shard: local pages must be [page_lo, page_lo + num_local_pages) of the "
                  "sequence with page_lo a multiple of page_size");
  int k_pages, k;
  step_budget(n_total, p->budget, p->sink, &k_pages, &k);
  AOAKV_CHECK_ARG(k <= p->cp.shape.max_slots,
                  "shard: plan made without AOAKV_PLAN_SHARD, or with a smaller budget");
  *a = {};
  a->q = static_cast<const __half*>(q);
  a->kv = static_cast<__half*>(p->kv);
  a->kv_indices = kv_indices;
  a->kv_cap = p->kv_cap;
  a->meta = static_cast<__half*>(p->meta);
  a->meta_indices = meta_indices;
  a->meta_cap = p->meta_cap;
  a->vlog = static_cast<__half*>(p->vlog);
  a->H = p->H;
  a->P = p->P;
  a->k_slots = k;
  a->mode = p->mode;
  a->two_rsqrt_d = 2.f / std::sqrt(static_cast<float>(p->D));
  a->scale_log2 = (1.f / std::sqrt(static_cast<float>(p->D))) * 1.4426950408889634f;
  a->err = dev_error_ptr();
  a->page_lo = page_lo;
  a->last_len = 1;
  *k_out = k;
  return AOAKV_OK;
}

}  // namespace
}  // namespace aoakv

// The mailboxes of the peer-store exchange (aoakv_shard_mailbox_*).
struct aoakv_shard_mailbox_s {
  int device, world, rank, H, D, max_prop;
  aoakv::ShardMail mail;
  uint8_t* local;
  size_t bytes;
  bool connected;
  bool opened[aoakv::kShardMaxWorld];
};

namespace aoakv {
namespace {

int shard_propose(const aoakv_step_plan_s* plan, const aoakv_shard_mailbox_s* mb,
                  const void* q, const int32_t* kv_indices, int n_local, int n_total,
                  int page_lo, const int32_t* meta_indices, void* cand_out, void* stream) {
  ClusterStepArgs a;
  int k = 0;
  int rc = shard_args(plan, &a, q, kv_indices, n_local, n_total, page_lo, meta_indices, &k);
  if (rc) return rc;
  AOAKV_CHECK_ARG(num_total_ok(n_total, k), "shard_propose: nothing to select (every page, "
                  "or only the last, is attended); run the finish pass with no candidates");
  AOAKV_CHECK_ARG(k - 1 <= kShardMaxProp, "shard_propose: page budget above 1025 pages");
  const bool owns_last = page_lo + n_local == n_total;
  // one page past the local ones stands for another GPU's last page: the
  // kernel scores pages [0, n_pages - 1) and never reads that entry
  a.n_pages = n_local + (owns_last ? 0 : 1);
  AOAKV_CHECK_ARG(a.n_pages <= plan->max_pages,
                  "shard_propose: more local pages than the plan's max_pages - 1");
  a.sink = plan->sink && page_lo == 0;
  a.shard = kShardPropose;
  a.n_prop = k - 1;
  if (mb) {
    AOAKV_CHECK_ARG(mb->connected && mb->H == plan->H && mb->D == plan->D &&
                        k - 1 <= mb->max_prop,
                    "shard_propose: mailbox not connected, or made for other sizes");
    a.p2p = 1;
    a.mail = mb->mail;
    a.world = mb->world;
    a.rank = mb->rank;
    a.cand_out = reinterpret_cast<uint2*>(mb->local + mb->mail.stage_off);
  } else {
    AOAKV_CHECK_ARG(cand_out != nullptr, "shard_propose: cand_out is NULL");
    a.cand_out = static_cast<uint2*>(cand_out);
  }
  return launch_cluster_step(a, plan->kv_sw, plan->meta_map, plan->D, plan->cp,
                             static_cast<cudaStream_t>(stream));
}

int shard_finish(const aoakv_step_plan_s* plan, const aoakv_shard_mailbox_s* mb, const void* q,
                 const void* k_new, const void* v_new, const int32_t* kv_indices, int n_local,
                 int n_total, int page_lo, int last_len, const int32_t* meta_indices,
                 const void* cand_all, int world, int rank, float* state_out,
                 int32_t* selected_out, void* stream) {
  ClusterStepArgs a;
  int k = 0;
  int rc = shard_args(plan, &a, q, kv_indices, n_local, n_total, page_lo, meta_indices, &k);
  if (rc) return rc;
  const bool owns_last = page_lo + n_local == n_total;
  const bool sparse = num_total_ok(n_total, k);
  if (mb) {
    AOAKV_CHECK_ARG(mb->connected && mb->H == plan->H && mb->D == plan->D &&
                        (!sparse || k - 1 <= mb->max_prop),
                    "shard_finish: mailbox not connected, or made for other sizes");
    world = mb->world;
    rank = mb->rank;
    cand_all = mb->local + mb->mail.cand_off;  // read as tagged words by the kernel
    a.p2p = 1;
    a.mail = mb->mail;
  } else {
    AOAKV_CHECK_ARG(state_out != nullptr, "shard_finish: state_out is NULL");
    if (!sparse) {  // no lists: world and rank are not used
      world = 1;
      rank = 0;
    }
  }
  if (owns_last) {
    AOAKV_CHECK_ARG(k_new && v_new, "shard_finish: the last page's owner needs k_new, v_new");
    AOAKV_CHECK_ARG(last_len >= 1 && last_len <= plan->P,
                    "shard_finish: kv_last_page_len must be in [1, page_size]");
  }
  AOAKV_CHECK_ARG(world >= 1 && world <= kShardMaxWorld && rank >= 0 && rank < world,
                  "shard_finish: world must be in [1, 8] and rank in [0, world)");
  if (sparse) {
    AOAKV_CHECK_ARG(cand_all != nullptr, "shard_finish: cand_all is NULL");
    AOAKV_CHECK_ARG(k - 1 <= kShardMaxProp && world * (k - 1) <= 2048,
                    "shard_finish: world * (k - 1) candidates above 2048");
  }
  AOAKV_CHECK_ARG(n_local <= plan->max_pages,
                  "shard_finish: more local pages than the plan's max_pages");
  a.k_new = static_cast<const __half*>(k_new);
  a.v_new = static_cast<const __half*>(v_new);
  a.n_pages = n_local;
  a.last_len = owns_last ? last_len : 1;
  a.shard = kShardFinish;
  a.n_prop = sparse ? k - 1 : 0;
  a.dense = n_total <= k;
  a.cand_in = static_cast<const uint2*>(cand_all);
  a.world = world;
  a.rank = rank;
  a.owns_last = owns_last;
  a.state_out = state_out;
  a.selected_out = sparse ? selected_out : nullptr;
  a.sel_cols = k - 1;
  return launch_cluster_step(a, plan->kv_sw, plan->meta_map, plan->D, plan->cp,
                             static_cast<cudaStream_t>(stream));
}

}  // namespace
int launch_merge_mailbox(const ShardMail& m, int world, int rank, int H, int D, int proposals,
                         void* o, cudaStream_t s);
}  // namespace aoakv

extern "C" int aoakv_shard_propose(aoakv_step_plan plan, const void* q,
                                   const int32_t* kv_indices, int32_t num_local_pages,
                                   int32_t num_total_pages, int32_t page_lo,
                                   const int32_t* metadata_indices, void* cand_out,
                                   void* stream) {
  AOAKV_NVTX("aoakv_shard_propose");
  return shard_propose(plan, nullptr, q, kv_indices, num_local_pages, num_total_pages, page_lo,
                       metadata_indices, cand_out, stream);
}

extern "C" int aoakv_shard_finish(aoakv_step_plan plan, const void* q, const void* k_new,
                                  const void* v_new, const int32_t* kv_indices,
                                  int32_t num_local_pages, int32_t num_total_pages,
                                  int32_t page_lo, int32_t kv_last_page_len,
                                  const int32_t* metadata_indices, const void* cand_all,
                                  int32_t world, int32_t rank, float* state_out,
                                  int32_t* selected_out, void* stream) {
  AOAKV_NVTX("aoakv_shard_finish");
  return shard_finish(plan, nullptr, q, k_new, v_new, kv_indices, num_local_pages,
                      num_total_pages, page_lo, kv_last_page_len, metadata_indices, cand_all,
                      world, rank, state_out, selected_out, stream);
}

// ------------------------------------------ peer-store exchange (mailboxes)
namespace {
size_t mb_up(size_t x) { return (x + 255) / 256 * 256; }
}  // namespace

extern "C" int aoakv_shard_mailbox_create(aoakv_shard_mailbox* mb_out, int32_t world,
                                          int32_t rank, int32_t num_heads, int32_t head_dim,
                                          int32_t max_proposals, void* ipc_handle_out) {
  AOAKV_NVTX("aoakv_shard_mailbox_create");
  AOAKV_CHECK_ARG(mb_out && ipc_handle_out, "shard_mailbox_create: NULL pointer argument");
  AOAKV_CHECK_ARG(world >= 1 && world <= kShardMaxWorld && rank >= 0 && rank < world &&
                      num_heads >= 1 && (head_dim == 64 || head_dim == 128) &&
                      max_proposals >= 1 && max_proposals <= kShardMaxProp,
                  "shard_mailbox_create: bad sizes");
  *mb_out = nullptr;
  aoakv_shard_mailbox_s* mb = new (std::nothrow) aoakv_shard_mailbox_s();
  AOAKV_CHECK_ARG(mb != nullptr, "shard_mailbox_create: out of host memory");
  mb->world = world;
  mb->rank = rank;
  mb->H = num_heads;
  mb->D = head_dim;
  mb->max_prop = max_proposals;
  ShardMail& m = mb->mail;
  size_t off = 0;
  m.cand_off = 0;  // two tagged 64-bit words per proposal
  off = mb_up(static_cast<size_t>(world) * num_heads * max_proposals * 16);
  m.state_off = static_cast<uint32_t>(off);  // one tagged 64-bit word per value
  off += mb_up(static_cast<size_t>(world) * num_heads * (head_dim + 1) * 8);
  m.stage_off = static_cast<uint32_t>(off);  // this GPU's own {key, page} list
  off += mb_up(static_cast<size_t>(num_heads) * max_proposals * 8);
  m.ep_off = static_cast<uint32_t>(off);
  off += 256;
  mb->bytes = off;
  cudaError_t e = cudaGetDevice(&mb->device);
  if (e == cudaSuccess) e = cudaMalloc(reinterpret_cast<void**>(&mb->local), mb->bytes);
  if (e == cudaSuccess) e = cudaMemset(mb->local, 0, mb->bytes);
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  cudaIpcMemHandle_t h;
  if (e == cudaSuccess) e = cudaIpcGetMemHandle(&h, mb->local);
  if (e != cudaSuccess) {
    if (mb->local) cudaFree(mb->local);
    delete mb;
    AOAKV_CUDA_TRY(e, "shard_mailbox_create");
  }
  std::memcpy(ipc_handle_out, &h, sizeof(h));
  m.base[rank] = mb->local;
  *mb_out = mb;
  return AOAKV_OK;
}

extern "C" int aoakv_shard_mailbox_connect(aoakv_shard_mailbox mb, const void* ipc_handles) {
  AOAKV_NVTX("aoakv_shard_mailbox_connect");
  AOAKV_CHECK_ARG(mb && ipc_handles, "shard_mailbox_connect: NULL pointer argument");
  AOAKV_CHECK_ARG(!mb->connected, "shard_mailbox_connect: already connected");
  const uint8_t* hs = static_cast<const uint8_t*>(ipc_handles);
  for (int g = 0; g < mb->world; ++g) {
    if (g == mb->rank) continue;
    cudaIpcMemHandle_t h;
    std::memcpy(&h, hs + static_cast<size_t>(g) * sizeof(h), sizeof(h));
    void* p = nullptr;
    const cudaError_t e = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
    if (e != cudaSuccess) {
      for (int j = 0; j < g; ++j)
        if (mb->opened[j]) {
          cudaIpcCloseMemHandle(mb->mail.base[j]);
          mb->opened[j] = false;
        }
      AOAKV_CUDA_TRY(e, "shard_mailbox_connect: cudaIpcOpenMemHandle");
    }
    mb->mail.base[g] = static_cast<uint8_t*>(p);
    mb->opened[g] = true;
  }
  mb->connected = true;
  return AOAKV_OK;
}

extern "C" int aoakv_shard_mailbox_destroy(aoakv_shard_mailbox mb) {
  if (!mb) return AOAKV_OK;
  for (int g = 0; g < mb->world; ++g)
    if (mb->opened[g]) cudaIpcCloseMemHandle(mb->mail.base[g]);
  if (mb->local) cudaFree(mb->local);
  delete mb;
  return AOAKV_OK;
}

extern "C" int aoakv_shard_propose_p2p(aoakv_step_plan plan, aoakv_shard_mailbox mb,
                                       const void* q, const int32_t* kv_indices,
                                       int32_t num_local_pages, int32_t num_total_pages,
                                       int32_t page_lo, const int32_t* metadata_indices,
                                       void* stream) {
  AOAKV_NVTX("aoakv_shard_propose_p2p");
  AOAKV_CHECK_ARG(mb != nullptr, "shard_propose_p2p: mailbox is NULL");
  return shard_propose(plan, mb, q, kv_indices, num_local_pages, num_total_pages, page_lo,
                       metadata_indices, nullptr, stream);
}

extern "C" int aoakv_shard_finish_p2p(aoakv_step_plan plan, aoakv_shard_mailbox mb,
                                      const void* q, const void* k_new, const void* v_new,
                                      const int32_t* kv_indices, int32_t num_local_pages,
                                      int32_t num_total_pages, int32_t page_lo,
                                      int32_t kv_last_page_len,
                                      const int32_t* metadata_indices, int32_t* selected_out,
                                      void* stream) {
  AOAKV_NVTX("aoakv_shard_finish_p2p");
  AOAKV_CHECK_ARG(mb != nullptr, "shard_finish_p2p: mailbox is NULL");
  return shard_finish(plan, mb, q, k_new, v_new, kv_indices, num_local_pages, num_total_pages,
                      page_lo, kv_last_page_len, metadata_indices, nullptr, 0, 0, nullptr,
                      selected_out, stream);
}

extern "C" int aoakv_shard_merge_p2p(aoakv_shard_mailbox mb, int32_t with_proposals, void* o,
                                     void* stream) {
  AOAKV_NVTX("aoakv_shard_merge_p2p");
  AOAKV_CHECK_ARG(mb && o, "shard_merge_p2p: NULL pointer argument");
  AOAKV_CHECK_ARG(mb->connected, "shard_merge_p2p: mailbox not connected");
  return launch_merge_mailbox(mb->mail, mb->world, mb->rank, mb->H, mb->D,
                              with_proposals != 0, o, static_cast<cudaStream_t>(stream));
}

extern "C" int aoakv_step_launches(int32_t num_heads, int32_t head_dim, int32_t page_size,
                                   int32_t num_kv_pages, int32_t page_budget,
                                   int32_t sink_first_page, int32_t want_selected,
                                   int32_t* kernels_out) {
  AOAKV_CHECK_ARG(kernels_out != nullptr, "step_launches: kernels_out is NULL");
  AOAKV_CHECK_ARG(num_heads >= 1 && (head_dim == 64 || head_dim == 128) && page_size >= 1 &&
                      num_kv_pages >= 1 && page_budget >= 1,
                  "step_launches: bad arguments");
  aoakv_step_plan_s p = {};
  p.budget = page_budget;
  p.sink = sink_first_page != 0;
  int k_pages, k;
  step_budget(num_kv_pages, page_budget, p.sink, &k_pages, &k);
  p.cluster_ok = cluster_step_plan(num_heads, head_dim, page_size, num_kv_pages, k_pages, 0,
                                   &p.cp) != 0;
  *kernels_out = plan_kernels(&p, num_kv_pages, want_selected != 0);
  return AOAKV_OK;
}

namespace {

// The stateless entry points: a plan on the stack for one call.
int decode_step_once(const void* q, const void* k_new, const void* v_new, void* o,
                     void* kv_data, const int32_t* kv_indices, int32_t num_kv_pages,
                     int32_t kv_last_page_len, int32_t kv_capacity_pages, void* metadata_data,
                     const int32_t* metadata_indices, int32_t metadata_capacity_pages,
                     void* v_log_norm, int32_t num_heads, int32_t head_dim, int32_t page_size,
                     int32_t page_budget, int32_t score_mode, int32_t sink_first_page,
                     int32_t* selected_out, void* workspace, size_t workspace_bytes,
                     int32_t max_ctas, void* stream) {
  AOAKV_CHECK_ARG(num_kv_pages >= 1 && num_kv_pages <= kv_capacity_pages,
                  "step: num_kv_pages must be in [1, kv_capacity_pages]");
  aoakv_step_plan_s p = {};
  const int rc = plan_init(&p, kv_data, kv_capacity_pages, metadata_data,
                           metadata_capacity_pages, v_log_norm, num_heads, head_dim, page_size,
                           page_budget, score_mode, sink_first_page, num_kv_pages, max_ctas, 0);
  if (rc) return rc;
  return plan_run(&p, q, k_new, v_new, o, kv_indices, num_kv_pages, kv_last_page_len,
                  metadata_indices, selected_out, workspace, workspace_bytes, stream);
}

}  // namespace

extern "C" int aoakv_decode_step(
    const void* q, const void* k_new, const void* v_new, void* o, void* kv_data,
    const int32_t* kv_indices, int32_t num_kv_pages, int32_t kv_last_page_len,
    int32_t kv_capacity_pages, void* metadata_data, const int32_t* metadata_indices,
    int32_t metadata_capacity_pages, void* v_log_norm, int32_t num_heads,
    int32_t head_dim, int32_t page_size, int32_t page_budget, int32_t score_mode,
    int32_t sink_first_page, int32_t* selected_out, void* workspace,
    size_t workspace_bytes, void* stream) {
  return decode_step_once(q, k_new, v_new, o, kv_data, kv_indices, num_kv_pages,
                          kv_last_page_len, kv_capacity_pages, metadata_data, metadata_indices,
                          metadata_capacity_pages, v_log_norm, num_heads, head_dim, page_size,
                          page_budget, score_mode, sink_first_page, selected_out, workspace,
                          workspace_bytes, 0, stream);
}

extern "C" int aoakv_decode_step_grid(
    const void* q, const void* k_new, const void* v_new, void* o, void* kv_data,
    const int32_t* kv_indices, int32_t num_kv_pages, int32_t kv_last_page_len,
    int32_t kv_capacity_pages, void* metadata_data, const int32_t* metadata_indices,
    int32_t metadata_capacity_pages, void* v_log_norm, int32_t num_heads,
    int32_t head_dim, int32_t page_size, int32_t page_budget, int32_t score_mode,
    int32_t sink_first_page, int32_t* selected_out, void* workspace,
    size_t workspace_bytes, int32_t max_ctas, void* stream) {
  AOAKV_CHECK_ARG(max_ctas >= 0, "step: max_ctas must be >= 0");
  return decode_step_once(q, k_new, v_new, o, kv_data, kv_indices, num_kv_pages,
                          kv_last_page_len, kv_capacity_pages, metadata_data, metadata_indices,
                          metadata_capacity_pages, v_log_norm, num_heads, head_dim, page_size,
                          page_budget, score_mode, sink_first_page, selected_out, workspace,
                          workspace_bytes, max_ctas, stream);
}

namespace aoakv {
// The batched step; kv_ends (optional) gives each request's page-list end
// (a device page table's layout) instead of kv_indptr[r + 1].
static int run_batched(const void* q, const void* k_new, const void* v_new, void* o,
                       void* kv_data, int32_t kv_capacity_pages, const int32_t* kv_indptr,
                       const int32_t* kv_ends, const int32_t* kv_indices,
                       const int32_t* kv_last_page_len, void* metadata_data,
                       int32_t metadata_capacity_pages, const int32_t* metadata_indptr,
                       const int32_t* metadata_indices, void* v_log_norm, int32_t num_requests,
                       int32_t max_pages, int32_t num_heads, int32_t head_dim, int32_t page_size,
                       int32_t page_budget, int32_t score_mode, int32_t sink_first_page,
                       int32_t* selected_out, void* stream, float rope_scale = 0.f,
                       float rope_theta = 0.f) {
  AOAKV_CHECK_ARG(rope_scale <= 0.f || rope_theta > 0.f, "step: rope_theta must be > 0");
  AOAKV_CHECK_ARG(q && k_new && v_new && o && kv_data && kv_indptr && kv_indices &&
                      kv_last_page_len && metadata_data && metadata_indptr && metadata_indices &&
                      v_log_norm,
                  "batched step: NULL pointer argument");
  AOAKV_CHECK_ARG(num_requests >= 1 && num_requests <= 65535,
                  "batched step: num_requests must be in [1, 65535]");
  int rc = check_plan_args(num_heads, head_dim, page_size, kv_capacity_pages,
                           metadata_capacity_pages, page_budget, score_mode);
  if (rc) return rc;
  AOAKV_CHECK_ARG(max_pages >= 1 && max_pages <= kv_capacity_pages,
                  "batched step: max_pages must be in [1, kv_capacity_pages]");
  const int H = num_heads, D = head_dim, P = page_size;
  int k_pages, k;
  step_budget(max_pages, page_budget, sink_first_page != 0, &k_pages, &k);
  // about one wave of (request, head) clusters: fewer CTAs per head when
  // there are many requests
  const int per_req = num_sms() / num_requests;
  ClusterPlan cp;
  if (!cluster_step_plan(H, D, P, max_pages, k_pages, per_req > 1 ? per_req : 1, &cp))
    return set_error(AOAKV_ERR_UNSUPPORTED,
                     "batched step: needs head_dim 64/128, page_size <= 16 and max_pages that "
                     "fit the kernel's shared memory");
  CUtensorMap kv_sw, meta_map;
  rc = make_kv_tmap_sw128(&kv_sw, kv_data, H, D, P, kv_capacity_pages);
  if (rc) return rc;
  rc = make_kv_tmap(&meta_map, metadata_data, H, D, P, metadata_capacity_pages);
  if (rc) return rc;
  ClusterStepArgs a = {};
  a.q = static_cast<const __half*>(q);
  a.k_new = static_cast<const __half*>(k_new);
  a.v_new = static_cast<const __half*>(v_new);
  a.o = static_cast<__half*>(o);
  a.kv = static_cast<__half*>(kv_data);
  a.kv_indices = kv_indices;
  a.kv_cap = kv_capacity_pages;
  a.meta = static_cast<__half*>(metadata_data);
  a.meta_indices = metadata_indices;
  a.meta_cap = metadata_capacity_pages;
  a.vlog = static_cast<__half*>(v_log_norm);
  a.H = H;
  a.P = P;
  a.sink = sink_first_page != 0;
  a.mode = score_mode;
  a.two_rsqrt_d = 2.f / std::sqrt(static_cast<float>(D));
  a.scale_log2 = (1.f / std::sqrt(static_cast<float>(D))) * 1.4426950408889634f;
  a.selected_out = selected_out;
  a.sel_cols = k_pages;
  a.err = dev_error_ptr();
  a.kv_indptr = kv_indptr;
  a.kv_ends = kv_ends;
  if (rope_scale > 0.f) {  // each request's own new-token position (rope_pos < 0)
    a.rope = 1;
    a.rope_pos = -1;
    a.rope_rcp_scale = 1.f / rope_scale;
    a.rope_log2_rcp_theta = std::log2(1.f / rope_theta);
  }
  a.meta_indptr = metadata_indptr;
  a.last_lens = kv_last_page_len;
  a.budget = page_budget;
  a.max_pages = max_pages;
  return launch_cluster_step(a, kv_sw, meta_map, D, cp, static_cast<cudaStream_t>(stream),
                             num_requests);
}
}  // namespace aoakv

extern "C" int aoakv_decode_step_batched(
    const void* q, const void* k_new, const void* v_new, void* o, void* kv_data,
    int32_t kv_capacity_pages, const int32_t* kv_indptr, const int32_t* kv_indices,
    const int32_t* kv_last_page_len, void* metadata_data, int32_t metadata_capacity_pages,
    const int32_t* metadata_indptr, const int32_t* metadata_indices, void* v_log_norm,
    int32_t num_requests, int32_t max_pages, int32_t num_heads, int32_t head_dim,
    int32_t page_size, int32_t page_budget, int32_t score_mode, int32_t sink_first_page,
    int32_t* selected_out, void* stream) {
  AOAKV_NVTX("aoakv_decode_step_batched");
  return run_batched(q, k_new, v_new, o, kv_data, kv_capacity_pages, kv_indptr, nullptr,
                     kv_indices, kv_last_page_len, metadata_data, metadata_capacity_pages,
                     metadata_indptr, metadata_indices, v_log_norm, num_requests, max_pages,
                     num_heads, head_dim, page_size, page_budget, score_mode, sink_first_page,
                     selected_out, stream);
}

extern "C" int aoakv_decode_step_table(
    aoakv_page_table table, const void* q, const void* k_new, const void* v_new, void* o,
    void* kv_data, int32_t kv_capacity_pages, void* metadata_data,
    int32_t metadata_capacity_pages, void* v_log_norm, int32_t num_heads, int32_t head_dim,
    int32_t page_budget, int32_t score_mode, int32_t sink_first_page, int32_t* selected_out,
    float rope_scale, float rope_theta, void* stream) {
  AOAKV_NVTX("aoakv_decode_step_table");
  AOAKV_CHECK_ARG(table != nullptr, "table step: NULL table");
  const PageTable* pt = reinterpret_cast<const PageTable*>(table);
  const PageTableLayout& L = pt->L;
  AOAKV_CHECK_ARG(L.cap <= kv_capacity_pages && L.mcap <= metadata_capacity_pages,
                  "table step: the table's pools are larger than the given caches");
  int32_t* b = pt->buf;
  return run_batched(q, k_new, v_new, o, kv_data, kv_capacity_pages, b + L.kv_start,
                     b + L.kv_end, b + L.kv_indices, b + L.last_len, metadata_data,
                     metadata_capacity_pages, b + L.meta_start, b + L.meta_indices, v_log_norm,
                     L.R, L.M, num_heads, head_dim, L.P, page_budget, score_mode,
                     sink_first_page, selected_out, stream, rope_scale, rope_theta);
}
