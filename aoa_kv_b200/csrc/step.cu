// Per-layer decode step for one request: append -> estimate -> top-k ->
// sparse decode, stream-ordered with programmatic dependent launch, no host
// synchronisation and no allocation.
//
// Reference call order: kernels/aoa_kv/quest/models/QuestAttention.py:99-157
// (append_kv, then need_estimate() ? estimate + topk + sparse decode : decode
// over every page), with the page budget of controller.py:118-127 and
// utils/__init__.py:237 (top-(k-1) plus the last page) or, with the sink,
// filtering/filter_util.py:226-231 and :373-377 (page 0 and the last page
// forced, k = min(max(3, budget), N)).
#include <cmath>
#include <cstdlib>
#include <cstring>

#include "decode.cuh"
#include "estimate.cuh"
#include "fused.h"
#include "plan.h"
#include "step_cluster.h"
#include "topk.cuh"

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

// Workspace: [sync words][decode partials][fp32 scores][selected ids]. The
// sync words and the decode tickets must be zero between calls.
struct StepWs {
  size_t sync_off, dec_off, scores_off, idx_off, total;
};

StepWs step_ws_layout(int H, int D, int max_pages, int max_budget) {
  auto up = [](size_t x) { return (x + 255) / 256 * 256; };
  const int max_slots = max_budget < 3 ? 3 : max_budget;
  StepWs w;
  w.sync_off = 0;
  size_t off = up(fused_sync_bytes(H));
  w.dec_off = off;
  off += up(decode_ws_bytes(H, D, max_slots));
  w.scores_off = off;
  off += up(static_cast<size_t>(H) * max_pages * 4);
  w.idx_off = off;
  off += up(static_cast<size_t>(H) * max_slots * 4);
  w.total = off;
  return w;
}

// Which kernel(s) run a sparse step: the phase-by-phase fused kernel
// (step_fused.cu) when the shape allows, else the four-launch chain.
// AOAKV_STEP_IMPL=pipe selects the pipelined two-role kernel (step_pipe.cu;
// measured slower at the headline shape: its scorers get half the SMs'
// loads in flight) and =chain the chain (read on every call, for A/B
// comparisons).
enum class StepImpl { kCluster, kPipe, kFused, kChain };

struct StepChoice {
  StepImpl impl;
  int grid, chunk, n_chunks;
  size_t smem;
  ClusterPlan cp;
};

StepChoice choose_step(int H, int D, int P, int N, int k, int max_grid = 0) {
  const char* e = std::getenv("AOAKV_STEP_IMPL");
  const bool want_chain = e && std::strcmp(e, "chain") == 0;
  const bool want_pipe = e && std::strcmp(e, "pipe") == 0;
  const bool want_fused = e && std::strcmp(e, "fused") == 0;
  StepChoice c = {StepImpl::kChain, 0, 0, 0, 0, {}};
  if (want_chain) return c;
  if (!want_pipe && !want_fused && max_grid == 0 && cluster_step_plan(H, D, P, N, k, &c.cp)) {
    c.impl = StepImpl::kCluster;
    return c;
  }
  if (want_pipe && pipe_supported(H, D, P, N - 1, k - 1, &c.grid, &c.smem, &c.chunk,
                                  &c.n_chunks)) {
    c.impl = StepImpl::kPipe;
    return c;
  }
  if (fused_supported(H, D, P, N - 1, k - 1, &c.grid, &c.smem, &c.chunk, &c.n_chunks,
                      max_grid))
    c.impl = StepImpl::kFused;
  return c;
}

}  // namespace
}  // namespace aoakv

using namespace aoakv;

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

extern "C" int aoakv_step_launches(int32_t num_heads, int32_t head_dim, int32_t page_size,
                                   int32_t num_kv_pages, int32_t page_budget,
                                   int32_t sink_first_page, int32_t want_selected,
                                   int32_t* kernels_out) {
  AOAKV_CHECK_ARG(kernels_out != nullptr, "step_launches: kernels_out is NULL");
  AOAKV_CHECK_ARG(num_heads >= 1 && (head_dim == 64 || head_dim == 128) && page_size >= 1 &&
                      num_kv_pages >= 1 && page_budget >= 1,
                  "step_launches: bad arguments");
  const int N = num_kv_pages;
  const int k_pages = sink_first_page ? (page_budget < 3 ? 3 : page_budget) : page_budget;
  const int k = k_pages < N ? k_pages : N;
  const bool sparse = N > k && k > 1;
  int n = sparse ? 4 : 2;
  const StepImpl im = choose_step(num_heads, head_dim, page_size, N, k).impl;
  if (im == StepImpl::kCluster || (sparse && im != StepImpl::kChain)) n = 1;
  if (want_selected && n > 1) ++n;
  *kernels_out = n;
  return AOAKV_OK;
}

namespace {

int decode_step_impl(
    const void* q, const void* k_new, const void* v_new, void* o, void* kv_data,
    const int32_t* kv_indices, int32_t num_kv_pages, int32_t kv_last_page_len,
    int32_t kv_capacity_pages, void* metadata_data, const int32_t* metadata_indices,
    int32_t metadata_capacity_pages, void* v_log_norm, int32_t num_heads,
    int32_t head_dim, int32_t page_size, int32_t page_budget, int32_t score_mode,
    int32_t sink_first_page, int32_t* selected_out, void* workspace,
    size_t workspace_bytes, void* stream, int max_ctas) {
  AOAKV_NVTX("aoakv_decode_step");
  AOAKV_CHECK_ARG(q && k_new && v_new && o && kv_data && kv_indices && metadata_data &&
                      metadata_indices && v_log_norm,
                  "step: NULL pointer argument");
  int rc = check_decode_shape(num_heads, head_dim, page_size, kv_capacity_pages,
                              AOAKV_LAYOUT_NHD);
  if (rc) return rc;
  AOAKV_CHECK_ARG(page_budget >= 1, "step: page_budget must be >= 1");
  AOAKV_CHECK_ARG(score_mode == AOAKV_SCORE_QUEST || score_mode == AOAKV_SCORE_AOAKV,
                  "step: score_mode must be QUEST or AOAKV");
  AOAKV_CHECK_ARG(num_kv_pages >= 1 && num_kv_pages <= kv_capacity_pages,
                  "step: num_kv_pages must be in [1, kv_capacity_pages]");
  const int N = num_kv_pages, P = page_size, H = num_heads, D = head_dim;
  const int n_meta = (N + P - 1) / P;
  const int meta_last = (N - 1) % P + 1;
  const int k_pages = sink_first_page ? (page_budget < 3 ? 3 : page_budget) : page_budget;
  const int k = k_pages < N ? k_pages : N;
  // k == 1 keeps only the last page: nothing to score.
  const bool sparse = N > k && k > 1;
  AOAKV_CHECK_ARG(!sparse || N - 1 <= kTopkMaxN, "step: more than 49153 pages");
  const StepWs lay = step_ws_layout(H, D, N, k_pages);
  AOAKV_CHECK_ARG(workspace != nullptr, "step: workspace is NULL");
  if (workspace_bytes < lay.total)
    return set_error(AOAKV_ERR_WORKSPACE,
                     "step: workspace smaller than aoakv_step_workspace_size(...) = " +
                         std::to_string(lay.total));
  AOAKV_CHECK_ARG(kv_last_page_len >= 1 && kv_last_page_len <= P,
                  "step: kv_last_page_len must be in [1, page_size]");
  AOAKV_CHECK_ARG(metadata_capacity_pages >= n_meta,
                  "step: metadata capacity below ceil(num_kv_pages / page_size)");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  uint8_t* ws = static_cast<uint8_t*>(workspace);

  const StepChoice sc = choose_step(H, D, P, N, k, max_ctas);
  if (sc.impl == StepImpl::kCluster) {
    ClusterStepArgs a = {};
    a.q = static_cast<const __half*>(q);
    a.k_new = static_cast<const __half*>(k_new);
    a.v_new = static_cast<const __half*>(v_new);
    a.o = static_cast<__half*>(o);
    a.kv = static_cast<__half*>(kv_data);
    a.kv_indices = kv_indices;
    a.n_pages = N;
    a.last_len = kv_last_page_len;
    a.kv_cap = kv_capacity_pages;
    a.meta = static_cast<__half*>(metadata_data);
    a.meta_indices = metadata_indices;
    a.meta_cap = metadata_capacity_pages;
    a.vlog = static_cast<__half*>(v_log_norm);
    a.H = H;
    a.P = P;
    a.k_slots = k;
    a.sink = sink_first_page != 0;
    a.mode = score_mode;
    a.two_rsqrt_d = 2.f / std::sqrt(static_cast<float>(D));
    a.scale_log2 = (1.f / std::sqrt(static_cast<float>(D))) * 1.4426950408889634f;
    a.selected_out = selected_out;
    a.sel_cols = k_pages;
    a.err = dev_error_ptr();
    CUtensorMap kmap, mmap;
    rc = make_kv_tmap_sw128(&kmap, kv_data, H, D, P, kv_capacity_pages);
    if (rc) return rc;
    rc = make_kv_tmap(&mmap, metadata_data, H, D, P, metadata_capacity_pages);
    if (rc) return rc;
    return launch_cluster_step(a, kmap, mmap, D, sc.cp, s);
  }
  if (sparse) {
    const int grid = sc.grid, chunk = sc.chunk, n_chunks = sc.n_chunks;
    const size_t smem = sc.smem;
    if (sc.impl != StepImpl::kChain) {
      FusedArgs f = {};
      f.k_new = static_cast<const __half*>(k_new);
      f.v_new = static_cast<const __half*>(v_new);
      f.kv = static_cast<__half*>(kv_data);
      f.kv_indices = kv_indices;
      f.n_pages = N;
      f.last_len = kv_last_page_len;
      f.kv_cap = kv_capacity_pages;
      f.meta = static_cast<__half*>(metadata_data);
      f.meta_indices = metadata_indices;
      f.meta_cap = metadata_capacity_pages;
      f.vlog = static_cast<__half*>(v_log_norm);
      f.H = H;
      f.P = P;
      f.k_sel = k - 1;
      f.sink = sink_first_page != 0;
      f.sel = reinterpret_cast<int32_t*>(ws + lay.idx_off);
      f.sync = reinterpret_cast<uint32_t*>(ws + lay.sync_off);
      f.selected_out = selected_out;
      f.sel_cols = k_pages;
      f.err = dev_error_ptr();
      const int per_cta = (N - 1 + grid - 1) / grid;
      const char* est_impl = std::getenv("AOAKV_EST_IMPL");  // "regs": A/B comparisons
      f.est_tma = H * (D / 8) == kFusedThreads && H % 8 == 0 && per_cta <= kEstMaxRange &&
                  reinterpret_cast<uintptr_t>(metadata_data) % 16 == 0 &&
                  (score_mode != AOAKV_SCORE_AOAKV ||
                   reinterpret_cast<uintptr_t>(v_log_norm) % 16 == 0) &&
                  !(est_impl && std::strcmp(est_impl, "regs") == 0);
      EstimateArgs& ea = f.est;
      ea.q = static_cast<const __half*>(q);
      ea.meta = f.meta;
      ea.meta_indices = metadata_indices;
      ea.kv_indices = kv_indices;
      ea.vlog = f.vlog;
      ea.out = ws + lay.scores_off;
      ea.out_stride = N;
      ea.out_f32 = 1;
      ea.n_score = N - 1;
      ea.H = H;
      ea.P = P;
      ea.meta_cap = metadata_capacity_pages;
      ea.kv_cap = kv_capacity_pages;
      ea.mode = score_mode;
      ea.two_rsqrt_d = 2.f / std::sqrt(static_cast<float>(D));
      ea.err = f.err;
      DecodeArgs& dd = f.dec;
      dd.q = ea.q;
      dd.o = static_cast<__half*>(o);
      dd.indices = f.sel;
      dd.idx_stride = k - 1;
      dd.n_sel = k - 1;
      dd.last_len = kv_last_page_len;
      dd.last_page_ptr = kv_indices + (N - 1);
      dd.H = H;
      dd.P = P;
      dd.kv_cap = kv_capacity_pages;
      dd.chunk_pages = chunk;
      dd.n_chunks = n_chunks;
      dd.scale_log2 = (1.f / std::sqrt(static_cast<float>(D))) * 1.4426950408889634f;
      dd.err = f.err;
      carve_decode_ws(ws + lay.dec_off, H, D, k, dd);
      CUtensorMap tmap, mtmap;
      rc = make_kv_tmap(&tmap, kv_data, H, D, P, kv_capacity_pages);
      if (rc) return rc;
      if (sc.impl == StepImpl::kPipe) {
        rc = make_meta_tmap(&mtmap, metadata_data, H, D, P, metadata_capacity_pages,
                            pipe_group_heads());
        if (rc) return rc;
        return launch_pipe(tmap, mtmap, f, D, grid, smem, s);
      }
      if (f.est_tma) {
        rc = make_meta_tmap(&mtmap, metadata_data, H, D, P, metadata_capacity_pages, H);
        if (rc) return rc;
      } else {
        mtmap = tmap;  // unused
      }
      return launch_fused(tmap, mtmap, f, D, grid, smem, s);
    }
  }

  rc = aoakv_append_kv_cache_decode(k_new, v_new, kv_data, kv_indices, N,
                                    kv_last_page_len, kv_capacity_pages, metadata_data,
                                    metadata_indices, n_meta, meta_last,
                                    metadata_capacity_pages, v_log_norm, H, D, P,
                                    AOAKV_LAYOUT_NHD, stream);
  if (rc) return rc;

  DecodeArgs da = {};
  da.q = static_cast<const __half*>(q);
  da.o = static_cast<__half*>(o);
  da.last_len = kv_last_page_len;
  da.last_page_ptr = kv_indices + (N - 1);
  da.H = H;
  da.P = P;
  da.kv_cap = kv_capacity_pages;
  da.scale_log2 = (1.f / std::sqrt(static_cast<float>(D))) * 1.4426950408889634f;
  da.err = dev_error_ptr();
  int32_t* sel_idx = reinterpret_cast<int32_t*>(ws + lay.idx_off);
  if (sparse) {
    EstimateArgs ea;
    ea.q = static_cast<const __half*>(q);
    ea.meta = static_cast<const __half*>(metadata_data);
    ea.meta_indices = metadata_indices;
    ea.kv_indices = kv_indices;
    ea.vlog = static_cast<const __half*>(v_log_norm);
    ea.out = ws + lay.scores_off;
    ea.out_stride = N;
    ea.out_f32 = 1;
    ea.n_score = N - 1;
    ea.H = H;
    ea.P = P;
    ea.meta_cap = metadata_capacity_pages;
    ea.kv_cap = kv_capacity_pages;
    ea.mode = score_mode;
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
    ta.sink = sink_first_page != 0;
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
  CUtensorMap tmap;
  rc = make_kv_tmap(&tmap, kv_data, H, D, P, kv_capacity_pages);
  if (rc) return rc;
  rc = launch_decode(da, tmap, D, pl, s, sparse);
  if (rc) return rc;
  if (selected_out) {
    fill_selected_kernel<<<H, 128, 0, s>>>(selected_out, k_pages, da.indices,
                                           da.idx_stride, da.n_sel, da.last_page_ptr, H);
    AOAKV_CUDA_TRY(cudaGetLastError(), "fill_selected launch");
  }
  return AOAKV_OK;
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
  return decode_step_impl(q, k_new, v_new, o, kv_data, kv_indices, num_kv_pages,
                          kv_last_page_len, kv_capacity_pages, metadata_data, metadata_indices,
                          metadata_capacity_pages, v_log_norm, num_heads, head_dim, page_size,
                          page_budget, score_mode, sink_first_page, selected_out, workspace,
                          workspace_bytes, stream, 0);
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
  return decode_step_impl(q, k_new, v_new, o, kv_data, kv_indices, num_kv_pages,
                          kv_last_page_len, kv_capacity_pages, metadata_data, metadata_indices,
                          metadata_capacity_pages, v_log_norm, num_heads, head_dim, page_size,
                          page_budget, score_mode, sink_first_page, selected_out, workspace,
                          workspace_bytes, stream, max_ctas);
}
