// Group-consistent page scoring for grouped-query attention (GQA): the
// page scores of the query heads that share a KV head are combined into one
// score per KV head and page, so every query head of the group attends the
// same pages.
//
// Reference: filtering/filter_util.py — Quest: the group's per-head page
// bounds are summed (local_heavy_hitter_mask_group_consistent_sum, :219-221);
// AOA-KV: each head's bound is scaled to 2*s/sqrt(D), the group is combined
// by logsumexp, then 2*log||mean V|| of the KV head's page is added
// (local_heavy_hitter_mask_value_aware_group_consistent_sum, :329, :352-361,
// :367). The reference's CUDA tree is MHA only (docs/KERNEL_DIFF.md:66-76).
//
// One warp per (KV head, page): the page's key max and min rows of the KV
// head are read once for the whole group (lane: D/32 channels), each query
// head's bound sum_i q_i * (q_i > 0 ? kmax_i : kmin_i) is reduced across the
// warp, and lane 0 combines and writes the fp32 score.
#include <cmath>

#include "common.cuh"
#include "decode.cuh"
#include "estimate.cuh"
#include "plan.h"

namespace aoakv {
namespace {

constexpr int kGqaWarps = 16;
constexpr int kGqaMaxGroup = 16;

template <int D>
__global__ void __launch_bounds__(kGqaWarps * 32)
    gqa_estimate_kernel(EstimateArgs a, int group) {
  constexpr int CPL = D / 32;
  __shared__ float qs[kGqaMaxGroup][D];
  const int hk = blockIdx.y, Hk = a.H;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  pdl_wait();  // the append before this kernel writes metadata and v_log_norm
  for (int i = threadIdx.x; i < group * D; i += blockDim.x)
    qs[i / D][i % D] = __half2float(a.q[(static_cast<size_t>(hk) * group + i / D) * D + i % D]);
  __syncthreads();
  const int p = blockIdx.x * kGqaWarps + warp;
  if (p >= a.n_score) return;
  const int mp = __ldcg(a.meta_indices + p / a.P), entry = p % a.P;
  if (mp < 0 || mp >= a.meta_cap) {
    if (lane == 0) {
      raise_dev_error(a.err, AOAKV_DEV_ERR_BAD_PAGE);
      static_cast<float*>(a.out)[static_cast<size_t>(hk) * a.out_stride + p] = NAN;
    }
    return;
  }
  const size_t row = static_cast<size_t>(Hk) * D;
  float mx[CPL], mn[CPL];
  load_row<CPL>(a.meta + (static_cast<size_t>(mp) * 2 * a.P + entry) * row + hk * D + lane * CPL,
                mx);
  load_row<CPL>(a.meta + ((static_cast<size_t>(mp) * 2 + 1) * a.P + entry) * row + hk * D +
                    lane * CPL,
                mn);
  const bool aoa = a.mode == AOAKV_SCORE_AOAKV;
  float total = 0.f, m = -INFINITY, se = 0.f;
  for (int i = 0; i < group; ++i) {
    float s = 0.f;
#pragma unroll
    for (int t = 0; t < CPL; ++t) {
      const float qv = qs[i][lane * CPL + t];
      s = fmaf(qv, qv > 0.f ? mx[t] : mn[t], s);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    if (aoa) {  // running logsumexp of 2*s/sqrt(D) over the group
      const float c = a.two_rsqrt_d * s;
      const float nm = fmaxf(m, c);
      se = (m == -INFINITY ? 0.f : se * expf(m - nm)) + expf(c - nm);
      m = nm;
    } else {
      total += s;
    }
  }
  if (lane != 0) return;
  float score = total;
  if (aoa) {
    const int pid = a.kv_indices ? __ldcg(a.kv_indices + p) : p;
    float vl = NAN;
    if (pid >= 0 && pid < a.kv_cap)
      vl = __half2float(a.vlog[static_cast<size_t>(pid) * Hk + hk]);
    else
      raise_dev_error(a.err, AOAKV_DEV_ERR_BAD_PAGE);
    score = m + logf(se) + 2.f * vl;
  }
  static_cast<float*>(a.out)[static_cast<size_t>(hk) * a.out_stride + p] = score;
}

}  // namespace

int launch_gqa_estimate(const EstimateArgs& a, int D, int group, cudaStream_t s) {
  AOAKV_CHECK_ARG(group >= 1 && group <= kGqaMaxGroup, "gqa: group size must be in [1, 16]");
  AOAKV_CHECK_ARG(a.out_f32, "gqa: fp32 scores only");
  if (a.n_score < 1) return AOAKV_OK;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((a.n_score + kGqaWarps - 1) / kGqaWarps, a.H);
  cfg.blockDim = dim3(kGqaWarps * 32);
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (D == 128)
    AOAKV_CUDA_TRY(cudaLaunchKernelEx(&cfg, gqa_estimate_kernel<128>, a, group), "gqa launch");
  else
    AOAKV_CUDA_TRY(cudaLaunchKernelEx(&cfg, gqa_estimate_kernel<64>, a, group), "gqa launch");
  return AOAKV_OK;
}

}  // namespace aoakv
