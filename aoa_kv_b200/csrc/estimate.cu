// a3 stand-alone entry point: aoakv_estimate_attn_score.
#include <cmath>
#include <cstdlib>
#include <cstring>

#include "estimate.cuh"
#include "plan.h"

namespace aoakv {
namespace {

template <int D>
__global__ void __launch_bounds__(kEstThreads) estimate_kernel(EstimateArgs a) {
  extern __shared__ float q_s[];
  stage_q<D>(a.q, q_s, a.H);
  __syncthreads();
  constexpr int RPS = kEstThreads / (D / 8);
  estimate_rows<D>(a, q_s, blockIdx.x * RPS * kEstUnroll, gridDim.x * RPS * kEstUnroll,
                   a.n_score * a.H);
}

constexpr int kHsUnroll = 4;

template <int D>
__global__ void __launch_bounds__(1024) estimate_hs_kernel(EstimateArgs a) {
  int b, e;
  page_range(a.n_score, blockIdx.x, gridDim.x, &b, &e);
  estimate_pages_hs<D, kHsUnroll>(a, b, e);
}

template <int D>
__global__ void __launch_bounds__(1024) estimate_tma_kernel(EstimateArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* stages = align_smem<128>(smem_raw);
  __shared__ uint64_t bars[kEstStages];
  __shared__ int ids_s[2 * kEstMaxRange];
  if (threadIdx.x == 0) {
    for (int j = 0; j < kEstStages; ++j) mbar_init(&bars[j], 1);
    fence_mbar_init();
  }
  __syncthreads();
  int b, e;
  page_range(a.n_score, blockIdx.x, gridDim.x, &b, &e);
  uint32_t phase = 0;
  estimate_pages_tma<D>(a, b, e, stages, bars, ids_s, &phase);
}

}  // namespace

// Head-stationary grid: enough CTAs of H*D/8 threads to cover every SM
// (up to 2048 threads per SM), each with a contiguous page range. With
// H % 8 == 0, 16-byte aligned buffers and <= kEstMaxRange pages per CTA the
// pages stream through a shared-memory ring by bulk copies; otherwise the
// threads load their 16-byte rows into registers.
int launch_estimate_hs(const EstimateArgs& a, int D, cudaStream_t s, bool tma);

int launch_estimate_hs(const EstimateArgs& a, int D, cudaStream_t s) {
  const bool aoa = a.mode == AOAKV_SCORE_AOAKV;
  const bool tma = a.H % 8 == 0 && reinterpret_cast<uintptr_t>(a.meta) % 16 == 0 &&
                   (!aoa || reinterpret_cast<uintptr_t>(a.vlog) % 16 == 0);
  return launch_estimate_hs(a, D, s, tma);
}

int launch_estimate_hs(const EstimateArgs& a, int D, cudaStream_t s, bool tma) {
  const int threads = a.H * (D / 8);
  const size_t smem = tma ? static_cast<size_t>(kEstStages) * est_stage_bytes(a.H, D) + 128 : 0;
  const void* fn =
      tma ? (D == 128 ? reinterpret_cast<const void*>(estimate_tma_kernel<128>)
                      : reinterpret_cast<const void*>(estimate_tma_kernel<64>))
          : (D == 128 ? reinterpret_cast<const void*>(estimate_hs_kernel<128>)
                      : reinterpret_cast<const void*>(estimate_hs_kernel<64>));
  if (smem > 48 * 1024)
    AOAKV_CUDA_TRY(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        static_cast<int>(smem)),
                   "estimate smem attribute");
  int per_sm = 0;
  AOAKV_CUDA_TRY(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, fn, threads, smem),
                 "estimate occupancy");
  int grid = num_sms() * (per_sm < 1 ? 1 : per_sm);
  const int min_pages = 2;  // at least a couple of pages per CTA
  if (grid > (a.n_score + min_pages - 1) / min_pages)
    grid = (a.n_score + min_pages - 1) / min_pages;
  if (grid < 1) grid = 1;
  if (tma && (a.n_score + grid - 1) / grid > kEstMaxRange)  // too long a range per CTA
    return launch_estimate_hs(a, D, s, false);
  if (tma) {
    if (D == 128)
      estimate_tma_kernel<128><<<grid, threads, smem, s>>>(a);
    else
      estimate_tma_kernel<64><<<grid, threads, smem, s>>>(a);
  } else {
    if (D == 128)
      estimate_hs_kernel<128><<<grid, threads, 0, s>>>(a);
    else
      estimate_hs_kernel<64><<<grid, threads, 0, s>>>(a);
  }
  AOAKV_CUDA_TRY(cudaGetLastError(), "estimate launch");
  return AOAKV_OK;
}

// Grid for a sweep over n_rows (page, head) rows: one resident wave (4 CTAs
// of 256 threads per SM at 64 registers), each CTA looping over sweeps so the
// q staging is paid once per CTA.
int estimate_grid(int64_t n_rows, int D) {
  const int64_t rows_per_cta = static_cast<int64_t>(kEstThreads / (D / 8)) * kEstUnroll;
  int64_t g = (n_rows + rows_per_cta - 1) / rows_per_cta;
  const int64_t cap = static_cast<int64_t>(num_sms()) * 4;
  if (g > cap) g = cap;
  if (g < 1) g = 1;
  return static_cast<int>(g);
}

int launch_estimate(const EstimateArgs& a, int D, cudaStream_t s) {
  const int64_t n_rows = static_cast<int64_t>(a.n_score) * a.H;
  if (n_rows == 0) return AOAKV_OK;
  const int hs_threads = a.H * (D / 8);
  if (hs_threads % 32 == 0 && hs_threads <= 1024) return launch_estimate_hs(a, D, s);
  const size_t smem = static_cast<size_t>(a.H) * D * sizeof(float);
  const int grid = estimate_grid(n_rows, D);
  if (D == 128) {
    if (smem > 48 * 1024)
      AOAKV_CUDA_TRY(cudaFuncSetAttribute(estimate_kernel<128>,
                                          cudaFuncAttributeMaxDynamicSharedMemorySize,
                                          static_cast<int>(smem)),
                     "estimate smem attribute");
    estimate_kernel<128><<<grid, kEstThreads, smem, s>>>(a);
  } else {
    if (smem > 48 * 1024)
      AOAKV_CUDA_TRY(cudaFuncSetAttribute(estimate_kernel<64>,
                                          cudaFuncAttributeMaxDynamicSharedMemorySize,
                                          static_cast<int>(smem)),
                     "estimate smem attribute");
    estimate_kernel<64><<<grid, kEstThreads, smem, s>>>(a);
  }
  AOAKV_CUDA_TRY(cudaGetLastError(), "estimate launch");
  return AOAKV_OK;
}

}  // namespace aoakv

using namespace aoakv;

extern "C" int aoakv_estimate_attn_score(
    const void* q, void* out, int32_t out_dtype, int64_t out_row_stride,
    const void* metadata_data, const int32_t* metadata_indices,
    int32_t num_metadata_pages, int32_t metadata_last_page_len,
    int32_t metadata_capacity_pages, const int32_t* kv_indices,
    int32_t kv_capacity_pages, const void* v_log_norm, int32_t num_heads,
    int32_t head_dim, int32_t page_size, int32_t layout, int32_t score_mode,
    void* stream) {
  AOAKV_NVTX("aoakv_estimate_attn_score");
  AOAKV_CHECK_ARG(q && out && metadata_data && metadata_indices,
                  "estimate: NULL pointer argument");
  if (layout != AOAKV_LAYOUT_NHD)
    return set_error(AOAKV_ERR_UNSUPPORTED, "estimate: only the NHD layout is built");
  AOAKV_CHECK_ARG(head_dim == 64 || head_dim == 128, "estimate: head_dim must be 64 or 128");
  AOAKV_CHECK_ARG(num_heads >= 1 && num_heads * head_dim * 4 <= 200 * 1024,
                  "estimate: num_heads out of range");
  AOAKV_CHECK_ARG(page_size >= 1 && page_size <= 1024, "estimate: page_size out of range");
  AOAKV_CHECK_ARG(num_metadata_pages >= 1, "estimate: num_metadata_pages must be >= 1");
  AOAKV_CHECK_ARG(metadata_last_page_len >= 1 && metadata_last_page_len <= page_size,
                  "estimate: metadata_last_page_len must be in [1, page_size]");
  AOAKV_CHECK_ARG(metadata_capacity_pages >= num_metadata_pages,
                  "estimate: metadata capacity below num_metadata_pages");
  AOAKV_CHECK_ARG(out_dtype == AOAKV_DTYPE_F16 || out_dtype == AOAKV_DTYPE_F32,
                  "estimate: out_dtype must be F16 or F32");
  AOAKV_CHECK_ARG(score_mode == AOAKV_SCORE_QUEST || score_mode == AOAKV_SCORE_AOAKV,
                  "estimate: score_mode must be QUEST or AOAKV");
  const int64_t n_kv = static_cast<int64_t>(num_metadata_pages - 1) * page_size +
                       metadata_last_page_len;
  AOAKV_CHECK_ARG(out_row_stride >= n_kv - 1, "estimate: out_row_stride below N-1");
  AOAKV_CHECK_ARG((n_kv - 1) * num_heads < (1LL << 31), "estimate: too many (page, head) rows");
  if (score_mode == AOAKV_SCORE_AOAKV) {
    AOAKV_CHECK_ARG(v_log_norm != nullptr, "estimate: AOAKV mode needs v_log_norm");
    AOAKV_CHECK_ARG(kv_capacity_pages >= 1, "estimate: kv_capacity_pages must be >= 1");
  }
  EstimateArgs a;
  a.q = static_cast<const __half*>(q);
  a.meta = static_cast<const __half*>(metadata_data);
  a.meta_indices = metadata_indices;
  a.kv_indices = kv_indices;
  a.vlog = static_cast<const __half*>(v_log_norm);
  a.out = out;
  a.out_stride = out_row_stride;
  a.out_f32 = out_dtype == AOAKV_DTYPE_F32;
  a.n_score = static_cast<int>(n_kv - 1);
  a.H = num_heads;
  a.P = page_size;
  a.meta_cap = metadata_capacity_pages;
  a.kv_cap = kv_capacity_pages;
  a.mode = score_mode;
  a.two_rsqrt_d = 2.f / std::sqrt(static_cast<float>(head_dim));
  a.err = dev_error_ptr();
  return launch_estimate(a, head_dim, static_cast<cudaStream_t>(stream));
}
