// a4 stand-alone entry point: aoakv_topk_filtering.
//
// k <= 256: one histogram pass and exact candidate ranking (topk_hist.cuh),
// or, when too many keys share the top bins, the warp-register bitonic
// top-K (topk_bitonic.cuh); 512 threads per row, results in descending score
// order either way. k > 256: shared-memory radix select (topk.cuh), 1024
// threads per row, results in ascending position order.
#include "plan.h"
#include "topk.cuh"
#include "topk_bitonic.cuh"
#include "topk_hist.cuh"

namespace aoakv {
namespace {

constexpr int kSmallThreads = 512;
constexpr int kSmallIdsMaxN = 16384;  // ids and bins staged in shared memory up to here

__global__ void __launch_bounds__(kTopkThreads) topk_kernel(TopkArgs a) {
  extern __shared__ uint32_t keys[];
  __shared__ TopkSmem sm;
  pdl_wait();
  topk_row(a, blockIdx.x, keys, sm);
}

// Dynamic shared memory: keys, then one region used either as the
// histogram state or, on the fallback, as the bitonic exchange buffer.
constexpr size_t kSmallUnion = sizeof(HistSmem) > bitonic_xbuf_bytes(kSmallThreads / 32, kBitonicMaxK)
                                   ? sizeof(HistSmem)
                                   : bitonic_xbuf_bytes(kSmallThreads / 32, kBitonicMaxK);

__global__ void __launch_bounds__(kSmallThreads, 1) topk_small_kernel(TopkArgs a) {
  extern __shared__ uint32_t keys[];
  const bool staged = a.n <= kSmallIdsMaxN;
  uint8_t* un = reinterpret_cast<uint8_t*>(keys) + hist_stage_bytes(a.n, staged);
  pdl_wait();
  if (!topk_row_hist(a, blockIdx.x, reinterpret_cast<uint8_t*>(keys), staged,
                     *reinterpret_cast<HistSmem*>(un)))
    topk_row_small(a, blockIdx.x, keys, reinterpret_cast<uint64_t*>(un));
}

}  // namespace

int launch_topk(const TopkArgs& a, int rows, cudaStream_t s, bool pdl) {
  const bool small = a.k <= kBitonicMaxK;
  const void* fn = small ? reinterpret_cast<const void*>(topk_small_kernel)
                         : reinterpret_cast<const void*>(topk_kernel);
  size_t smem = static_cast<size_t>(a.n) * sizeof(uint32_t);
  if (small)
    smem = static_cast<size_t>(hist_stage_bytes(a.n, a.n <= kSmallIdsMaxN)) + kSmallUnion;
  if (smem > 48 * 1024)
    AOAKV_CUDA_TRY(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        static_cast<int>(smem)),
                   "topk smem attribute");
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(rows);
  cfg.blockDim = dim3(small ? kSmallThreads : kTopkThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  if (small)
    AOAKV_CUDA_TRY(cudaLaunchKernelEx(&cfg, topk_small_kernel, a), "topk launch");
  else
    AOAKV_CUDA_TRY(cudaLaunchKernelEx(&cfg, topk_kernel, a), "topk launch");
  return AOAKV_OK;
}

}  // namespace aoakv

using namespace aoakv;

extern "C" int aoakv_topk_filtering(
    const void* scores, int32_t scores_dtype, int64_t scores_row_stride,
    const int32_t* in_indices, int64_t in_indices_row_stride, int32_t num_rows,
    int32_t num_pages, int32_t k, void* out_values, int64_t out_values_row_stride,
    int32_t* out_indices, int64_t out_indices_row_stride, int32_t sink_first_page,
    void* stream) {
  AOAKV_NVTX("aoakv_topk_filtering");
  AOAKV_CHECK_ARG(scores != nullptr, "topk: scores is NULL");
  AOAKV_CHECK_ARG(out_values || out_indices, "topk: no output requested");
  AOAKV_CHECK_ARG(scores_dtype == AOAKV_DTYPE_F16 || scores_dtype == AOAKV_DTYPE_F32,
                  "topk: scores_dtype must be F16 or F32");
  AOAKV_CHECK_ARG(num_rows >= 1, "topk: num_rows must be >= 1");
  AOAKV_CHECK_ARG(num_pages >= 1 && num_pages <= kTopkMaxN,
                  "topk: num_pages must be in [1, 49152]");
  AOAKV_CHECK_ARG(k >= 1 && k <= num_pages, "topk: k must be in [1, num_pages]");
  AOAKV_CHECK_ARG(scores_row_stride >= num_pages || num_rows == 1,
                  "topk: scores_row_stride below num_pages");
  AOAKV_CHECK_ARG(!in_indices || in_indices_row_stride == 0 ||
                      in_indices_row_stride >= num_pages,
                  "topk: in_indices_row_stride must be 0 or >= num_pages");
  AOAKV_CHECK_ARG(!out_values || out_values_row_stride >= k || num_rows == 1,
                  "topk: out_values_row_stride below k");
  AOAKV_CHECK_ARG(!out_indices || out_indices_row_stride >= k || num_rows == 1,
                  "topk: out_indices_row_stride below k");
  TopkArgs a;
  a.scores = scores;
  a.s_stride = scores_row_stride;
  a.in_idx = in_indices;
  a.in_stride = in_indices_row_stride;
  a.out_vals = out_values;
  a.ov_stride = out_values_row_stride;
  a.out_idx = out_indices;
  a.oi_stride = out_indices_row_stride;
  a.f32 = scores_dtype == AOAKV_DTYPE_F32;
  a.n = num_pages;
  a.k = k;
  a.sink = sink_first_page != 0;
  return launch_topk(a, num_rows, static_cast<cudaStream_t>(stream), false);
}
