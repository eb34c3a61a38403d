// a5 stand-alone entry points: aoakv_decode_workspace_size, aoakv_sparse_decode.
#include <cudaTypedefs.h>

#include <cmath>
#include <mutex>

#include "decode.cuh"
#include "plan.h"

namespace aoakv {
namespace {

template <int D>
__global__ void __launch_bounds__(kDecThreads)
    sparse_decode_kernel(const __grid_constant__ CUtensorMap tmap, DecodeArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align_smem<128>(smem_raw);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem);
  int* tok = reinterpret_cast<int*>(smem + 64);
  int* flag = tok + kDecMaxChunk;
  float* mrg = reinterpret_cast<float*>(smem + kDecHeader);
  __half* tiles = reinterpret_cast<__half*>(smem + dec_tile_offset(D));
  const int c = blockIdx.x, h = blockIdx.y;
  if (threadIdx.x == 0) {
    for (int j = 0; j < kDecMaxChunk; ++j) mbar_init(&bars[j], 1);
    fence_mbar_init();
    tma_prefetch_desc(&tmap);
  }
  __syncthreads();
  pdl_wait();  // indices may be produced by the previous kernel
  if (threadIdx.x == 0) decode_issue(a, &tmap, h, c, bars, tok, tiles, D);
  __syncthreads();
  decode_compute<D>(a, h, c, bars, tok, tiles, mrg, flag, 0u);
}

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000,
                                         cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

}  // namespace

int make_kv_tmap(CUtensorMap* map, const void* kv, int H, int D, int P, int cap) {
  auto fn = encode_fn();
  if (!fn) return set_error(AOAKV_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
  if (reinterpret_cast<uintptr_t>(kv) % 16)
    return set_error(AOAKV_ERR_INVALID_ARG, "kv_data must be 16-byte aligned");
  cuuint64_t dims[3] = {static_cast<cuuint64_t>(D), static_cast<cuuint64_t>(H),
                        static_cast<cuuint64_t>(cap) * 2 * P};
  cuuint64_t strides[2] = {static_cast<cuuint64_t>(D) * 2,
                           static_cast<cuuint64_t>(H) * D * 2};
  cuuint32_t box[3] = {static_cast<cuuint32_t>(D), 1u, static_cast<cuuint32_t>(P)};
  cuuint32_t estr[3] = {1u, 1u, 1u};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, const_cast<void*>(kv),
                  dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return set_error(AOAKV_ERR_CUDA,
                     "cuTensorMapEncodeTiled failed with CUresult " + std::to_string(r));
  return AOAKV_OK;
}

int make_kv_tmap_sw128(CUtensorMap* map, const void* kv, int H, int D, int P, int cap) {
  auto fn = encode_fn();
  if (!fn) return set_error(AOAKV_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
  if (reinterpret_cast<uintptr_t>(kv) % 16)
    return set_error(AOAKV_ERR_INVALID_ARG, "kv_data must be 16-byte aligned");
  if (D % 64)
    return set_error(AOAKV_ERR_UNSUPPORTED, "swizzled page tiles need head_dim % 64 == 0");
  cuuint64_t dims[3] = {static_cast<cuuint64_t>(D), static_cast<cuuint64_t>(H),
                        static_cast<cuuint64_t>(cap) * 2 * P};
  cuuint64_t strides[2] = {static_cast<cuuint64_t>(D) * 2,
                           static_cast<cuuint64_t>(H) * D * 2};
  cuuint32_t box[3] = {64u, 1u, static_cast<cuuint32_t>(P)};
  cuuint32_t estr[3] = {1u, 1u, 1u};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, const_cast<void*>(kv), dims, strides,
                  box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return set_error(AOAKV_ERR_CUDA,
                     "cuTensorMapEncodeTiled (swizzled) failed with CUresult " + std::to_string(r));
  return AOAKV_OK;
}

int make_q_tmap_sw128(CUtensorMap* map, const void* q, int H, int D, int rows) {
  auto fn = encode_fn();
  if (!fn) return set_error(AOAKV_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
  if (reinterpret_cast<uintptr_t>(q) % 16)
    return set_error(AOAKV_ERR_INVALID_ARG, "q must be 16-byte aligned");
  if (D % 64) return set_error(AOAKV_ERR_UNSUPPORTED, "swizzled q tiles need head_dim % 64 == 0");
  cuuint64_t dims[3] = {static_cast<cuuint64_t>(D), static_cast<cuuint64_t>(H),
                        static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[2] = {static_cast<cuuint64_t>(D) * 2,
                           static_cast<cuuint64_t>(H) * D * 2};
  cuuint32_t box[3] = {64u, 1u, 128u};
  cuuint32_t estr[3] = {1u, 1u, 1u};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, const_cast<void*>(q), dims, strides,
                  box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return set_error(AOAKV_ERR_CUDA,
                     "cuTensorMapEncodeTiled (q rows) failed with CUresult " + std::to_string(r));
  return AOAKV_OK;
}

int make_meta_tmap(CUtensorMap* map, const void* meta, int H, int D, int P, int meta_cap,
                   int box_heads) {
  auto fn = encode_fn();
  if (!fn) return set_error(AOAKV_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
  if (reinterpret_cast<uintptr_t>(meta) % 16)
    return set_error(AOAKV_ERR_INVALID_ARG, "metadata_data must be 16-byte aligned");
  if (H > 256 || D > 256)
    return set_error(AOAKV_ERR_UNSUPPORTED, "metadata tensor map: heads or head_dim above 256");
  cuuint64_t dims[3] = {static_cast<cuuint64_t>(D), static_cast<cuuint64_t>(H),
                        static_cast<cuuint64_t>(meta_cap) * 2 * P};
  cuuint64_t strides[2] = {static_cast<cuuint64_t>(D) * 2,
                           static_cast<cuuint64_t>(H) * D * 2};
  cuuint32_t box[3] = {static_cast<cuuint32_t>(D), static_cast<cuuint32_t>(box_heads), 1u};
  cuuint32_t estr[3] = {1u, 1u, 1u};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, const_cast<void*>(meta), dims,
                  strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return set_error(AOAKV_ERR_CUDA,
                     "cuTensorMapEncodeTiled (metadata) failed with CUresult " + std::to_string(r));
  return AOAKV_OK;
}

DecodePlan plan_decode(int H, int n_slots, int D, int P) {
  DecodePlan pl;
  const int64_t target = static_cast<int64_t>(num_sms()) * 4;
  int64_t c = (static_cast<int64_t>(H) * n_slots + target - 1) / target;
  int cmax = static_cast<int>((100 * 1024 - dec_tile_offset(D)) / (4LL * P * D));
  if (cmax > kDecMaxChunk) cmax = kDecMaxChunk;
  if (cmax < 1) cmax = 1;
  if (c < 1) c = 1;
  if (c > cmax) c = cmax;
  pl.chunk_pages = static_cast<int>(c);
  pl.n_chunks = (n_slots + pl.chunk_pages - 1) / pl.chunk_pages;
  pl.smem = dec_smem_bytes(D, P, pl.chunk_pages) + 128;  // + alignment slack
  return pl;
}

size_t decode_ws_bytes(int H, int D, int max_slots) {
  auto up = [](size_t x) { return (x + 255) / 256 * 256; };
  return up(static_cast<size_t>(H) * 4) + up(static_cast<size_t>(H) * max_slots * 8) +
         up(static_cast<size_t>(H) * max_slots * D * 4);
}

void carve_decode_ws(void* ws, int H, int D, int max_slots, DecodeArgs& a) {
  auto up = [](size_t x) { return (x + 255) / 256 * 256; };
  uint8_t* p = static_cast<uint8_t*>(ws);
  a.ws_cnt = reinterpret_cast<int*>(p);
  p += up(static_cast<size_t>(H) * 4);
  a.ws_ml = reinterpret_cast<float2*>(p);
  p += up(static_cast<size_t>(H) * max_slots * 8);
  a.ws_o = reinterpret_cast<float*>(p);
}

int launch_decode(const DecodeArgs& a, const CUtensorMap& tmap, int D,
                  const DecodePlan& pl, cudaStream_t s, bool pdl) {
  const void* fn = D == 128 ? reinterpret_cast<const void*>(sparse_decode_kernel<128>)
                            : reinterpret_cast<const void*>(sparse_decode_kernel<64>);
  if (pl.smem > 48 * 1024)
    AOAKV_CUDA_TRY(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        static_cast<int>(pl.smem)),
                   "decode smem attribute");
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(pl.n_chunks, a.H);
  cfg.blockDim = dim3(kDecThreads);
  cfg.dynamicSmemBytes = pl.smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = pdl ? 1 : 0;
  if (D == 128)
    AOAKV_CUDA_TRY(cudaLaunchKernelEx(&cfg, sparse_decode_kernel<128>, tmap, a),
                   "decode launch");
  else
    AOAKV_CUDA_TRY(cudaLaunchKernelEx(&cfg, sparse_decode_kernel<64>, tmap, a),
                   "decode launch");
  return AOAKV_OK;
}

int check_decode_shape(int H, int D, int P, int kv_cap, int layout) {
  if (layout != AOAKV_LAYOUT_NHD)
    return set_error(AOAKV_ERR_UNSUPPORTED, "decode: only the NHD layout is built");
  AOAKV_CHECK_ARG(D == 64 || D == 128, "decode: head_dim must be 64 or 128");
  AOAKV_CHECK_ARG(H >= 1 && H <= 65535, "decode: num_heads out of range");
  AOAKV_CHECK_ARG(P >= 1 && P <= 256, "decode: page_size must be in [1, 256]");
  AOAKV_CHECK_ARG(kv_cap >= 1 && static_cast<int64_t>(kv_cap) * 2 * P < (1LL << 31),
                  "decode: kv_capacity_pages out of range");
  return AOAKV_OK;
}

}  // namespace aoakv

using namespace aoakv;

extern "C" int aoakv_decode_workspace_size(int32_t num_heads, int32_t head_dim,
                                           int32_t max_pages_per_head, size_t* bytes) {
  AOAKV_CHECK_ARG(bytes != nullptr, "decode_workspace_size: bytes is NULL");
  AOAKV_CHECK_ARG(num_heads >= 1 && (head_dim == 64 || head_dim == 128) &&
                      max_pages_per_head >= 0,
                  "decode_workspace_size: bad arguments");
  *bytes = decode_ws_bytes(num_heads, head_dim, max_pages_per_head + 1);
  return AOAKV_OK;
}

namespace {

// Shared body of aoakv_sparse_decode (fp16 o) and aoakv_sparse_decode_partial
// (fp32 o plus lse; last_page_idx -1 = no last page on this shard).
int sparse_decode_impl(const void* q, void* o, float* o_f32, float* lse, const void* kv_data,
                       int32_t kv_capacity_pages, const int32_t* indices,
                       int64_t indices_row_stride, int32_t num_selected, int32_t last_page_idx,
                       int32_t last_page_len, int32_t num_heads, int32_t head_dim,
                       int32_t page_size, int32_t layout, float sm_scale, void* workspace,
                       size_t workspace_bytes, void* stream, bool allow_no_last) {
  AOAKV_NVTX("aoakv_sparse_decode");
  int rc = check_decode_shape(num_heads, head_dim, page_size, kv_capacity_pages, layout);
  if (rc) return rc;
  AOAKV_CHECK_ARG(num_selected >= 0, "decode: num_selected must be >= 0");
  AOAKV_CHECK_ARG(num_selected == 0 || indices, "decode: indices is NULL");
  AOAKV_CHECK_ARG(indices_row_stride == 0 || indices_row_stride >= num_selected,
                  "decode: indices_row_stride must be 0 or >= num_selected");
  AOAKV_CHECK_ARG(last_page_len >= 1 && last_page_len <= page_size,
                  "decode: last_page_len must be in [1, page_size]");
  AOAKV_CHECK_ARG((last_page_idx >= 0 && last_page_idx < kv_capacity_pages) ||
                      (allow_no_last && last_page_idx == -1),
                  "decode: last_page_idx out of range");
  const int n_slots = num_selected + 1;
  DecodePlan pl = plan_decode(num_heads, n_slots, head_dim, page_size);
  DecodeArgs a = {};
  a.q = static_cast<const __half*>(q);
  a.o = static_cast<__half*>(o);
  a.o_f32 = o_f32;
  a.lse = lse;
  a.indices = indices;
  a.idx_stride = indices_row_stride;
  a.n_sel = num_selected;
  a.last_page = last_page_idx;
  a.last_len = last_page_len;
  a.H = num_heads;
  a.P = page_size;
  a.kv_cap = kv_capacity_pages;
  a.chunk_pages = pl.chunk_pages;
  a.n_chunks = pl.n_chunks;
  const float sc = sm_scale > 0.f ? sm_scale : 1.f / std::sqrt(static_cast<float>(head_dim));
  a.scale_log2 = sc * 1.4426950408889634f;
  a.err = dev_error_ptr();
  if (pl.n_chunks > 1) {
    const size_t need = decode_ws_bytes(num_heads, head_dim, n_slots);
    if (!workspace || workspace_bytes < need)
      return set_error(AOAKV_ERR_WORKSPACE,
                       "decode: workspace must hold aoakv_decode_workspace_size(" +
                           std::to_string(num_heads) + ", " + std::to_string(head_dim) +
                           ", " + std::to_string(num_selected) + ") = " +
                           std::to_string(need) + " bytes");
    carve_decode_ws(workspace, num_heads, head_dim, n_slots, a);
  }
  CUtensorMap tmap;
  rc = make_kv_tmap(&tmap, kv_data, num_heads, head_dim, page_size, kv_capacity_pages);
  if (rc) return rc;
  return launch_decode(a, tmap, head_dim, pl, static_cast<cudaStream_t>(stream), false);
}

}  // namespace

extern "C" int aoakv_sparse_decode(const void* q, void* o, const void* kv_data,
                                   int32_t kv_capacity_pages, const int32_t* indices,
                                   int64_t indices_row_stride, int32_t num_selected,
                                   int32_t last_page_idx, int32_t last_page_len,
                                   int32_t num_heads, int32_t head_dim, int32_t page_size,
                                   int32_t layout, float sm_scale, void* workspace,
                                   size_t workspace_bytes, void* stream) {
  AOAKV_CHECK_ARG(q && o && kv_data, "decode: NULL pointer argument");
  return sparse_decode_impl(q, o, nullptr, nullptr, kv_data, kv_capacity_pages, indices,
                            indices_row_stride, num_selected, last_page_idx, last_page_len,
                            num_heads, head_dim, page_size, layout, sm_scale, workspace,
                            workspace_bytes, stream, false);
}

extern "C" int aoakv_sparse_decode_partial(
    const void* q, float* o_partial, float* lse, const void* kv_data, int32_t kv_capacity_pages,
    const int32_t* indices, int64_t indices_row_stride, int32_t num_selected,
    int32_t last_page_idx, int32_t last_page_len, int32_t num_heads, int32_t head_dim,
    int32_t page_size, int32_t layout, float sm_scale, void* workspace, size_t workspace_bytes,
    void* stream) {
  AOAKV_CHECK_ARG(q && o_partial && lse && kv_data, "decode_partial: NULL pointer argument");
  return sparse_decode_impl(q, nullptr, o_partial, lse, kv_data, kv_capacity_pages, indices,
                            indices_row_stride, num_selected, last_page_idx, last_page_len,
                            num_heads, head_dim, page_size, layout, sm_scale, workspace,
                            workspace_bytes, stream, true);
}
