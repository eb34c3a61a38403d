// aoakv_sparse_decode_noalloc: the split-KV sparse decode for callers that
// cannot allocate device memory.
//
// Who needs it: a serving engine that reserves all device memory for its own
// pool at start-up, so that any later cudaMalloc fails or is forbidden; a
// plugin whose host runtime owns every allocation and gives its plugins no
// allocator; a latency-critical caller that must not risk the device-wide
// synchronisation cudaMalloc/cudaFree can cause. aoakv_sparse_decode needs a
// caller-provided workspace for the partial softmax states of its page
// chunks; this variant keeps them in a fixed device array that the library
// owns instead.
//
// The limit: the partial states of one call, num_heads x chunks x
// (8 + 4 * head_dim) bytes plus the tickets, must fit the array; a chunk holds
// up to 8 pages. For 32 heads of head_dim 128 that is num_selected <= 503
// pages (about 8,000 tokens at page size 16); larger problems are refused.
//
// The array is a file-scope __device__ variable of kScratchBytes (1 MiB). It
// exists once per GPU that loads the library and lives until the process
// exits. Host code cannot use the array's name as a device address, so the
// first call on each device resolves the address with cudaGetSymbolAddress
// while that device is current, and caches it; make that first call before
// any stream capture. Because every call shares the
// one array, calls whose kernels overlap on the GPU (two streams, or two host
// threads on one device) race on it: serialise them. The chunk tickets at the
// start of the array must be zero when a call starts; each call clears them
// with cudaMemsetAsync on its own stream before launching.
#include <cmath>
#include <mutex>

#include "decode.cuh"
#include "plan.h"

namespace aoakv {

constexpr size_t kScratchBytes = size_t(1) << 20;
static __device__ __align__(256) unsigned char g_decode_scratch[kScratchBytes];

namespace {

constexpr int kMaxDev = 64;
std::mutex g_scratch_mu;
void* g_scratch_addr[kMaxDev] = {nullptr};

// Device address of g_decode_scratch on the current device (set-up on the
// first call per device).
int scratch_address(void** out) {
  int dev = 0;
  AOAKV_CUDA_TRY(cudaGetDevice(&dev), "noalloc decode: cudaGetDevice");
  if (dev < 0 || dev >= kMaxDev)
    return set_error(AOAKV_ERR_UNSUPPORTED, "noalloc decode: device ordinal above 63");
  std::lock_guard<std::mutex> lk(g_scratch_mu);
  if (!g_scratch_addr[dev]) {
    void* p = nullptr;
    AOAKV_CUDA_TRY(cudaGetSymbolAddress(&p, g_decode_scratch),
                   "noalloc decode: cudaGetSymbolAddress(g_decode_scratch)");
    g_scratch_addr[dev] = p;
  }
  *out = g_scratch_addr[dev];
  return AOAKV_OK;
}

}  // namespace
}  // namespace aoakv

using namespace aoakv;

extern "C" int aoakv_sparse_decode_noalloc(const void* q, void* o, const void* kv_data,
                                           int32_t kv_capacity_pages, const int32_t* indices,
                                           int64_t indices_row_stride, int32_t num_selected,
                                           int32_t last_page_idx, int32_t last_page_len,
                                           int32_t num_heads, int32_t head_dim,
                                           int32_t page_size, int32_t layout, float sm_scale,
                                           void* stream) {
  AOAKV_NVTX("aoakv_sparse_decode_noalloc");
  AOAKV_CHECK_ARG(q && o && kv_data, "noalloc decode: NULL pointer argument");
  int rc = check_decode_shape(num_heads, head_dim, page_size, kv_capacity_pages, layout);
  if (rc) return rc;
  AOAKV_CHECK_ARG(num_selected >= 0, "noalloc decode: num_selected must be >= 0");
  AOAKV_CHECK_ARG(num_selected == 0 || indices, "noalloc decode: indices is NULL");
  AOAKV_CHECK_ARG(indices_row_stride == 0 || indices_row_stride >= num_selected,
                  "noalloc decode: indices_row_stride must be 0 or >= num_selected");
  AOAKV_CHECK_ARG(last_page_len >= 1 && last_page_len <= page_size,
                  "noalloc decode: last_page_len must be in [1, page_size]");
  AOAKV_CHECK_ARG(last_page_idx >= 0 && last_page_idx < kv_capacity_pages,
                  "noalloc decode: last_page_idx out of range");
  const DecodePlan pl = plan_decode(num_heads, num_selected + 1, head_dim, page_size);
  // The partial states need one (max, sum, numerator) record per head and chunk.
  const size_t need = decode_ws_bytes(num_heads, head_dim, pl.n_chunks);
  if (need > kScratchBytes)
    return set_error(AOAKV_ERR_UNSUPPORTED,
                     "noalloc decode: " + std::to_string(num_heads) + " heads x " +
                         std::to_string(pl.n_chunks) + " chunks need " + std::to_string(need) +
                         " bytes of scratch, above the fixed 1 MiB; use aoakv_sparse_decode "
                         "with a workspace");
  void* scratch = nullptr;
  rc = scratch_address(&scratch);
  if (rc) return rc;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  DecodeArgs a = {};
  a.q = static_cast<const __half*>(q);
  a.o = static_cast<__half*>(o);
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
    carve_decode_ws(scratch, num_heads, head_dim, pl.n_chunks, a);
    AOAKV_CUDA_TRY(cudaMemsetAsync(a.ws_cnt, 0, static_cast<size_t>(num_heads) * sizeof(int), s),
                   "noalloc decode: clear chunk tickets");
  }
  CUtensorMap tmap;
  rc = make_kv_tmap(&tmap, kv_data, num_heads, head_dim, page_size, kv_capacity_pages);
  if (rc) return rc;
  return launch_decode(a, tmap, head_dim, pl, s, false);
}
