// Device-resident page table and page allocator (the reference keeps both
// on the host: quest/utils/kv_cache.py:7-133 KvPool / KvCache, and
// controller.py:82-141 builds index tensors from Python lists every step).
//
// One device buffer holds, for R sequences, each sequence's KV page list
// (room for M pages) and metadata page list (room for ceil(M / P)), its page
// count, last-page length and token count, plus the free stacks of the KV
// and metadata pools. Appending tokens allocates pages on the device, so a
// decode token (append + every layer's step) can be captured once as a CUDA
// graph and replayed: no host work and no host-to-device index copy per
// token. Counting follows KvCache.append_seq (kv_cache.py:115-126): a new
// page when the last page is full (or the sequence is empty); metadata
// pages count KV pages the same way (controller.py:82-87, prepare_metadata).
// Page ids come from a stack: a fresh pool hands out 0, 1, 2, ... like the
// reference's fresh set; released pages are handed out again last-released-
// first (the reference's set.pop order after frees is a hash detail).
#include <algorithm>
#include <new>

#include "common.cuh"
#include "page_table.h"

namespace aoakv {

PageTableLayout page_table_layout(int R, int M, int cap, int mcap, int P) {
  auto up4 = [](size_t x) { return (x + 3) / 4 * 4; };
  PageTableLayout L;
  L.R = R;
  L.M = M;
  L.Mm = (M + P - 1) / P;
  L.P = P;
  L.cap = cap;
  L.mcap = mcap;
  L.kv_top = 0;
  L.meta_top = 1;
  size_t o = 4;
  L.kv_start = o;
  o += up4(R);
  L.kv_end = o;
  o += up4(R);
  L.last_len = o;
  o += up4(R);
  L.seq_len = o;
  o += up4(R);
  L.meta_start = o;
  o += up4(R);
  L.meta_count = o;
  o += up4(R);
  L.kv_indices = o;
  o += up4(static_cast<size_t>(R) * M);
  L.meta_indices = o;
  o += up4(static_cast<size_t>(R) * L.Mm);
  L.kv_free = o;
  o += up4(cap);
  L.meta_free = o;
  o += up4(mcap);
  L.words = o;
  return L;
}

namespace {

__global__ void page_table_init_kernel(int32_t* t, PageTableLayout L) {
  const int stride = gridDim.x * blockDim.x;
  const int i0 = blockIdx.x * blockDim.x + threadIdx.x;
  for (int i = i0; i < L.cap; i += stride) t[L.kv_free + i] = L.cap - 1 - i;  // top pops 0 first
  for (int i = i0; i < L.mcap; i += stride) t[L.meta_free + i] = L.mcap - 1 - i;
  for (int r = i0; r < L.R; r += stride) {
    t[L.kv_start + r] = r * L.M;
    t[L.kv_end + r] = r * L.M;
    t[L.last_len + r] = L.P;  // an empty sequence's "last page" is full
    t[L.seq_len + r] = 0;
    t[L.meta_start + r] = r * L.Mm;
    t[L.meta_count + r] = 0;
  }
  if (i0 == 0) {
    t[L.kv_top] = L.cap;
    t[L.meta_top] = L.mcap;
  }
}

__device__ __forceinline__ int ceil_div(int a, int b) { return (a + b - 1) / b; }

// One thread, sequences in order (deterministic page ids). Per sequence:
// pages and metadata pages needed after num_tokens more tokens, popped from
// the free stacks; a sequence that would exceed its room or the pools is left
// unchanged and AOAKV_DEV_ERR_NO_PAGES is recorded.
__global__ void page_table_append_kernel(int32_t* t, PageTableLayout L, int seq_lo, int seq_hi,
                                         int num_tokens, int* err) {
  if (threadIdx.x != 0 || blockIdx.x != 0) return;
  int kv_top = t[L.kv_top], meta_top = t[L.meta_top];
  for (int r = seq_lo; r < seq_hi; ++r) {
    const int len = t[L.seq_len + r];
    const int n = t[L.kv_end + r] - t[L.kv_start + r];
    const int nm = t[L.meta_count + r];
    const int new_len = len + num_tokens;
    const int n_new = ceil_div(new_len, L.P);
    const int nm_new = ceil_div(n_new, L.P);
    const int need = n_new - n, need_m = nm_new - nm;
    if (n_new > L.M || need > kv_top || need_m > meta_top) {
      raise_dev_error(err, AOAKV_DEV_ERR_NO_PAGES);
      continue;
    }
    const int s = t[L.kv_start + r], sm = t[L.meta_start + r];
    for (int i = 0; i < need; ++i) t[L.kv_indices + s + n + i] = t[L.kv_free + --kv_top];
    for (int i = 0; i < need_m; ++i) t[L.meta_indices + sm + nm + i] = t[L.meta_free + --meta_top];
    t[L.kv_end + r] = s + n_new;
    t[L.meta_count + r] = nm_new;
    t[L.seq_len + r] = new_len;
    t[L.last_len + r] = new_len > 0 ? (new_len - 1) % L.P + 1 : L.P;
  }
  t[L.kv_top] = kv_top;
  t[L.meta_top] = meta_top;
}

// Pages back on the stacks, last page first (so they are handed out again
// in their old order), and the sequences emptied (kv_cache.py:128-133).
__global__ void page_table_release_kernel(int32_t* t, PageTableLayout L, int seq_lo,
                                          int seq_hi) {
  if (threadIdx.x != 0 || blockIdx.x != 0) return;
  int kv_top = t[L.kv_top], meta_top = t[L.meta_top];
  for (int r = seq_hi - 1; r >= seq_lo; --r) {
    const int s = t[L.kv_start + r], sm = t[L.meta_start + r];
    const int n = t[L.kv_end + r] - s, nm = t[L.meta_count + r];
    for (int i = n - 1; i >= 0; --i) t[L.kv_free + kv_top++] = t[L.kv_indices + s + i];
    for (int i = nm - 1; i >= 0; --i) t[L.meta_free + meta_top++] = t[L.meta_indices + sm + i];
    t[L.kv_end + r] = s;
    t[L.meta_count + r] = 0;
    t[L.seq_len + r] = 0;
    t[L.last_len + r] = L.P;
  }
  t[L.kv_top] = kv_top;
  t[L.meta_top] = meta_top;
}

int seq_range(const PageTable* pt, int seq, int* lo, int* hi) {
  AOAKV_CHECK_ARG(seq >= -1 && seq < pt->L.R, "page table: seq must be -1 (all) or in [0, R)");
  *lo = seq < 0 ? 0 : seq;
  *hi = seq < 0 ? pt->L.R : seq + 1;
  return AOAKV_OK;
}

}  // namespace
}  // namespace aoakv

using namespace aoakv;

extern "C" int aoakv_page_table_bytes(int32_t num_seqs, int32_t max_pages_per_seq,
                                      int32_t kv_capacity_pages, int32_t metadata_capacity_pages,
                                      int32_t page_size, size_t* bytes) {
  AOAKV_CHECK_ARG(bytes != nullptr, "page_table_bytes: bytes is NULL");
  AOAKV_CHECK_ARG(num_seqs >= 1 && num_seqs <= 65535 && max_pages_per_seq >= 1 &&
                      kv_capacity_pages >= 1 && metadata_capacity_pages >= 1 && page_size >= 1 &&
                      static_cast<int64_t>(num_seqs) * max_pages_per_seq < (1LL << 30),
                  "page_table_bytes: bad sizes");
  *bytes = page_table_layout(num_seqs, max_pages_per_seq, kv_capacity_pages,
                             metadata_capacity_pages, page_size).words * 4;
  return AOAKV_OK;
}

extern "C" int aoakv_page_table_create(aoakv_page_table* table_out, int32_t num_seqs,
                                       int32_t max_pages_per_seq, int32_t kv_capacity_pages,
                                       int32_t metadata_capacity_pages, int32_t page_size,
                                       void* device_buffer, size_t buffer_bytes, void* stream) {
  AOAKV_NVTX("aoakv_page_table_create");
  AOAKV_CHECK_ARG(table_out != nullptr && device_buffer != nullptr,
                  "page_table_create: NULL argument");
  size_t need = 0;
  int rc = aoakv_page_table_bytes(num_seqs, max_pages_per_seq, kv_capacity_pages,
                                  metadata_capacity_pages, page_size, &need);
  if (rc) return rc;
  AOAKV_CHECK_ARG(buffer_bytes >= need, "page_table_create: buffer smaller than "
                                        "aoakv_page_table_bytes");
  AOAKV_CHECK_ARG(reinterpret_cast<uintptr_t>(device_buffer) % 16 == 0,
                  "page_table_create: buffer must be 16-byte aligned");
  auto* pt = new (std::nothrow) PageTable;
  if (!pt) return set_error(AOAKV_ERR_CUDA, "page_table_create: out of host memory");
  pt->buf = static_cast<int32_t*>(device_buffer);
  pt->L = page_table_layout(num_seqs, max_pages_per_seq, kv_capacity_pages,
                            metadata_capacity_pages, page_size);
  const int n = std::max(std::max(kv_capacity_pages, metadata_capacity_pages), num_seqs);
  page_table_init_kernel<<<std::min((n + 255) / 256, 1024), 256, 0,
                           static_cast<cudaStream_t>(stream)>>>(pt->buf, pt->L);
  rc = cuda_status(cudaGetLastError(), "page table init launch");
  if (rc) {
    delete pt;
    return rc;
  }
  *table_out = reinterpret_cast<aoakv_page_table>(pt);
  return AOAKV_OK;
}

extern "C" int aoakv_page_table_destroy(aoakv_page_table table) {
  delete reinterpret_cast<PageTable*>(table);
  return AOAKV_OK;
}

extern "C" int aoakv_page_table_append(aoakv_page_table table, int32_t seq, int32_t num_tokens,
                                       void* stream) {
  AOAKV_NVTX("aoakv_page_table_append");
  AOAKV_CHECK_ARG(table != nullptr, "page_table_append: NULL table");
  AOAKV_CHECK_ARG(num_tokens >= 0, "page_table_append: num_tokens must be >= 0");
  auto* pt = reinterpret_cast<PageTable*>(table);
  int lo, hi;
  int rc = seq_range(pt, seq, &lo, &hi);
  if (rc) return rc;
  page_table_append_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(
      pt->buf, pt->L, lo, hi, num_tokens, dev_error_ptr());
  return cuda_status(cudaGetLastError(), "page table append launch");
}

extern "C" int aoakv_page_table_release(aoakv_page_table table, int32_t seq, void* stream) {
  AOAKV_NVTX("aoakv_page_table_release");
  AOAKV_CHECK_ARG(table != nullptr, "page_table_release: NULL table");
  auto* pt = reinterpret_cast<PageTable*>(table);
  int lo, hi;
  int rc = seq_range(pt, seq, &lo, &hi);
  if (rc) return rc;
  page_table_release_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(pt->buf, pt->L,
                                                                             lo, hi);
  return cuda_status(cudaGetLastError(), "page table release launch");
}

extern "C" int aoakv_page_table_layout(aoakv_page_table table, int64_t* words) {
  AOAKV_CHECK_ARG(table != nullptr && words != nullptr, "page_table_layout: NULL argument");
  const PageTableLayout& L = reinterpret_cast<PageTable*>(table)->L;
  const size_t v[16] = {L.kv_top,     L.meta_top,     L.kv_start,  L.kv_end,
                        L.last_len,   L.seq_len,      L.meta_start, L.meta_count,
                        L.kv_indices, L.meta_indices, L.kv_free,    L.meta_free,
                        L.words,      static_cast<size_t>(L.R), static_cast<size_t>(L.M),
                        static_cast<size_t>(L.Mm)};
  for (int i = 0; i < 16; ++i) words[i] = static_cast<int64_t>(v[i]);
  return AOAKV_OK;
}
