// a1 / a2: KV append fused with the per-page key max/min metadata and the
// page value log-norm.
//
// Reference behaviour followed (kernels/aoa_kv/kernels/include/decode/):
//   decode_page.cuh:392-506  decode append: running max/min of the last page
//                            (init -/+65504 when the token opens the page,
//                            :425-435); on page fill v_log_norm =
//                            log(||(1/P) sum_e V_e||_2 + 1e-6) (:459-504).
//   decode_page.cuh:522-692  prefill append: same, for a ragged run of
//                            tokens; partial pages get max/min only.
// Design: the decode append is latency-bound (one token); it runs one
// 16-byte vector per thread over all (head, channel-group) pairs. The
// prefill append gives every touched page its own CTA (the reference uses
// one CTA per head for the whole prompt) and accumulates the V mean in
// registers while copying, so V is read once.
#include "common.cuh"

namespace aoakv {
namespace {

constexpr float kHalfMax = 65504.f;

struct AppendArgs {
  const __half* k;  // [S, H, D]
  const __half* v;
  __half* kv;       // [kv_cap, 2, P, H, D]
  const int32_t* kv_indices;
  __half* meta;     // [meta_cap, 2, P, H, D]
  const int32_t* meta_indices;
  __half* vlog;     // [kv_cap, H]
  int* err;
  int H, P;
  int kv_cap, meta_cap;
  int n_pages;      // pages of the sequence including the new tokens
  int seq_total;    // tokens including the new ones
  int seq_new;      // tokens being appended (1 for decode)
};

__device__ __forceinline__ size_t row_off(int page, int kv, int entry, int h,
                                          int H, int P, int D) {
  return ((static_cast<size_t>(page) * 2 + kv) * P + entry) *
             static_cast<size_t>(H) * D +
         static_cast<size_t>(h) * D;
}

__device__ __forceinline__ void hmax8(uint4& m, const uint4& x) {
  __half2* a = reinterpret_cast<__half2*>(&m);
  const __half2* b = reinterpret_cast<const __half2*>(&x);
#pragma unroll
  for (int i = 0; i < 4; ++i) a[i] = __hmax2(a[i], b[i]);
}
__device__ __forceinline__ void hmin8(uint4& m, const uint4& x) {
  __half2* a = reinterpret_cast<__half2*>(&m);
  const __half2* b = reinterpret_cast<const __half2*>(&x);
#pragma unroll
  for (int i = 0; i < 4; ++i) a[i] = __hmin2(a[i], b[i]);
}
__device__ __forceinline__ uint4 fill8(float x) {
  __half2 h = __float2half2_rn(x);
  uint4 r;
  r.x = r.y = r.z = r.w = *reinterpret_cast<uint32_t*>(&h);
  return r;
}
__device__ __forceinline__ void acc8(float s[8], const uint4& x) {
  float f[8];
  u4_to_f8(x, f);
#pragma unroll
  for (int i = 0; i < 8; ++i) s[i] += f[i];
}

// Sum over the L lanes of one (page, head) group; L divides 32 and groups
// are lane-aligned, so xor offsets < L stay inside the group.
template <int L>
__device__ __forceinline__ float group_sum(float x) {
#pragma unroll
  for (int off = L / 2; off > 0; off >>= 1)
    x += __shfl_xor_sync(0xffffffffu, x, off);
  return x;
}

// Squared L2 norm of this lane's 8 channels of the page mean sum/P.
__device__ __forceinline__ float mean_sq_norm(const float s[8], float inv_p) {
  float l2 = 0.f;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    float m = s[i] * inv_p;
    l2 += m * m;
  }
  return l2;
}

// One new token; thread t owns (head t / L, channels 8*(t % L) .. +8).
template <int D>
__global__ void __launch_bounds__(128) append_decode_kernel(AppendArgs a) {
  constexpr int L = D / 8;
  const int t = blockIdx.x * blockDim.x + threadIdx.x;
  const int h = t / L, lane = t % L;
  const bool active = h < a.H;
  const int page_iter = a.n_pages - 1;
  const int entry = (a.seq_total - 1) % a.P;
  const int meta_iter = page_iter / a.P;
  const int meta_entry = page_iter % a.P;

  int pid = 0, mpid = 0;
  bool ok = active;
  if (active) {
    pid = __ldg(a.kv_indices + page_iter);
    mpid = __ldg(a.meta_indices + meta_iter);
    if (pid < 0 || pid >= a.kv_cap || mpid < 0 || mpid >= a.meta_cap) {
      raise_dev_error(a.err, AOAKV_DEV_ERR_BAD_PAGE);
      ok = false;
    }
  }
  uint4 vv = make_uint4(0, 0, 0, 0);
  if (ok) {
    const size_t src = static_cast<size_t>(h) * D + lane * 8;
    const uint4 kk = *reinterpret_cast<const uint4*>(a.k + src);
    vv = *reinterpret_cast<const uint4*>(a.v + src);
    const size_t mk = row_off(mpid, 0, meta_entry, h, a.H, a.P, D) + lane * 8;
    const size_t mv = row_off(mpid, 1, meta_entry, h, a.H, a.P, D) + lane * 8;
    uint4 mx, mn;
    if (entry > 0) {
      mx = *reinterpret_cast<const uint4*>(a.meta + mk);
      mn = *reinterpret_cast<const uint4*>(a.meta + mv);
    } else {
      mx = fill8(-kHalfMax);
      mn = fill8(kHalfMax);
    }
    hmax8(mx, kk);
    hmin8(mn, kk);
    *reinterpret_cast<uint4*>(a.kv + row_off(pid, 0, entry, h, a.H, a.P, D) +
                              lane * 8) = kk;
    *reinterpret_cast<uint4*>(a.kv + row_off(pid, 1, entry, h, a.H, a.P, D) +
                              lane * 8) = vv;
    *reinterpret_cast<uint4*>(a.meta + mk) = mx;
    *reinterpret_cast<uint4*>(a.meta + mv) = mn;
  }
  if (entry + 1 == a.P) {  // uniform across the grid
    float s[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    if (ok) {  // the page's earlier V rows: 8 loads in flight, summed in order
      for (int e0 = 0; e0 + 1 < a.P; e0 += 8) {
        uint4 r[8];
#pragma unroll
        for (int u = 0; u < 8; ++u)
          if (e0 + u + 1 < a.P)
            r[u] = ld_stream_u4(a.kv + row_off(pid, 1, e0 + u, h, a.H, a.P, D) + lane * 8);
#pragma unroll
        for (int u = 0; u < 8; ++u)
          if (e0 + u + 1 < a.P) acc8(s, r[u]);
      }
      acc8(s, vv);
    }
    float l2 = group_sum<L>(mean_sq_norm(s, 1.f / a.P));
    if (ok && lane == 0)
      a.vlog[static_cast<size_t>(pid) * a.H + h] =
          __float2half_rn(logf(sqrtf(l2) + 1e-6f));
  }
}

// Prefill: CTA b owns logical page p0 + b; threads sweep (head, lane) pairs.
template <int D>
__global__ void __launch_bounds__(256) append_prefill_kernel(AppendArgs a,
                                                             int first_page) {
  constexpr int L = D / 8;
  const int p = first_page + blockIdx.x;
  const int start_seq = a.seq_total - a.seq_new;
  const int e0 = max(0, start_seq - p * a.P);
  const int e1 = min(a.P, a.seq_total - p * a.P);
  const int pid = __ldg(a.kv_indices + p);
  const int mpid = __ldg(a.meta_indices + p / a.P);
  const int mentry = p % a.P;
  if (pid < 0 || pid >= a.kv_cap || mpid < 0 || mpid >= a.meta_cap) {
    if (threadIdx.x == 0) raise_dev_error(a.err, AOAKV_DEV_ERR_BAD_PAGE);
    return;  // uniform over the CTA
  }
  const int pairs = a.H * L;
  for (int base = 0; base < pairs; base += blockDim.x) {
    const int pair = base + threadIdx.x;
    const bool active = pair < pairs;
    const int h = active ? pair / L : 0;
    const int lane = pair % L;
    float s[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    if (active) {
      const size_t mk = row_off(mpid, 0, mentry, h, a.H, a.P, D) + lane * 8;
      const size_t mv = row_off(mpid, 1, mentry, h, a.H, a.P, D) + lane * 8;
      uint4 mx, mn;
      if (e0 > 0) {
        mx = *reinterpret_cast<const uint4*>(a.meta + mk);
        mn = *reinterpret_cast<const uint4*>(a.meta + mv);
        if (e1 == a.P)  // page completes: older entries join the V mean first
          for (int e = 0; e < e0; ++e)
            acc8(s, *reinterpret_cast<const uint4*>(
                        a.kv + row_off(pid, 1, e, h, a.H, a.P, D) + lane * 8));
      } else {
        mx = fill8(-kHalfMax);
        mn = fill8(kHalfMax);
      }
      const size_t tok_stride = static_cast<size_t>(a.H) * D;
      // Entry e of page p is input token p*P + e - start_seq (>= 0 for e >= e0).
      const long long tok0 = static_cast<long long>(p) * a.P - start_seq;
      const size_t col = static_cast<size_t>(h) * D + lane * 8;
#define AOAKV_SRC(e) (static_cast<size_t>(tok0 + (e)) * tok_stride + col)
      int e = e0;
      for (; e + 4 <= e1; e += 4) {
        uint4 kk[4], vv[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          kk[u] = ld_stream_u4(a.k + AOAKV_SRC(e + u));
          vv[u] = ld_stream_u4(a.v + AOAKV_SRC(e + u));
        }
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          hmax8(mx, kk[u]);
          hmin8(mn, kk[u]);
          acc8(s, vv[u]);
          *reinterpret_cast<uint4*>(
              a.kv + row_off(pid, 0, e + u, h, a.H, a.P, D) + lane * 8) = kk[u];
          *reinterpret_cast<uint4*>(
              a.kv + row_off(pid, 1, e + u, h, a.H, a.P, D) + lane * 8) = vv[u];
        }
      }
      for (; e < e1; ++e) {
        const uint4 kk = ld_stream_u4(a.k + AOAKV_SRC(e));
        const uint4 vv = ld_stream_u4(a.v + AOAKV_SRC(e));
        hmax8(mx, kk);
        hmin8(mn, kk);
        acc8(s, vv);
        *reinterpret_cast<uint4*>(a.kv + row_off(pid, 0, e, h, a.H, a.P, D) +
                                  lane * 8) = kk;
        *reinterpret_cast<uint4*>(a.kv + row_off(pid, 1, e, h, a.H, a.P, D) +
                                  lane * 8) = vv;
      }
#undef AOAKV_SRC
      *reinterpret_cast<uint4*>(a.meta + mk) = mx;
      *reinterpret_cast<uint4*>(a.meta + mv) = mn;
    }
    if (e1 == a.P) {  // uniform over the CTA
      float l2 = group_sum<L>(mean_sq_norm(s, 1.f / a.P));
      if (active && lane == 0)
        a.vlog[static_cast<size_t>(pid) * a.H + h] =
            __float2half_rn(logf(sqrtf(l2) + 1e-6f));
    }
  }
}

int check_common(const void* k, const void* v, void* kv_data,
                 const int32_t* kv_indices, int32_t num_kv_pages,
                 int32_t kv_last_page_len, int32_t kv_cap, void* meta,
                 const int32_t* meta_indices, int32_t num_meta_pages,
                 int32_t meta_last_len, int32_t meta_cap, void* vlog,
                 int32_t H, int32_t D, int32_t P, int32_t layout) {
  AOAKV_CHECK_ARG(k && v && kv_data && kv_indices && meta && meta_indices && vlog,
                  "append: NULL pointer argument");
  if (layout != AOAKV_LAYOUT_NHD)
    return set_error(AOAKV_ERR_UNSUPPORTED, "append: only the NHD layout is built");
  AOAKV_CHECK_ARG(D == 64 || D == 128, "append: head_dim must be 64 or 128");
  AOAKV_CHECK_ARG(H >= 1 && H <= 4096, "append: num_heads out of range");
  AOAKV_CHECK_ARG(P >= 1 && P <= 1024, "append: page_size out of range");
  AOAKV_CHECK_ARG(num_kv_pages >= 1, "append: num_kv_pages must be >= 1");
  AOAKV_CHECK_ARG(kv_last_page_len >= 1 && kv_last_page_len <= P,
                  "append: kv_last_page_len must be in [1, page_size]");
  AOAKV_CHECK_ARG(kv_cap >= num_kv_pages, "append: kv capacity below num_kv_pages");
  AOAKV_CHECK_ARG(num_meta_pages == (num_kv_pages + P - 1) / P,
                  "append: num_metadata_pages != ceil(num_kv_pages / page_size)");
  AOAKV_CHECK_ARG(meta_last_len == (num_kv_pages - 1) % P + 1,
                  "append: metadata_last_page_len inconsistent with num_kv_pages");
  AOAKV_CHECK_ARG(meta_cap >= num_meta_pages,
                  "append: metadata capacity below num_metadata_pages");
  return AOAKV_OK;
}

}  // namespace
}  // namespace aoakv

using namespace aoakv;

extern "C" int aoakv_append_kv_cache_decode(
    const void* k, const void* v, void* kv_data, const int32_t* kv_indices,
    int32_t num_kv_pages, int32_t kv_last_page_len, int32_t kv_capacity_pages,
    void* metadata_data, const int32_t* metadata_indices,
    int32_t num_metadata_pages, int32_t metadata_last_page_len,
    int32_t metadata_capacity_pages, void* v_log_norm, int32_t num_heads,
    int32_t head_dim, int32_t page_size, int32_t layout, void* stream) {
  AOAKV_NVTX("aoakv_append_kv_cache_decode");
  int rc = check_common(k, v, kv_data, kv_indices, num_kv_pages,
                        kv_last_page_len, kv_capacity_pages, metadata_data,
                        metadata_indices, num_metadata_pages,
                        metadata_last_page_len, metadata_capacity_pages,
                        v_log_norm, num_heads, head_dim, page_size, layout);
  if (rc) return rc;
  AppendArgs a;
  a.k = static_cast<const __half*>(k);
  a.v = static_cast<const __half*>(v);
  a.kv = static_cast<__half*>(kv_data);
  a.kv_indices = kv_indices;
  a.meta = static_cast<__half*>(metadata_data);
  a.meta_indices = metadata_indices;
  a.vlog = static_cast<__half*>(v_log_norm);
  a.err = dev_error_ptr();
  a.H = num_heads;
  a.P = page_size;
  a.kv_cap = kv_capacity_pages;
  a.meta_cap = metadata_capacity_pages;
  a.n_pages = num_kv_pages;
  a.seq_total = (num_kv_pages - 1) * page_size + kv_last_page_len;
  a.seq_new = 1;
  const int threads = num_heads * (head_dim / 8);
  const int blocks = (threads + 127) / 128;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (head_dim == 128)
    append_decode_kernel<128><<<blocks, 128, 0, s>>>(a);
  else
    append_decode_kernel<64><<<blocks, 128, 0, s>>>(a);
  AOAKV_CUDA_TRY(cudaGetLastError(), "append_decode launch");
  return AOAKV_OK;
}

extern "C" int aoakv_append_kv_cache_prefill(
    const void* k, const void* v, int32_t seq_len, void* kv_data,
    const int32_t* kv_indices, int32_t num_kv_pages, int32_t kv_last_page_len,
    int32_t kv_capacity_pages, void* metadata_data,
    const int32_t* metadata_indices, int32_t num_metadata_pages,
    int32_t metadata_last_page_len, int32_t metadata_capacity_pages,
    void* v_log_norm, int32_t num_heads, int32_t head_dim, int32_t page_size,
    int32_t layout, void* stream) {
  AOAKV_NVTX("aoakv_append_kv_cache_prefill");
  int rc = check_common(k, v, kv_data, kv_indices, num_kv_pages,
                        kv_last_page_len, kv_capacity_pages, metadata_data,
                        metadata_indices, num_metadata_pages,
                        metadata_last_page_len, metadata_capacity_pages,
                        v_log_norm, num_heads, head_dim, page_size, layout);
  if (rc) return rc;
  const int64_t seq_total =
      static_cast<int64_t>(num_kv_pages - 1) * page_size + kv_last_page_len;
  AOAKV_CHECK_ARG(seq_len >= 1 && seq_len <= seq_total,
                  "append_prefill: seq_len must be in [1, sequence length]");
  AppendArgs a;
  a.k = static_cast<const __half*>(k);
  a.v = static_cast<const __half*>(v);
  a.kv = static_cast<__half*>(kv_data);
  a.kv_indices = kv_indices;
  a.meta = static_cast<__half*>(metadata_data);
  a.meta_indices = metadata_indices;
  a.vlog = static_cast<__half*>(v_log_norm);
  a.err = dev_error_ptr();
  a.H = num_heads;
  a.P = page_size;
  a.kv_cap = kv_capacity_pages;
  a.meta_cap = metadata_capacity_pages;
  a.n_pages = num_kv_pages;
  a.seq_total = static_cast<int>(seq_total);
  a.seq_new = seq_len;
  const int first_page = static_cast<int>((seq_total - seq_len) / page_size);
  const int blocks = num_kv_pages - first_page;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (head_dim == 128)
    append_prefill_kernel<128><<<blocks, 256, 0, s>>>(a, first_page);
  else
    append_prefill_kernel<64><<<blocks, 256, 0, s>>>(a, first_page);
  AOAKV_CUDA_TRY(cudaGetLastError(), "append_prefill launch");
  return AOAKV_OK;
}
