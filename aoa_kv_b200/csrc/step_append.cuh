// a1 inside the fused step kernels: one warp appends head h of the new
// token (decode_page.cuh:392-506): K and V into the last page, the page's
// key max/min (init -+65504 at entry 0), and on page fill the page's
// v_log_norm = log(||mean V||_2 + 1e-6) from the V rows re-read with 8
// loads in flight. Called by threads 0..31 of a CTA.
#pragma once

#include "fused.h"

namespace aoakv {

// The append's inputs that do not depend on the metadata page id — the new
// token's K and V rows and the last page's ids — copied to shared memory
// with cp.async at kernel start, so that the append itself costs one
// round trip (the metadata rows) when it runs later.
constexpr int kAppendStaged = 2;  // heads per CTA staged this way

struct AppendStage {
  uint4 kv[kAppendStaged][2][16];  // [head slot][k, v][D / 8 lanes], D <= 128
  int ids[2];                      // kv page id, metadata page id of the last page
};

__device__ __forceinline__ void cp_async_16(void* dst, const void* src) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 16;" ::"r"(smem_addr(dst)), "l"(src)
               : "memory");
}
__device__ __forceinline__ void cp_async_4(void* dst, const void* src) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(smem_addr(dst)), "l"(src)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() {
  asm volatile("cp.async.commit_group;" ::: "memory");
}

// Warp 0: start the copies for head h into slot `slot` (< kAppendStaged).
template <int D>
__device__ __forceinline__ void append_prefetch(const FusedArgs& f, int h, int slot,
                                                AppendStage& st) {
  constexpr int L = D / 8;
  const int lane = threadIdx.x;
  const size_t col = static_cast<size_t>(h) * D + lane * 8;
  if (lane < L) {
    cp_async_16(&st.kv[slot][0][lane], f.k_new + col);
    cp_async_16(&st.kv[slot][1][lane], f.v_new + col);
  }
  if (slot == 0 && lane == 0) cp_async_4(&st.ids[0], f.kv_indices + f.n_pages - 1);
  if (slot == 0 && lane == 1) cp_async_4(&st.ids[1], f.meta_indices + (f.n_pages - 1) / f.P);
  cp_async_commit();
}

// Appends head h with one warp (any warp of the CTA); st (may be NULL)
// holds its prefetched inputs in `slot`. A is any argument struct with the
// fields of FusedArgs that name the token, the page tables and the buffers.
template <int D, typename A>
__device__ __forceinline__ void append_head(const A& f, int h,
                                            const AppendStage* st = nullptr, int slot = 0) {
  const int H = f.H, P = f.P;
  constexpr int L = D / 8;
  const int lane = threadIdx.x & 31;
  const int page_iter = f.n_pages - 1;
  const int entry = f.last_len - 1;
  if (st) {
    asm volatile("cp.async.wait_all;" ::: "memory");
    __syncwarp();
  }
  const int pid = st ? st->ids[0] : __ldcg(f.kv_indices + page_iter);
  const int mpid = st ? st->ids[1] : __ldcg(f.meta_indices + page_iter / P);
  const int mentry = page_iter % P;
  const bool ok = pid >= 0 && pid < f.kv_cap && mpid >= 0 && mpid < f.meta_cap;
  if (!ok && lane == 0) raise_dev_error(f.err, AOAKV_DEV_ERR_BAD_PAGE);
  float s[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
  if (ok && lane < L) {
    const size_t HD = static_cast<size_t>(H) * D;
    const size_t col = static_cast<size_t>(h) * D + lane * 8;
    const uint4 kk = st ? st->kv[slot][0][lane] : *reinterpret_cast<const uint4*>(f.k_new + col);
    const uint4 vv = st ? st->kv[slot][1][lane] : *reinterpret_cast<const uint4*>(f.v_new + col);
    __half* mk = f.meta + ((static_cast<size_t>(mpid) * 2 + 0) * P + mentry) * HD + col;
    __half* mv = f.meta + ((static_cast<size_t>(mpid) * 2 + 1) * P + mentry) * HD + col;
    uint4 mx, mn;
    if (entry > 0) {
      mx = *reinterpret_cast<const uint4*>(mk);
      mn = *reinterpret_cast<const uint4*>(mv);
    } else {
      const __half2 lo = __float2half2_rn(-65504.f), hi = __float2half2_rn(65504.f);
      mx.x = mx.y = mx.z = mx.w = *reinterpret_cast<const uint32_t*>(&lo);
      mn.x = mn.y = mn.z = mn.w = *reinterpret_cast<const uint32_t*>(&hi);
    }
    __half2* a2 = reinterpret_cast<__half2*>(&mx);
    __half2* n2 = reinterpret_cast<__half2*>(&mn);
    const __half2* k2 = reinterpret_cast<const __half2*>(&kk);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      a2[i] = __hmax2(a2[i], k2[i]);
      n2[i] = __hmin2(n2[i], k2[i]);
    }
    __half* kvk = f.kv + ((static_cast<size_t>(pid) * 2 + 0) * P + entry) * HD + col;
    __half* kvv = f.kv + ((static_cast<size_t>(pid) * 2 + 1) * P + entry) * HD + col;
    *reinterpret_cast<uint4*>(kvk) = kk;
    *reinterpret_cast<uint4*>(kvv) = vv;
    *reinterpret_cast<uint4*>(mk) = mx;
    *reinterpret_cast<uint4*>(mv) = mn;
    if (entry + 1 == P) {  // earlier V rows of the page: 8 loads in flight
      for (int e0 = 0; e0 + 1 < P; e0 += 8) {
        uint4 r[8];
#pragma unroll
        for (int u = 0; u < 8; ++u)
          if (e0 + u + 1 < P)
            r[u] = ld_stream_u4(f.kv + ((static_cast<size_t>(pid) * 2 + 1) * P + e0 + u) * HD +
                                col);
#pragma unroll
        for (int u = 0; u < 8; ++u) {
          if (e0 + u + 1 < P) {
            float t[8];
            u4_to_f8(r[u], t);
#pragma unroll
            for (int i = 0; i < 8; ++i) s[i] += t[i];
          }
        }
      }
      float t[8];
      u4_to_f8(vv, t);
#pragma unroll
      for (int i = 0; i < 8; ++i) s[i] += t[i];
    }
  }
  if (entry + 1 == P) {
    const float inv = 1.f / P;
    float l2 = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) l2 += (s[i] * inv) * (s[i] * inv);
#pragma unroll
    for (int off = L / 2; off > 0; off >>= 1) l2 += __shfl_xor_sync(0xffffffffu, l2, off);
    if (ok && lane == 0)
      f.vlog[static_cast<size_t>(pid) * H + h] = __float2half_rn(logf(sqrtf(l2) + 1e-6f));
  }
  fence_proxy_async();  // the appended rows are read by TMA (async proxy) later
}

}  // namespace aoakv
