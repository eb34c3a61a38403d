// a4 top-k page selector: one CTA per row, keys resident in shared memory.
//
// Reference: kernels/aoa_kv/kernels/include/topk/decode_select_k.cuh:25-61
// launches RAFT radix_topk_one_block_kernel<T, int, 8 bits/pass, 512>
// (rapidsai/raft branch-24.02, not vendored) with one block per head; its
// output order is unspecified and it needs a caller scratch buffer.
// Published algorithm restated here: most-significant-digit radix select
// over order-preserving 32-bit keys, 8 bits per pass, which finds the exact
// k-th largest key T and how many keys equal to T are taken. Selection is
// then exact: every key > T, plus the lowest-position keys == T. Output is in
// ascending position order via one block-wide prefix sum; no scratch in
// global memory.
#pragma once

#include "common.cuh"

namespace aoakv {

constexpr int kTopkThreads = 1024;
constexpr int kTopkMaxN = 49152;  // 192 KB of keys

struct TopkArgs {
  const void* scores;
  int64_t s_stride;
  const int32_t* in_idx;
  int64_t in_stride;
  void* out_vals;
  int64_t ov_stride;
  int32_t* out_idx;
  int64_t oi_stride;
  int f32;
  int n, k;
  int sink;
};

struct TopkSmem {
  uint32_t hist[256];
  uint32_t warp_tot[32];
  uint32_t sel_digit;
  uint32_t sel_rank;
};

// kL2: read through L2 only (scores written by other CTAs of the same launch).
template <bool kL2 = false>
__device__ __forceinline__ float load_score(const void* s, int f32, size_t i) {
  if constexpr (kL2)
    return f32 ? __ldcg(static_cast<const float*>(s) + i)
               : __half2float(__ldcg(static_cast<const __half*>(s) + i));
  return f32 ? static_cast<const float*>(s)[i]
             : __half2float(static_cast<const __half*>(s)[i]);
}

// Block-wide MSD radix select of the k-th largest of keys[0..n). Returns the
// threshold key T (via *thr) and the number of keys == T to take (via *need).
__device__ __forceinline__ void radix_select(const uint32_t* keys, int n, int k,
                                             TopkSmem& sm, uint32_t* thr,
                                             int* need) {
  uint32_t prefix = 0, mask = 0, kr = static_cast<uint32_t>(k);
  for (int shift = 24; shift >= 0; shift -= 8) {
    for (int i = threadIdx.x; i < 256; i += blockDim.x) sm.hist[i] = 0;
    __syncthreads();
    // Warp-aggregated histogram: scores of similar magnitude share their top
    // key bits, so equal digits are grouped per warp (one atomic per group).
    for (int base = 0; base < n; base += blockDim.x) {
      const int i = base + threadIdx.x;
      uint32_t d = 256u;  // sentinel: not counted
      if (i < n) {
        const uint32_t key = keys[i];
        if ((key & mask) == prefix) d = (key >> shift) & 255u;
      }
      const uint32_t peers = __match_any_sync(0xffffffffu, d);
      if (d < 256u && (threadIdx.x & 31) == __ffs(peers) - 1)
        atomicAdd(&sm.hist[d], static_cast<uint32_t>(__popc(peers)));
    }
    __syncthreads();
    if (threadIdx.x < 32) {
      const int lane = threadIdx.x;
      uint32_t c[8], tot = 0;
#pragma unroll
      for (int j = 0; j < 8; ++j) {  // digits in descending order
        c[j] = sm.hist[255 - (8 * lane + j)];
        tot += c[j];
      }
      uint32_t incl = tot;
#pragma unroll
      for (int off = 1; off < 32; off <<= 1) {
        const uint32_t y = __shfl_up_sync(0xffffffffu, incl, off);
        if (lane >= off) incl += y;
      }
      const uint32_t excl = incl - tot;
      if (excl < kr && kr <= incl) {
        uint32_t run = excl;
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          if (run + c[j] >= kr) {
            sm.sel_digit = 255u - (8u * lane + j);
            sm.sel_rank = kr - run;
            break;
          }
          run += c[j];
        }
      }
    }
    __syncthreads();
    prefix |= sm.sel_digit << shift;
    mask |= 255u << shift;
    kr = sm.sel_rank;
    __syncthreads();
  }
  *thr = prefix;
  *need = static_cast<int>(kr);
}

// Exclusive block prefix sum of a packed (gt << 16 | eq) counter pair.
__device__ __forceinline__ uint32_t block_excl_scan(uint32_t v, TopkSmem& sm) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  uint32_t incl = v;
#pragma unroll
  for (int off = 1; off < 32; off <<= 1) {
    const uint32_t y = __shfl_up_sync(0xffffffffu, incl, off);
    if (lane >= off) incl += y;
  }
  if (lane == 31) sm.warp_tot[warp] = incl;
  __syncthreads();
  if (warp == 0) {
    const int nw = blockDim.x >> 5;
    uint32_t t = lane < nw ? sm.warp_tot[lane] : 0u;
    uint32_t ti = t;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
      const uint32_t y = __shfl_up_sync(0xffffffffu, ti, off);
      if (lane >= off) ti += y;
    }
    if (lane < nw) sm.warp_tot[lane] = ti - t;  // exclusive warp offsets
  }
  __syncthreads();
  const uint32_t r = sm.warp_tot[warp] + incl - v;
  __syncthreads();
  return r;
}

// Selects row `row`'s top-k into out arrays. keys: shared buffer of >= n.
// Must be called by every thread of the block. Optionally also copies the
// selected ids whose output position lies in [win_lo, win_hi) to
// win[pos - win_lo] (a shared-memory window).
template <bool kL2 = false>
__device__ __forceinline__ void topk_row(const TopkArgs& a, int row,
                                         uint32_t* keys, TopkSmem& sm,
                                         int* win = nullptr, int win_lo = 0,
                                         int win_hi = 0) {
  const size_t sbase = static_cast<size_t>(row) * a.s_stride;
  for (int i = threadIdx.x; i < a.n; i += blockDim.x) {
    uint32_t key = float_to_key(load_score<kL2>(a.scores, a.f32, sbase + i));
    if (a.sink && i == 0) key = 0xffffffffu;  // above every float key
    keys[i] = key;
  }
  __syncthreads();
  uint32_t T;
  int need;
  radix_select(keys, a.n, a.k, sm, &T, &need);
  // Contiguous segment per thread keeps output in position order.
  const int seg = (a.n + blockDim.x - 1) / blockDim.x;
  const int b = min(a.n, static_cast<int>(threadIdx.x) * seg);
  const int e = min(a.n, b + seg);
  uint32_t gt = 0, eq = 0;
  for (int i = b; i < e; ++i) {
    const uint32_t key = keys[i];
    gt += key > T;
    eq += key == T;
  }
  const uint32_t pre = block_excl_scan((gt << 16) | eq, sm);
  uint32_t gt_before = pre >> 16, eq_before = pre & 0xffffu;
  const uint32_t need_u = static_cast<uint32_t>(need);
  const size_t ibase = static_cast<size_t>(row) * a.in_stride;
  for (int i = b; i < e; ++i) {
    const uint32_t key = keys[i];
    bool take = false;
    uint32_t pos = 0;
    if (key > T) {
      take = true;
      pos = gt_before + min(eq_before, need_u);
      ++gt_before;
    } else if (key == T) {
      if (eq_before < need_u) {
        take = true;
        pos = gt_before + eq_before;
      }
      ++eq_before;
    }
    if (take) {
      const int id = a.in_idx ? __ldg(a.in_idx + ibase + i) : i;
      if (a.out_idx) a.out_idx[static_cast<size_t>(row) * a.oi_stride + pos] = id;
      if (win && static_cast<int>(pos) >= win_lo && static_cast<int>(pos) < win_hi)
        win[pos - win_lo] = id;
      if (a.out_vals) {
        const size_t o = static_cast<size_t>(row) * a.ov_stride + pos;
        if (a.f32)
          static_cast<float*>(a.out_vals)[o] = static_cast<const float*>(a.scores)[sbase + i];
        else
          static_cast<__half*>(a.out_vals)[o] = static_cast<const __half*>(a.scores)[sbase + i];
      }
    }
  }
  __syncthreads();
}

// topk_row for scores produced earlier in the same launch by other CTAs.
__device__ __forceinline__ void topk_row_cg(const TopkArgs& a, int row, uint32_t* keys,
                                            TopkSmem& sm, int* win = nullptr, int win_lo = 0,
                                            int win_hi = 0) {
  topk_row<true>(a, row, keys, sm, win, win_lo, win_hi);
}

}  // namespace aoakv
