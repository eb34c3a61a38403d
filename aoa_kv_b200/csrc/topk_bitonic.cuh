// Top-K page selection for K <= 256 with warp-register bitonic networks.
//
// Same selection rule as the radix select (topk.cuh): the k largest scores,
// ties to the lower position, NaN below every number, optional forced
// position 0. It replaces the radix passes — whose histogram, scan and
// broadcast each cost a block-wide barrier — by work that stays inside
// warps: every element is a 64-bit composite (order-preserving score key in
// the high word, ~position in the low word, so larger is better and equal
// scores prefer the lower position; 0 is padding). Warp w sorts batches of K
// composites held as K/32 registers per lane (element i = register i/32 of
// lane i%32) with a bitonic network (shuffles for strides < 32, register
// swaps above), folds each batch into its running top-K with the bitonic
// top-K merge (max of one list and the other reversed, then a bitonic
// clean), and the warps' lists merge pairwise through shared memory in
// log2(warps) barrier steps. The result is in descending score order.
#pragma once

#include "topk.cuh"

namespace aoakv {

constexpr int kBitonicMaxK = 256;

__device__ __forceinline__ uint64_t make_ckey(uint32_t key, uint32_t pos) {
  return (static_cast<uint64_t>(key) << 32) | static_cast<uint32_t>(~pos);
}
__device__ __forceinline__ uint32_t ckey_pos(uint64_t c) { return ~static_cast<uint32_t>(c); }

__device__ __forceinline__ uint64_t shfl_xor64(uint64_t x, int m) {
  const uint32_t lo = __shfl_xor_sync(0xffffffffu, static_cast<uint32_t>(x), m);
  const uint32_t hi = __shfl_xor_sync(0xffffffffu, static_cast<uint32_t>(x >> 32), m);
  return (static_cast<uint64_t>(hi) << 32) | lo;
}
__device__ __forceinline__ uint64_t shfl_idx64(uint64_t x, int src) {
  const uint32_t lo = __shfl_sync(0xffffffffu, static_cast<uint32_t>(x), src);
  const uint32_t hi = __shfl_sync(0xffffffffu, static_cast<uint32_t>(x >> 32), src);
  return (static_cast<uint64_t>(hi) << 32) | lo;
}

// Sorts the warp's 32*E composites into descending order.
template <int E>
__device__ __forceinline__ void warp_bitonic_sort_desc(uint64_t (&v)[E]) {
  const int lane = threadIdx.x & 31;
  constexpr int K = 32 * E;
#pragma unroll
  for (int size = 2; size <= K; size <<= 1) {
#pragma unroll
    for (int j = size >> 1; j > 0; j >>= 1) {
      if (j >= 32) {
        const int jj = j >> 5;
#pragma unroll
        for (int e = 0; e < E; ++e) {
          if ((e & jj) == 0) {
            const bool desc = ((e * 32 + lane) & size) == 0;
            const uint64_t a = v[e], b = v[e | jj];
            const bool sw = desc ? (a < b) : (a > b);
            v[e] = sw ? b : a;
            v[e | jj] = sw ? a : b;
          }
        }
      } else {
        const bool lower = (lane & j) == 0;
#pragma unroll
        for (int e = 0; e < E; ++e) {
          const uint64_t p = shfl_xor64(v[e], j);
          const bool desc = ((e * 32 + lane) & size) == 0;
          v[e] = (lower == desc) ? (v[e] > p ? v[e] : p) : (v[e] < p ? v[e] : p);
        }
      }
    }
  }
}

// Sorts a bitonic sequence of 32*E composites into descending order.
template <int E>
__device__ __forceinline__ void warp_bitonic_merge_desc(uint64_t (&v)[E]) {
  const int lane = threadIdx.x & 31;
  constexpr int K = 32 * E;
#pragma unroll
  for (int j = K >> 1; j > 0; j >>= 1) {
    if (j >= 32) {
      const int jj = j >> 5;
#pragma unroll
      for (int e = 0; e < E; ++e) {
        if ((e & jj) == 0) {
          const uint64_t a = v[e], b = v[e | jj];
          v[e] = a > b ? a : b;
          v[e | jj] = a > b ? b : a;
        }
      }
    } else {
      const bool lower = (lane & j) == 0;
#pragma unroll
      for (int e = 0; e < E; ++e) {
        const uint64_t p = shfl_xor64(v[e], j);
        v[e] = lower ? (v[e] > p ? v[e] : p) : (v[e] < p ? v[e] : p);
      }
    }
  }
}

// v <- top-K of (v ∪ w), both sorted descending; w_rev holds w reversed
// (element i of w_rev = element K-1-i of w).
template <int E>
__device__ __forceinline__ void warp_topk_fold_rev(uint64_t (&v)[E], const uint64_t (&w_rev)[E]) {
#pragma unroll
  for (int e = 0; e < E; ++e) v[e] = v[e] > w_rev[e] ? v[e] : w_rev[e];
  warp_bitonic_merge_desc(v);
}

template <int E>
__device__ __forceinline__ void warp_topk_fold(uint64_t (&v)[E], const uint64_t (&w)[E]) {
  const int lane = threadIdx.x & 31;
  uint64_t r[E];
#pragma unroll
  for (int e = 0; e < E; ++e) r[e] = shfl_idx64(w[E - 1 - e], 31 - lane);
  warp_topk_fold_rev(v, r);
}

__host__ __device__ constexpr size_t bitonic_xbuf_bytes(int nwarps, int K) {
  return static_cast<size_t>(nwarps / 2 > 0 ? nwarps / 2 : 1) * K * 8;
}

// Block-wide top-K (K = 32*E, k <= K <= 256) of row `row` of a.scores.
// keys: shared u32[>= n]; xbuf: shared, bitonic_xbuf_bytes(warps, K). Every
// thread must call it; blockDim.x is a power-of-two multiple of 32. Writes
// the k best in descending order to out_idx / out_vals / the window like
// topk_row.
template <int E, bool kL2 = false>
__device__ __forceinline__ void topk_row_bitonic(const TopkArgs& a, int row, uint32_t* keys,
                                                 uint64_t* xbuf, int* win = nullptr,
                                                 int win_lo = 0, int win_hi = 0) {
  constexpr int K = 32 * E;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int NW = blockDim.x >> 5;
  const size_t sbase = static_cast<size_t>(row) * a.s_stride;
  // 1. scores -> order-preserving keys in shared memory, 4 loads in flight
  for (int i0 = threadIdx.x * 4; i0 < a.n; i0 += blockDim.x * 4) {
    float s[4];
#pragma unroll
    for (int u = 0; u < 4; ++u)
      s[u] = i0 + u < a.n ? load_score<kL2>(a.scores, a.f32, sbase + i0 + u) : 0.f;
#pragma unroll
    for (int u = 0; u < 4; ++u)
      if (i0 + u < a.n)
        keys[i0 + u] = (a.sink && i0 + u == 0) ? 0xffffffffu : float_to_key(s[u]);
  }
  __syncthreads();
  // 2. per-warp running top-K over the warp's span, in batches of K
  const int per = (a.n + NW - 1) / NW;
  const int span = (per + K - 1) / K * K;
  const int p0 = warp * span, p1 = min(a.n, p0 + span);
  uint64_t v[E];
#pragma unroll
  for (int e = 0; e < E; ++e) v[e] = 0;
  for (int base = p0; base < p1; base += K) {
    uint64_t w[E];
#pragma unroll
    for (int e = 0; e < E; ++e) {
      const int pos = base + e * 32 + lane;
      w[e] = pos < p1 ? make_ckey(keys[pos], static_cast<uint32_t>(pos)) : 0ull;
    }
    warp_bitonic_sort_desc(w);
    if (base == p0) {
#pragma unroll
      for (int e = 0; e < E; ++e) v[e] = w[e];
    } else {
      warp_topk_fold(v, w);
    }
  }
  // 3. pairwise merge of the warps' lists through shared memory
  for (int step = 1; step < NW; step <<= 1) {
    const int slot = warp / (2 * step);
    if ((warp & (2 * step - 1)) == step) {
#pragma unroll
      for (int e = 0; e < E; ++e) xbuf[static_cast<size_t>(slot) * K + e * 32 + lane] = v[e];
    }
    __syncthreads();
    if ((warp & (2 * step - 1)) == 0 && warp + step < NW) {
      uint64_t r[E];
#pragma unroll
      for (int e = 0; e < E; ++e)
        r[e] = xbuf[static_cast<size_t>(slot) * K + (K - 1 - (e * 32 + lane))];
      warp_topk_fold_rev(v, r);
    }
    __syncthreads();
  }
  // 4. warp 0 holds the K best, descending: emit the first k
  if (warp == 0) {
    const size_t ibase = static_cast<size_t>(row) * a.in_stride;
#pragma unroll
    for (int e = 0; e < E; ++e) {
      const int i = e * 32 + lane;
      if (i < a.k) {
        const uint32_t pos = ckey_pos(v[e]);
        const int id = a.in_idx ? __ldg(a.in_idx + ibase + pos) : static_cast<int>(pos);
        if (a.out_idx) a.out_idx[static_cast<size_t>(row) * a.oi_stride + i] = id;
        if (win && i >= win_lo && i < win_hi) win[i - win_lo] = id;
        if (a.out_vals) {
          const size_t o = static_cast<size_t>(row) * a.ov_stride + i;
          if (a.f32)
            static_cast<float*>(a.out_vals)[o] = load_score<kL2>(a.scores, 1, sbase + pos);
          else
            static_cast<__half*>(a.out_vals)[o] =
                __float2half_rn(load_score<kL2>(a.scores, 0, sbase + pos));
        }
      }
    }
  }
  __syncthreads();
}

// Dispatches on K = the smallest power of two >= max(k, 32); requires
// k <= 32 * kMaxE (kMaxE in {1, 2, 4, 8}; smaller instantiates fewer
// register-heavy variants).
template <bool kL2 = false, int kMaxE = 8>
__device__ __forceinline__ void topk_row_small(const TopkArgs& a, int row, uint32_t* keys,
                                               uint64_t* xbuf, int* win = nullptr,
                                               int win_lo = 0, int win_hi = 0) {
  if (a.k <= 32 || kMaxE == 1)
    topk_row_bitonic<1, kL2>(a, row, keys, xbuf, win, win_lo, win_hi);
  else if (a.k <= 64 || kMaxE == 2)
    topk_row_bitonic<(kMaxE < 2 ? kMaxE : 2), kL2>(a, row, keys, xbuf, win, win_lo, win_hi);
  else if (a.k <= 128 || kMaxE == 4)
    topk_row_bitonic<(kMaxE < 4 ? kMaxE : 4), kL2>(a, row, keys, xbuf, win, win_lo, win_hi);
  else
    topk_row_bitonic<kMaxE, kL2>(a, row, keys, xbuf, win, win_lo, win_hi);
}

}  // namespace aoakv
