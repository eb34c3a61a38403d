// Top-k page selection by one histogram pass and exact candidate ranking.
//
// Same selection rule as the radix select (topk.cuh) and the bitonic top-K
// (topk_bitonic.cuh): the k largest scores, ties to the lower position, NaN
// below every number, -0 == +0, optional forced position 0; the output is in
// descending order of the 64-bit composite (score key, ~position), like the
// bitonic path.
//
// 1. Every score becomes its order-preserving 32-bit key; one shared-memory
//    histogram counts the keys' top 12 bits (sign, exponent, 3 mantissa
//    bits: 4096 bins).
// 2. One block-wide scan over the bins finds the bin b* holding the k-th
//    largest key: fewer than k keys lie in bins above it.
// 3. Every key in bins >= b* is a candidate (k <= candidates; usually a few
//    more than k). Candidates are gathered as composites.
// 4. Each candidate's rank is the number of candidates with a larger
//    composite (composites are distinct); rank < k is selected and rank is
//    its output slot.
// When bin b* holds many keys (scores packed in a narrow range), a second
// 256-bin histogram over bits 19..12 of b*'s keys narrows the threshold to
// a sub-bin first, so the candidates stay close to k.
// Steps 1-4 cost four (six with the refinement) block barriers and
// O(n / threads + c^2 / threads) work per thread, against log-depth sorting
// networks or four radix passes.
// When more than kHistMaxCand keys share the top bins (many equal scores)
// the routine returns false without writing anything and the caller runs
// another exact path.
#pragma once

#include "topk_bitonic.cuh"

// Development timing hook (a phase stamp); compiled to nothing unless the
// including file defines it.
#ifndef AOAKV_TOPK_STAMP
#define AOAKV_TOPK_STAMP(i) \
  do {                      \
  } while (0)
#endif

namespace aoakv {

constexpr int kHistBins = 4096;
constexpr int kHistShift = 20;  // key >> 20: the top 12 bits
constexpr int kHistMaxCand = 512;

constexpr int kHistSubBins = 256;  // refinement: key bits 19..12 inside b*
constexpr int kHistRefineSlack = 64;  // refine when candidates > k + this

struct HistSmem {
  uint32_t hist[kHistBins];
  uint32_t hist2[kHistSubBins];
  uint64_t cand[kHistMaxCand];
  uint32_t warp_sum[32];
  uint32_t thr;  // candidates are the keys >= thr
  int bstar, c_gt, cnt, n_cand;
};

// Exact top-k (1 <= k <= n) of row `row`; keys: shared u32[>= n]. Every
// thread of the block calls it (blockDim.x a multiple of 32, <= 1024, and a
// divisor of kHistBins). Returns false, having written nothing, if the
// candidates would exceed kHistMaxCand. Writes out_idx / out_vals / the
// window [win_lo, win_hi) of output slots like topk_row_bitonic.
template <bool kL2 = false>
__device__ __forceinline__ bool topk_row_hist(const TopkArgs& a, int row, uint32_t* keys,
                                              HistSmem& hs, int* win = nullptr, int win_lo = 0,
                                              int win_hi = 0) {
  const int tid = threadIdx.x, nt = blockDim.x;
  const int lane = tid & 31, warp = tid >> 5, nw = nt >> 5;
  const int n = a.n, k = a.k;
  const size_t sbase = static_cast<size_t>(row) * a.s_stride;
  for (int i = tid * 4; i < kHistBins + kHistSubBins; i += nt * 4)
    *reinterpret_cast<uint4*>(&hs.hist[i]) = make_uint4(0u, 0u, 0u, 0u);  // hist, hist2
  if (tid == 0) {
    hs.bstar = 0;  // k > n cannot happen; every key would be a candidate
    hs.c_gt = 0;
    hs.cnt = n;
    hs.n_cand = 0;
  }
  __syncthreads();
  // 1. keys + histogram (4 score loads in flight per thread)
  for (int i0 = tid * 4; i0 < n; i0 += nt * 4) {
    float s[4];
#pragma unroll
    for (int u = 0; u < 4; ++u)
      s[u] = i0 + u < n ? load_score<kL2>(a.scores, a.f32, sbase + i0 + u) : 0.f;
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      if (i0 + u < n) {
        const uint32_t key = (a.sink && i0 + u == 0) ? 0xffffffffu : float_to_key(s[u]);
        keys[i0 + u] = key;
        atomicAdd(&hs.hist[key >> kHistShift], 1u);
      }
    }
  }
  __syncthreads();
  AOAKV_TOPK_STAMP(5);
  // 2. the bin of the k-th largest: thread t owns bins [t*bpt, (t+1)*bpt)
  const int bpt = kHistBins / nt;  // a multiple of 4 for nt <= 1024
  uint32_t mine = 0;
  for (int j = 0; j < bpt; j += 4) {
    const uint4 h4 = *reinterpret_cast<const uint4*>(&hs.hist[tid * bpt + j]);
    mine += h4.x + h4.y + h4.z + h4.w;
  }
  uint32_t incl = mine;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const uint32_t v = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += v;
  }
  if (lane == 31) hs.warp_sum[warp] = incl;
  __syncthreads();
  uint32_t before = 0, total = 0;
  for (int w = 0; w < nw; ++w) {
    const uint32_t v = hs.warp_sum[w];
    if (w < warp) before += v;
    total += v;
  }
  const uint32_t above = total - (before + incl);  // keys in bins above mine
  const uint32_t kk = static_cast<uint32_t>(k);
  if (above < kk && above + mine >= kk) {
    uint32_t c = above;
    for (int j = bpt - 1; j >= 0; --j) {
      const uint32_t h = hs.hist[tid * bpt + j];
      if (c + h >= kk) {
        hs.bstar = tid * bpt + j;
        hs.c_gt = static_cast<int>(c);
        hs.cnt = static_cast<int>(c + h);
        break;
      }
      c += h;
    }
  }
  __syncthreads();
  const uint32_t bstar = static_cast<uint32_t>(hs.bstar);
  uint32_t thr = bstar << kHistShift;
  if (hs.cnt > k + kHistRefineSlack) {
    // 2b. crowded bin b*: histogram its keys on bits 19..12 and find the
    // sub-bin holding the (k - c_gt)-th largest of them (warp 0 scans).
    for (int i = tid; i < n; i += nt) {
      const uint32_t key = keys[i];
      if ((key >> kHistShift) == bstar) atomicAdd(&hs.hist2[(key >> 12) & 0xffu], 1u);
    }
    __syncthreads();
    if (warp == 0) {
      constexpr int SB = kHistSubBins / 32;
      uint32_t h8[SB], m8 = 0;
#pragma unroll
      for (int j = 0; j < SB; ++j) {
        h8[j] = hs.hist2[lane * SB + j];
        m8 += h8[j];
      }
      uint32_t inc = m8;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const uint32_t v = __shfl_down_sync(0xffffffffu, inc, o);
        if (lane + o < 32) inc += v;
      }
      const uint32_t ab = inc - m8;  // keys of b* in sub-bins above this lane's
      const uint32_t kr = kk - static_cast<uint32_t>(hs.c_gt);
      if (ab < kr && ab + m8 >= kr) {
        uint32_t c = ab;
#pragma unroll
        for (int j = SB - 1; j >= 0; --j) {
          if (c + h8[j] >= kr) {
            hs.thr = thr | (static_cast<uint32_t>(lane * SB + j) << 12);
            hs.cnt = hs.c_gt + static_cast<int>(c + h8[j]);
            break;
          }
          c += h8[j];
        }
      }
    }
    __syncthreads();
    thr = hs.thr;
  }
  AOAKV_TOPK_STAMP(6);
  if (hs.cnt > kHistMaxCand) return false;  // uniform: every thread reads it
  // 3. gather the candidates (warp-aggregated slots)
  for (int base = warp * 32; base < n; base += nt) {
    const int i = base + lane;
    const uint32_t key = i < n ? keys[i] : 0u;
    const bool take = i < n && key >= thr;
    const uint32_t m = __ballot_sync(0xffffffffu, take);
    if (m) {
      int slot0 = 0;
      if (lane == 0) slot0 = atomicAdd(&hs.n_cand, __popc(m));
      slot0 = __shfl_sync(0xffffffffu, slot0, 0);
      if (take) hs.cand[slot0 + __popc(m & ((1u << lane) - 1u))] = make_ckey(key, i);
    }
  }
  __syncthreads();
  AOAKV_TOPK_STAMP(7);
  // 4. rank = candidates with a larger composite; G threads per candidate
  const int c = hs.n_cand;
  int G = 32;
  while (G > 1 && G * c > nt) G >>= 1;
  const int per_pass = nt / G;
  const int sub = tid & (G - 1);
  const size_t ibase = static_cast<size_t>(row) * a.in_stride;
  for (int j0 = 0; j0 < c; j0 += per_pass) {
    const int j = j0 + tid / G;
    const bool valid = j < c;
    const uint64_t me = valid ? hs.cand[j] : 0ull;
    int r = 0;
    if (valid)
      for (int m = sub; m < c; m += G) r += hs.cand[m] > me ? 1 : 0;
    for (int o = 1; o < G; o <<= 1) r += __shfl_xor_sync(0xffffffffu, r, o);
    if (valid && sub == 0 && r < k) {
      const uint32_t pos = ckey_pos(me);
      const int id = a.in_idx ? __ldg(a.in_idx + ibase + pos) : static_cast<int>(pos);
      if (a.out_idx) a.out_idx[static_cast<size_t>(row) * a.oi_stride + r] = id;
      if (win && r >= win_lo && r < win_hi) win[r - win_lo] = id;
      if (a.out_vals) {
        const size_t o = static_cast<size_t>(row) * a.ov_stride + r;
        if (a.f32)
          static_cast<float*>(a.out_vals)[o] = load_score<kL2>(a.scores, 1, sbase + pos);
        else
          static_cast<__half*>(a.out_vals)[o] =
              __float2half_rn(load_score<kL2>(a.scores, 0, sbase + pos));
      }
    }
  }
  __syncthreads();
  return true;
}

}  // namespace aoakv
