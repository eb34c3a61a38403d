// Top-k page selection by one histogram pass and exact candidate ranking.
//
// Same selection rule as the radix select (topk.cuh) and the bitonic top-K
// (topk_bitonic.cuh): the k largest scores, ties to the lower position, NaN
// below every number, -0 == +0, optional forced position 0; the output is in
// descending order of the 64-bit composite (score key, ~position), like the
// bitonic path.
//
// 1. Every score becomes its order-preserving 32-bit key (kept in shared
//    memory, with its page id when staged); one block reduction finds the
//    row's finite min and max.
// 2. Each key falls in one of 4096 bins (kept when staged) by a monotone
//    map: NaN and -inf in bin 0, finite scores linearly over bins 1..4093
//    between min and max, +inf in 4094, the forced position in 4095. A linear grid over the
//    row's own range keeps the bin around the k-th largest sparse for any
//    score scale or offset.
// 3. One block-wide scan over the bins finds the bin b* holding the k-th
//    largest key: fewer than k keys lie in bins above it.
// 4. Every key in bins >= b* is a candidate (k <= candidates, usually a
//    few more than k), gathered with its page id (loaded in step 1 when
//    the caller has room for n ids).
// 5. Each candidate's rank is the number of candidates with a larger
//    composite (composites are distinct); rank < k is selected and rank is
//    its output slot.
// Six block barriers; O(n / threads + c^2 / threads) work per thread.
// Because the bin map is monotone, the candidates always contain the true
// top k, so the result is exact. When more than kHistMaxCand keys share the
// top bins (many equal scores) the routine returns false without writing
// anything and the caller runs another exact path.
#pragma once

#include "topk_bitonic.cuh"

namespace aoakv {

constexpr int kHistBins = 4096;
constexpr int kHistMaxCand = 512;

struct HistSmem {
  uint32_t hist[kHistBins];
  uint64_t cand[kHistMaxCand];
  int cand_id[kHistMaxCand];
  float wmin[32], wmax[32];
  uint32_t warp_sum[32];
  int bstar, cnt;
};

// The monotone bin of a key (see the file comment); scale = 4092 / (max -
// min) over the row's finite scores, 0 when they are all equal.
__device__ __forceinline__ int hist_bin(uint32_t key, float mn, float scale) {
  if (key == 0xffffffffu) return kHistBins - 1;  // forced position
  if (key <= 0x007fffffu) return 0;              // NaN (key 0), -inf
  if (key >= 0xff800000u) return kHistBins - 2;  // +inf
  const float f = key_to_float(key);
  const int b = 1 + static_cast<int>((f - mn) * scale);
  return b < 1 ? 1 : (b > kHistBins - 3 ? kHistBins - 3 : b);
}

// Shared-memory staging of topk_row_hist for n scores: keys (u32), and
// when `staged`, the ids (int) and bins (u16) too; 16-byte multiple.
__host__ __device__ constexpr int hist_stage_bytes(int n, bool staged) {
  return staged ? (n + 7) / 8 * 80 : (n + 3) / 4 * 16;
}

// Step 3 of every path: the bin b* of the k-th largest key from the full
// histogram; thread t owns bins [t*bpt, (t+1)*bpt) (blockDim.x 512 or 1024).
// Sets hs.bstar / hs.cnt (keys in bins >= b*), ends with a block barrier.
__device__ __forceinline__ void hist_find_bin(HistSmem& hs, int k) {
  const int tid = threadIdx.x, nt = blockDim.x;
  const int lane = tid & 31, warp = tid >> 5, nw = nt >> 5;
  const int bpt = kHistBins / nt;  // 8 or 4 for nt = 512 or 1024
  uint32_t hb[8];
  uint32_t mine = 0;
#pragma unroll
  for (int j = 0; j < 8; j += 4) {
    if (j < bpt) {
      const uint4 h4 = *reinterpret_cast<const uint4*>(&hs.hist[tid * bpt + j]);
      hb[j] = h4.x;
      hb[j + 1] = h4.y;
      hb[j + 2] = h4.z;
      hb[j + 3] = h4.w;
      mine += h4.x + h4.y + h4.z + h4.w;
    }
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
#pragma unroll 4
  for (int w = 0; w < nw; ++w) {
    const uint32_t v = hs.warp_sum[w];
    before += w < warp ? v : 0u;
    total += v;
  }
  const uint32_t above = total - (before + incl);  // keys in bins above mine
  const uint32_t kk = static_cast<uint32_t>(k);
  if (above < kk && above + mine >= kk) {
    uint32_t c = above;
#pragma unroll
    for (int j = 7; j >= 0; --j) {
      if (j < bpt) {
        if (c + hb[j] >= kk) {
          hs.bstar = tid * bpt + j;
          hs.cnt = static_cast<int>(c + hb[j]);
          break;
        }
        c += hb[j];
      }
    }
  }
  __syncthreads();
}

// Step 5 of every path: rank the c gathered candidates (G threads per
// candidate) and write the k best to out_idx / out_vals / the window.
template <bool kL2>
__device__ __forceinline__ void hist_rank_emit(const TopkArgs& a, int row, HistSmem& hs, int c,
                                               int* win, int win_lo, int win_hi) {
  const int tid = threadIdx.x, nt = blockDim.x, k = a.k;
  const size_t sbase = static_cast<size_t>(row) * a.s_stride;
  int G = 32;
  while (G > 1 && G * c > nt) G >>= 1;
  const int per_pass = nt / G;
  const int sub = tid & (G - 1);
  for (int j0 = 0; j0 < c; j0 += per_pass) {
    const int j = j0 + tid / G;
    const bool valid = j < c;
    const uint64_t me = valid ? hs.cand[j] : 0ull;
    int r = 0;
    if (valid) {
#pragma unroll 4
      for (int m = sub; m < c; m += G) r += hs.cand[m] > me ? 1 : 0;
    }
    for (int o = 1; o < G; o <<= 1) r += __shfl_xor_sync(0xffffffffu, r, o);
    if (valid && sub == 0 && r < k) {
      const int id = hs.cand_id[j];
      if (a.out_idx) a.out_idx[static_cast<size_t>(row) * a.oi_stride + r] = id;
      if (win && r >= win_lo && r < win_hi) win[r - win_lo] = id;
      if (a.out_vals) {
        const uint32_t pos = ckey_pos(me);
        const uint32_t key = static_cast<uint32_t>(me >> 32);
        // the key is the score itself except at a forced position
        const float v = key == 0xffffffffu ? load_score<kL2>(a.scores, a.f32, sbase + pos)
                                           : key_to_float(key);
        const size_t o = static_cast<size_t>(row) * a.ov_stride + r;
        if (a.f32)
          static_cast<float*>(a.out_vals)[o] = v;
        else
          static_cast<__half*>(a.out_vals)[o] = __float2half_rn(v);
      }
    }
  }
  __syncthreads();
}

// Register path for n <= 4 * blockDim.x: thread t holds positions
// [4t, 4t + 4) (key, id, bin) in registers from load to gather, so no
// shared-memory staging is needed and the loads are 16-byte vectors.
template <bool kL2>
__device__ __forceinline__ bool topk_row_hist_regs(const TopkArgs& a, int row, HistSmem& hs,
                                                   int* win, int win_lo, int win_hi) {
  const int tid = threadIdx.x, nt = blockDim.x;
  const int lane = tid & 31, warp = tid >> 5, nw = nt >> 5;
  const int n = a.n;
  const size_t sbase = static_cast<size_t>(row) * a.s_stride;
  const size_t ibase = static_cast<size_t>(row) * a.in_stride;
  for (int i = tid * 4; i < kHistBins; i += nt * 4)
    *reinterpret_cast<uint4*>(&hs.hist[i]) = make_uint4(0u, 0u, 0u, 0u);
  if (tid == 0) {
    hs.bstar = 0;
    hs.cnt = n;
  }
  const int i0 = tid * 4;
  float s[4] = {0.f, 0.f, 0.f, 0.f};
  int id[4] = {i0, i0 + 1, i0 + 2, i0 + 3};
  const float* srow = static_cast<const float*>(a.scores) + sbase;
  if (a.f32 && i0 + 4 <= n && (reinterpret_cast<uintptr_t>(srow) & 15) == 0) {
    const float4 v4 = kL2 ? __ldcg(reinterpret_cast<const float4*>(srow + i0))
                          : *reinterpret_cast<const float4*>(srow + i0);
    s[0] = v4.x; s[1] = v4.y; s[2] = v4.z; s[3] = v4.w;
  } else {
#pragma unroll
    for (int u = 0; u < 4; ++u)
      if (i0 + u < n) s[u] = load_score<kL2>(a.scores, a.f32, sbase + i0 + u);
  }
  if (a.in_idx) {
    const int* irow = a.in_idx + ibase;
    if (i0 + 4 <= n && (reinterpret_cast<uintptr_t>(irow) & 15) == 0) {
      const int4 v4 = __ldg(reinterpret_cast<const int4*>(irow + i0));
      id[0] = v4.x; id[1] = v4.y; id[2] = v4.z; id[3] = v4.w;
    } else {
#pragma unroll
      for (int u = 0; u < 4; ++u)
        if (i0 + u < n) id[u] = __ldg(irow + i0 + u);
    }
  }
  uint32_t kr[4];
  float mn = INFINITY, mx = -INFINITY;
#pragma unroll
  for (int u = 0; u < 4; ++u) {
    const bool valid = i0 + u < n;
    const bool forced = a.sink && i0 + u == 0;
    kr[u] = forced ? 0xffffffffu : float_to_key(s[u]);
    if (valid && !forced && isfinite(s[u])) {
      mn = fminf(mn, s[u]);
      mx = fmaxf(mx, s[u]);
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    mn = fminf(mn, __shfl_xor_sync(0xffffffffu, mn, o));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  }
  if (lane == 0) {
    hs.wmin[warp] = mn;
    hs.wmax[warp] = mx;
  }
  __syncthreads();
#pragma unroll 4
  for (int w = 0; w < nw; ++w) {
    mn = fminf(mn, hs.wmin[w]);
    mx = fmaxf(mx, hs.wmax[w]);
  }
  const float range = mx - mn;
  const float scale =
      (range > 0.f && isfinite(range)) ? static_cast<float>(kHistBins - 4) / range : 0.f;
  int b[4];
#pragma unroll
  for (int u = 0; u < 4; ++u) {
    b[u] = i0 + u < n ? hist_bin(kr[u], mn, scale) : -1;
    if (b[u] >= 0) atomicAdd(&hs.hist[b[u]], 1u);
  }
  __syncthreads();
  hist_find_bin(hs, a.k);
  if (hs.cnt > kHistMaxCand) return false;  // uniform: every thread reads it
  const int bstar = hs.bstar;
  uint32_t m[4], wc = 0;
#pragma unroll
  for (int u = 0; u < 4; ++u) {
    m[u] = __ballot_sync(0xffffffffu, b[u] >= bstar);
    wc += __popc(m[u]);
  }
  if (lane == 0) hs.warp_sum[warp] = wc;
  __syncthreads();
  uint32_t off = 0, c_all = 0;
#pragma unroll 4
  for (int w = 0; w < nw; ++w) {
    const uint32_t v = hs.warp_sum[w];
    off += w < warp ? v : 0u;
    c_all += v;
  }
  const uint32_t lt = (1u << lane) - 1u;
#pragma unroll
  for (int u = 0; u < 4; ++u) {
    if (b[u] >= bstar) {
      const int slot = static_cast<int>(off) + __popc(m[u] & lt);
      hs.cand[slot] = make_ckey(kr[u], static_cast<uint32_t>(i0 + u));
      hs.cand_id[slot] = id[u];
    }
    off += __popc(m[u]);
  }
  __syncthreads();
  hist_rank_emit<kL2>(a, row, hs, static_cast<int>(c_all), win, win_lo, win_hi);
  return true;
}

// Exact top-k (1 <= k <= n) of row `row`; stage: hist_stage_bytes(n,
// staged) bytes of shared memory. With `staged`, the ids (loaded with the
// scores) and each key's bin are kept there; otherwise the bins are
// recomputed and the candidates' ids loaded while gathering; for n <= 4 *
// blockDim.x the register path runs and the stage is not used. Every thread
// of the block calls it (blockDim.x 512 or 1024). Returns false, having
// written nothing, if the candidates would exceed kHistMaxCand. Writes
// out_idx / out_vals / the window [win_lo, win_hi) of output slots like
// topk_row_bitonic.
template <bool kL2 = false>
__device__ __forceinline__ bool topk_row_hist(const TopkArgs& a, int row, uint8_t* stage,
                                              bool staged, HistSmem& hs, int* win = nullptr,
                                              int win_lo = 0, int win_hi = 0) {
  if (a.n <= 4 * static_cast<int>(blockDim.x))
    return topk_row_hist_regs<kL2>(a, row, hs, win, win_lo, win_hi);
  const int tid = threadIdx.x, nt = blockDim.x;
  const int lane = tid & 31, warp = tid >> 5, nw = nt >> 5;
  const int n = a.n, k = a.k;
  const int n8 = (n + 7) / 8 * 8;
  uint32_t* keys = reinterpret_cast<uint32_t*>(stage);
  int* ids = staged ? reinterpret_cast<int*>(stage + n8 * 4) : nullptr;
  uint16_t* bins = staged ? reinterpret_cast<uint16_t*>(stage + n8 * 8) : nullptr;
  const size_t sbase = static_cast<size_t>(row) * a.s_stride;
  for (int i = tid * 4; i < kHistBins; i += nt * 4)
    *reinterpret_cast<uint4*>(&hs.hist[i]) = make_uint4(0u, 0u, 0u, 0u);
  if (tid == 0) {
    hs.bstar = 0;  // k > n cannot happen; every key would be a candidate
    hs.cnt = n;
  }
  // 1. keys, ids and the finite min / max (4 score and 4 id loads in flight
  // per thread: the ids are at hand when the candidates are gathered)
  const size_t ibase = static_cast<size_t>(row) * a.in_stride;
  float mn = INFINITY, mx = -INFINITY;
  // fp32 rows on a 16-byte boundary load as float4, id rows as int4
  const bool vec_s = a.f32 && (reinterpret_cast<uintptr_t>(
                                   static_cast<const float*>(a.scores) + sbase) & 15) == 0;
  const bool vec_i = ids && a.in_idx &&
                     (reinterpret_cast<uintptr_t>(a.in_idx + ibase) & 15) == 0;
  for (int i0 = tid * 4; i0 < n; i0 += nt * 4) {
    float s[4];
    int id[4];
    if (vec_s && i0 + 4 <= n) {
      const float* sp = static_cast<const float*>(a.scores) + sbase + i0;
      const float4 v4 = kL2 ? __ldcg(reinterpret_cast<const float4*>(sp))
                            : *reinterpret_cast<const float4*>(sp);
      s[0] = v4.x; s[1] = v4.y; s[2] = v4.z; s[3] = v4.w;
    } else {
#pragma unroll
      for (int u = 0; u < 4; ++u)
        s[u] = i0 + u < n ? load_score<kL2>(a.scores, a.f32, sbase + i0 + u) : 0.f;
    }
    if (vec_i && i0 + 4 <= n) {
      const int4 v4 = __ldg(reinterpret_cast<const int4*>(a.in_idx + ibase + i0));
      id[0] = v4.x; id[1] = v4.y; id[2] = v4.z; id[3] = v4.w;
    } else {
#pragma unroll
      for (int u = 0; u < 4; ++u)
        id[u] = (ids && a.in_idx && i0 + u < n) ? __ldg(a.in_idx + ibase + i0 + u) : i0 + u;
    }
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      if (i0 + u < n) {
        const bool forced = a.sink && i0 + u == 0;
        if (ids) ids[i0 + u] = id[u];
        keys[i0 + u] = forced ? 0xffffffffu : float_to_key(s[u]);
        if (!forced && isfinite(s[u])) {
          mn = fminf(mn, s[u]);
          mx = fmaxf(mx, s[u]);
        }
      }
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    mn = fminf(mn, __shfl_xor_sync(0xffffffffu, mn, o));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  }
  if (lane == 0) {
    hs.wmin[warp] = mn;
    hs.wmax[warp] = mx;
  }
  __syncthreads();
#pragma unroll 4
  for (int w = 0; w < nw; ++w) {
    mn = fminf(mn, hs.wmin[w]);
    mx = fmaxf(mx, hs.wmax[w]);
  }
  const float range = mx - mn;
  const float scale =
      (range > 0.f && isfinite(range)) ? static_cast<float>(kHistBins - 4) / range : 0.f;
  // 2. histogram
  for (int i = tid; i < n; i += nt) {
    const int bin = hist_bin(keys[i], mn, scale);
    if (bins) bins[i] = static_cast<uint16_t>(bin);
    atomicAdd(&hs.hist[bin], 1u);
  }
  __syncthreads();
  // 3. the bin of the k-th largest
  hist_find_bin(hs, k);
  if (hs.cnt > kHistMaxCand) return false;  // uniform: every thread reads it
  // 4. gather the candidates with their ids: warp w owns positions
  // w*32 + it*nt + lane; slots come from a prefix over per-warp counts (no
  // shared-memory atomics, which serialise across warps on one address)
  const int bstar = hs.bstar;
  const int n_it = (n + nt - 1) / nt;
  uint32_t wcnt = 0;
  auto taken = [&](int i) {
    return i < n && (bins ? static_cast<int>(bins[i]) : hist_bin(keys[i], mn, scale)) >= bstar;
  };
  for (int it = 0; it < n_it; ++it)
    wcnt += __popc(__ballot_sync(0xffffffffu, taken(warp * 32 + it * nt + lane)));
  if (lane == 0) hs.warp_sum[warp] = wcnt;
  __syncthreads();
  uint32_t off = 0, c_all = 0;
#pragma unroll 4
  for (int w = 0; w < nw; ++w) {
    const uint32_t v = hs.warp_sum[w];
    off += w < warp ? v : 0u;
    c_all += v;
  }
  for (int it = 0; it < n_it; ++it) {
    const int i = warp * 32 + it * nt + lane;
    const bool take = taken(i);
    const uint32_t m = __ballot_sync(0xffffffffu, take);
    if (take) {
      const int slot = static_cast<int>(off) + __popc(m & ((1u << lane) - 1u));
      hs.cand[slot] = make_ckey(keys[i], static_cast<uint32_t>(i));
      hs.cand_id[slot] = ids ? ids[i] : (a.in_idx ? __ldg(a.in_idx + ibase + i) : i);
    }
    off += __popc(m);
  }
  __syncthreads();
  // 5. rank
  hist_rank_emit<kL2>(a, row, hs, static_cast<int>(c_all), win, win_lo, win_hi);
  return true;
}

}  // namespace aoakv
