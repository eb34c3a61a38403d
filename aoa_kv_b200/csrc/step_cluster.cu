// The per-layer decode step as ONE launch of thread-block clusters: one
// cluster of C CTAs per head runs append, page scoring, exact top-k page
// selection, sparse decode and the log-sum-exp merge, exchanging scores'
// histograms, candidates, selected page ids and partial softmax states
// through distributed shared memory. No grid-wide barrier, no global-memory
// flags, no workspace.
//
// Reference (kernels/aoa_kv/): the decode branch of
// quest/models/QuestAttention.py:99-157 issues append_kv
// (kernels/include/decode/decode_page.cuh:392-506), decode_estimate
// (decode_attn.cuh:263-443 with compute_max_possible :143-199), decode_topk
// (topk/decode_select_k.cuh:25-61, RAFT radix select) and
// decode_sparse_attn (decode_attn.cuh:469-688, split-KV merge :937-1047)
// as four launches with host work between them.
//
// Per cluster (head h), CTA c of C:
//   1  scoring: CTA c owns a contiguous run of metadata pages (P scored KV
//      pages each). Warp w owns ring slot w and handles the CTA's metadata
//      pages w, w + 16, ...: one TMA box {D, 1, P} of the page's key maxima
//      and one of its minima per step, and a fp32 dot product per KV page,
//      sum_i q_i * (q_i > 0 ? kmax_i : kmin_i), which equals
//      sum_i max(q_i*kmax_i, q_i*kmin_i) because kmax >= kmin; AOA-KV adds
//      2*v_log_norm of the page after scaling by 2/sqrt(D). Scores stay in
//      shared memory. Warp 15 of the last CTA appends the head's new token
//      (and on page fill its v_log_norm) while its first box is in flight.
//   2  selection: the exact top-(k-1) (with the sink: page 0 plus the
//      top-(k-2) of pages 1..N-2), ties toward the lower page, NaN lowest.
//      Each level exchanges the candidates' finite score range, then a
//      2048-bin histogram (NaN, -inf, 2045 linear bins, +inf: monotone in
//      the score, so bins order the scores exactly) and finds the bin that
//      holds the threshold. Pages above it are in; if the threshold bin
//      must be split, its candidates are ranked exactly by (score, page)
//      when few (<= 512), by page when they are all equal, else the next
//      level bins the threshold bin alone.
//   3  decode: the k attended slots (selected pages in page order, then the
//      last page) are split evenly over the C CTAs; a warp gathers a slot's
//      K and V tiles with two TMA boxes {D, 1, P} into its ring slot and
//      updates an online softmax in the log2 domain; warps merge in shared
//      memory, CTAs through distributed shared memory (CTA c finalises
//      channels [c*D/C, (c+1)*D/C)).
// Under programmatic dependent launch nothing in global memory is read
// before griddepcontrol.wait, so the previous kernel on the stream (even
// this layer's previous step) may write any of it. Device waits on TMA
// completions are bounded (AOAKV_DEV_ERR_TIMEOUT); cluster barriers are
// reached by every CTA on every path.
#include <cooperative_groups.h>

#include <atomic>
#include <cmath>
#include <map>
#include <mutex>
#include <tuple>

#include "common.cuh"
#include "decode.cuh"
#include "step_append.cuh"
#include "step_cluster.h"

namespace cg = cooperative_groups;

namespace aoakv {
namespace {

constexpr int kCsThreads = 512;
constexpr int kCsWarps = kCsThreads / 32;
constexpr int kCsBins = 2048;             // 0 NaN, 1 -inf, 2..2046 linear, 2047 +inf
constexpr int kCsLinBins = kCsBins - 3;
constexpr int kCsBinsPerThread = kCsBins / kCsThreads;
constexpr int kCsMaxCand = 512;           // exact ranking of the threshold bin
constexpr int kCsMaxLevels = 6;
constexpr int kCsMaxPage = 16;
static_assert(kCsBinsPerThread == 4, "one uint4 of bins per thread");

struct CsLayout {
  int ring, scores, state, hist, cand, candall, sel, mrg, xo, total;
};

__host__ __device__ inline int cs_up(int x) { return (x + 127) / 128 * 128; }
__host__ __device__ inline int cs_slot_bytes(int D, int P) { return cs_up(2 * P * D * 2); }

__host__ __device__ inline CsLayout cs_layout(int D, int P, int max_local) {
  CsLayout L;
  int off = 0;
  L.ring = off;
  off += kCsWarps * cs_slot_bytes(D, P);
  L.scores = off;
  off += cs_up(max_local * 4);
  L.state = off;
  off += cs_up(max_local);
  L.hist = off;
  off += kCsBins * 4;
  L.cand = off;
  off += kCsMaxCand * 8;
  L.candall = off;
  off += kCsMaxCand * 8;
  L.sel = off;
  off += cs_up(max_local * 4);
  L.mrg = off;
  off += cs_up(kCsWarps * (D + 2) * 4);
  L.xo = off;
  off += cs_up(D * 4);
  L.total = off;
  return L;
}

// What peer CTAs read from this CTA's shared memory besides the arrays.
struct CsXchg {
  float fmin, fmax;  // finite score range of this CTA's candidates
  int n_sel;         // selected pages in the `sel` array
  float M, L;        // decode partial: running max (log2 units), denominator
};

// Exclusive prefix sum over the CTA in thread order; *total = the sum.
__device__ __forceinline__ int cs_block_scan(int v, int* total) {
  __shared__ int ws[kCsWarps];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  int x = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, x, o);
    if (lane >= o) x += y;
  }
  if (lane == 31) ws[warp] = x;
  __syncthreads();
  if (warp == 0) {
    int y = lane < kCsWarps ? ws[lane] : 0;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int z = __shfl_up_sync(0xffffffffu, y, o);
      if (lane >= o) y += z;
    }
    if (lane < kCsWarps) ws[lane] = y;
  }
  __syncthreads();
  const int base = warp ? ws[warp - 1] : 0;
  *total = ws[kCsWarps - 1];
  __syncthreads();
  return base + x - v;
}

// CTA-wide min of lo and max of hi, written to *out_lo / *out_hi.
__device__ __forceinline__ void cs_block_minmax(float lo, float hi, float* out_lo,
                                                float* out_hi) {
  __shared__ float wl[kCsWarps], wh[kCsWarps];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    lo = fminf(lo, __shfl_xor_sync(0xffffffffu, lo, o));
    hi = fmaxf(hi, __shfl_xor_sync(0xffffffffu, hi, o));
  }
  if (lane == 0) {
    wl[warp] = lo;
    wh[warp] = hi;
  }
  __syncthreads();
  if (warp == 0) {
    lo = lane < kCsWarps ? wl[lane] : INFINITY;
    hi = lane < kCsWarps ? wh[lane] : -INFINITY;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      lo = fminf(lo, __shfl_xor_sync(0xffffffffu, lo, o));
      hi = fmaxf(hi, __shfl_xor_sync(0xffffffffu, hi, o));
    }
    if (lane == 0) {
      *out_lo = lo;
      *out_hi = hi;
    }
  }
  __syncthreads();
}

// Histogram bin of a candidate score, monotone non-decreasing in x:
// NaN < -inf < finite (linear over [gmin, gmin + range]) < +inf. A zero
// range (equal or unbounded candidates) puts every finite score in bin 2.
__device__ __forceinline__ int cs_bin(float x, float gmin, float range) {
  if (isnan(x)) return 0;
  if (x == -INFINITY) return 1;
  if (x == INFINITY) return kCsBins - 1;
  if (!(range > 0.f)) return 2;
  const float t = __fdiv_rn(x - gmin, range) * static_cast<float>(kCsLinBins);
  const int b = t < static_cast<float>(kCsLinBins) ? __float2int_rz(t) : kCsLinBins - 1;
  return 2 + (b < 0 ? 0 : b);
}

// Sums part[j] (j < 16) over the 32 lanes of the warp: afterwards every
// lane holds the total of page j = (lane >> 1) & 15 (16 shuffles).
__device__ __forceinline__ float cs_reduce16(const float part[16]) {
  const int lane = threadIdx.x & 31;
  const bool b4 = lane & 16, b3 = lane & 8, b2 = lane & 4, b1 = lane & 2;
  float r8[8], r4[4], r2[2], r1;
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const float send = b4 ? part[i] : part[8 + i];
    const float keep = b4 ? part[8 + i] : part[i];
    r8[i] = keep + __shfl_xor_sync(0xffffffffu, send, 16);
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float send = b3 ? r8[i] : r8[4 + i];
    const float keep = b3 ? r8[4 + i] : r8[i];
    r4[i] = keep + __shfl_xor_sync(0xffffffffu, send, 8);
  }
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    const float send = b2 ? r4[i] : r4[2 + i];
    const float keep = b2 ? r4[2 + i] : r4[i];
    r2[i] = keep + __shfl_xor_sync(0xffffffffu, send, 4);
  }
  {
    const float send = b1 ? r2[0] : r2[1];
    const float keep = b1 ? r2[1] : r2[0];
    r1 = keep + __shfl_xor_sync(0xffffffffu, send, 2);
  }
  return r1 + __shfl_xor_sync(0xffffffffu, r1, 1);
}

template <int D, int C>
__global__ void __launch_bounds__(kCsThreads, 1)
    cluster_step_kernel(const __grid_constant__ CUtensorMap kv_map,
                        const __grid_constant__ CUtensorMap meta_map, ClusterStepArgs a,
                        int max_local) {
  constexpr int CPL = D / 32;  // channels per lane
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 127) & ~static_cast<uintptr_t>(127));
  __shared__ uint64_t bars[kCsWarps];
  __shared__ CsXchg xs;
  __shared__ int bc[3];  // threshold bin, count above it, count in it
  __shared__ int peer_cnt[C], peer_off[C + 1];
  __shared__ float gsh[2];
  __shared__ int cnt_s;

  cg::cluster_group cluster = cg::this_cluster();
  const int c = static_cast<int>(cluster.block_rank());
  const int h = blockIdx.y;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int P = a.P, H = a.H;
  const CsLayout lay = cs_layout(D, P, max_local);
  uint8_t* slot = smem + lay.ring + warp * cs_slot_bytes(D, P);
  float* sc = reinterpret_cast<float*>(smem + lay.scores);
  uint8_t* st = smem + lay.state;
  uint32_t* hist = reinterpret_cast<uint32_t*>(smem + lay.hist);
  uint2* cand = reinterpret_cast<uint2*>(smem + lay.cand);
  uint2* candall = reinterpret_cast<uint2*>(smem + lay.candall);
  int* sel = reinterpret_cast<int*>(smem + lay.sel);
  float* mrg = reinterpret_cast<float*>(smem + lay.mrg);
  float* xo = reinterpret_cast<float*>(smem + lay.xo);
  uint64_t* bar = &bars[warp];
  const uint32_t tile_bytes = static_cast<uint32_t>(P * D * 2);

  if (tid == 0) {
    for (int i = 0; i < kCsWarps; ++i) mbar_init(&bars[i], 1);
    fence_mbar_init();
    tma_prefetch_desc(&kv_map);
    tma_prefetch_desc(&meta_map);
  }
  __syncthreads();
  // Everything in global memory may be written by the previous kernel on
  // the stream (under programmatic dependent launch it can still be
  // running), so every global read comes after this wait.
  pdl_wait();
  pdl_launch_dependents();

  const int N = a.n_pages, n = N - 1;
  const int k = a.k_slots;
  const bool sparse = N > k && k > 1;
  const bool aoa = a.mode == AOAKV_SCORE_AOAKV;
  const int n_st = sparse ? (n + P - 1) / P : 0;  // metadata pages holding scored pages
  const int st_lo = (c * n_st) / C, st_hi = ((c + 1) * n_st) / C;
  const int pos_lo = st_lo * P;
  const int nloc = sparse ? max(0, min(n, st_hi * P) - pos_lo) : 0;
  const int r_lo = a.sink ? 1 : 0;
  const bool appender = c == C - 1 && warp == kCsWarps - 1;

  float qv[CPL];
  load_row<CPL>(a.q + static_cast<size_t>(h) * D + lane * CPL, qv);
  uint32_t msk[CPL / 2];
#pragma unroll
  for (int i = 0; i < CPL / 2; ++i)
    msk[i] = (qv[2 * i] > 0.f ? 0x0000ffffu : 0u) | (qv[2 * i + 1] > 0.f ? 0xffff0000u : 0u);
  uint32_t par = 0;  // phase of this warp's ring-slot barrier

  // ------------------------------------------------------------ 1 scoring
  float fmin_l = INFINITY, fmax_l = -INFINITY;
  if (sparse) {
    const int jp = (lane >> 1) & 15;           // page of the stage this lane scores
    const bool writer = (lane & 1) == 0 && jp < P;
    auto issue = [&](int t) -> bool {
      int ok = 0;
      if (lane == 0) {
        const int mp = __ldcg(a.meta_indices + t);
        if (mp >= 0 && mp < a.meta_cap) {
          ok = 1;
          fence_proxy_async_smem();
          mbar_arrive_expect_tx(bar, 2u * tile_bytes);
          tma_load_3d(slot, &meta_map, 0, h, mp * 2 * P, bar);
          tma_load_3d(slot + tile_bytes, &meta_map, 0, h, mp * 2 * P + P, bar);
        } else {
          raise_dev_error(a.err, AOAKV_DEV_ERR_BAD_PAGE);
        }
      }
      return __shfl_sync(0xffffffffu, ok, 0) != 0;
    };
    // v_log_norm of the lane's page of stage t (AOA-KV), NaN for a bad id
    auto vlog_of = [&](int t) -> float {
      const int pos = t * P + jp;
      if (!aoa || !writer || pos >= n) return 0.f;
      const int pid = __ldcg(a.kv_indices + pos);
      if (pid < 0 || pid >= a.kv_cap) {
        raise_dev_error(a.err, AOAKV_DEV_ERR_BAD_PAGE);
        return NAN;
      }
      return __half2float(__ldcg(a.vlog + static_cast<size_t>(pid) * H + h));
    };
    int t = st_lo + warp;
    bool ok = false;
    float vl = 0.f;
    if (t < st_hi) {
      ok = issue(t);
      vl = vlog_of(t);
    }
    if (appender) append_head<D>(a, h);  // while the first boxes are in flight
    for (; t < st_hi; t += kCsWarps) {
      bool got = ok;
      if (ok) {
        got = mbar_wait_bounded(bar, par, a.err);
        par ^= 1u;
      }
      float part[16];
      const __half* mx = reinterpret_cast<const __half*>(slot);
      const __half* mn = mx + P * D;
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        part[j] = 0.f;
        if (j < P && got) {
          uint32_t hx[CPL / 2], hn[CPL / 2];
          if constexpr (CPL == 4) {
            const uint2 ux = *reinterpret_cast<const uint2*>(mx + j * D + lane * CPL);
            const uint2 un = *reinterpret_cast<const uint2*>(mn + j * D + lane * CPL);
            hx[0] = ux.x; hx[1] = ux.y; hn[0] = un.x; hn[1] = un.y;
          } else {
            hx[0] = *reinterpret_cast<const uint32_t*>(mx + j * D + lane * CPL);
            hn[0] = *reinterpret_cast<const uint32_t*>(mn + j * D + lane * CPL);
          }
#pragma unroll
          for (int i = 0; i < CPL / 2; ++i) {
            const uint32_t s2 = (hx[i] & msk[i]) | (hn[i] & ~msk[i]);
            const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&s2));
            part[j] = fmaf(qv[2 * i], f.x, part[j]);
            part[j] = fmaf(qv[2 * i + 1], f.y, part[j]);
          }
        }
      }
      const float s = cs_reduce16(part);
      const float vl_t = vl;
      const int pos = t * P + jp;
      __syncwarp();  // every lane is done with the slot before it is refilled
      const int tn = t + kCsWarps;
      if (tn < st_hi) {
        ok = issue(tn);
        vl = vlog_of(tn);
      }
      if (writer && pos < n) {
        const float score = !got ? NAN : (aoa ? a.two_rsqrt_d * s + 2.f * vl_t : s);
        const int i = pos - pos_lo;
        sc[i] = score;
        const uint8_t s0 = pos >= r_lo ? 1 : 2;  // the sink page is forced
        st[i] = s0;
        if (s0 == 1 && isfinite(score)) {
          fmin_l = fminf(fmin_l, score);
          fmax_l = fmaxf(fmax_l, score);
        }
      }
    }
  } else if (appender) {
    append_head<D>(a, h);
  }
  __syncthreads();

  // ---------------------------------------------------------- 2 selection
  if (sparse) {
    int need = (k - 1) - r_lo;  // pages to choose among the ranked ones
    bool done = need <= 0;
    for (int level = 0; !done; ++level) {
      // A: finite range of the candidates (state 1), cluster-wide
      float lo = fmin_l, hi = fmax_l;
      if (level > 0) {
        lo = INFINITY;
        hi = -INFINITY;
        for (int i = tid; i < nloc; i += kCsThreads) {
          if (st[i] != 1) continue;
          const float x = sc[i];
          if (isfinite(x)) {
            lo = fminf(lo, x);
            hi = fmaxf(hi, x);
          }
        }
      }
      cs_block_minmax(lo, hi, &xs.fmin, &xs.fmax);
      cluster.sync();  // ranges published; peers are done with this CTA's histogram
      if (warp == 0) {
        float gl = INFINITY, gh = -INFINITY;
        if (lane < C) {
          const CsXchg* px = cluster.map_shared_rank(&xs, lane);
          gl = px->fmin;
          gh = px->fmax;
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
          gl = fminf(gl, __shfl_xor_sync(0xffffffffu, gl, o));
          gh = fmaxf(gh, __shfl_xor_sync(0xffffffffu, gh, o));
        }
        if (lane == 0) {
          gsh[0] = gl;
          gsh[1] = gh;
        }
      }
      for (int b = tid; b < kCsBins; b += kCsThreads) hist[b] = 0u;
      __syncthreads();
      const float gmin = gsh[0], gmax = gsh[1];
      const float range = (gmax > gmin && gmax - gmin < INFINITY) ? gmax - gmin : 0.f;
      // B: histogram of the candidates, cluster-wide
      for (int i = tid; i < nloc; i += kCsThreads)
        if (st[i] == 1) atomicAdd(&hist[cs_bin(sc[i], gmin, range)], 1u);
      __syncthreads();
      cluster.sync();  // histograms published
      // C: the bin holding the need-th largest candidate
      uint4 pv[C];
      uint32_t tot[4] = {0u, 0u, 0u, 0u};
#pragma unroll
      for (int cc = 0; cc < C; ++cc) {
        pv[cc] = reinterpret_cast<const uint4*>(cluster.map_shared_rank(hist, cc))[tid];
        tot[0] += pv[cc].x;
        tot[1] += pv[cc].y;
        tot[2] += pv[cc].z;
        tot[3] += pv[cc].w;
      }
      const int mine = static_cast<int>(tot[0] + tot[1] + tot[2] + tot[3]);
      int all_cnt;
      const int excl = cs_block_scan(mine, &all_cnt);
      int run = all_cnt - excl - mine;  // candidates in higher bins (higher threads)
#pragma unroll
      for (int j = 3; j >= 0; --j) {
        const int tj = static_cast<int>(tot[j]);
        if (run < need && need <= run + tj) {
          bc[0] = tid * 4 + j;
          bc[1] = run;
          bc[2] = tj;
        }
        run += tj;
      }
      __syncthreads();
      const int bstar = bc[0], above = bc[1], cnt = bc[2];
      if (tid == (bstar >> 2)) {  // each CTA's share of the threshold bin
#pragma unroll
        for (int cc = 0; cc < C; ++cc) {
          const uint32_t v4[4] = {pv[cc].x, pv[cc].y, pv[cc].z, pv[cc].w};
          peer_cnt[cc] = static_cast<int>(v4[bstar & 3]);
        }
      }
      __syncthreads();
      const int need2 = need - above;  // 1 <= need2 <= cnt
      const bool take_all = need2 == cnt;
      const bool by_page = !take_all && (bstar < 2 || bstar == kCsBins - 1 ||
                                         !(range > 0.f) || level == kCsMaxLevels - 1);
      const bool exact = !take_all && !by_page && cnt <= kCsMaxCand;
      for (int i = tid; i < nloc; i += kCsThreads) {
        if (st[i] != 1) continue;
        const int b = cs_bin(sc[i], gmin, range);
        st[i] = b > bstar ? 2 : (b < bstar ? 0 : (take_all ? 2 : 1));
      }
      __syncthreads();
      if (take_all) break;
      if (by_page) {
        // equal scores: the lower pages win; pages of lower CTAs are lower
        int base = 0;
        for (int cc = 0; cc < c; ++cc) base += peer_cnt[cc];
        const int ch = (nloc + kCsThreads - 1) / kCsThreads;
        const int i0 = min(nloc, tid * ch), i1 = min(nloc, i0 + ch);
        int m = 0;
        for (int i = i0; i < i1; ++i) m += st[i] == 1;
        int tot_m;
        int r = base + cs_block_scan(m, &tot_m);
        for (int i = i0; i < i1; ++i)
          if (st[i] == 1) st[i] = (r++ < need2) ? 2 : 0;
        __syncthreads();
        break;
      }
      if (exact) {
        // few candidates: rank each by (score, page) against all of them
        if (tid == 0) cnt_s = 0;
        __syncthreads();
        for (int i = tid; i < nloc; i += kCsThreads)
          if (st[i] == 1)
            cand[atomicAdd(&cnt_s, 1)] =
                make_uint2(float_to_key(sc[i]), static_cast<uint32_t>(pos_lo + i));
        __syncthreads();
        cluster.sync();  // candidate lists published
        for (int g = tid; g < cnt; g += kCsThreads) {
          int cc = 0, off = 0;
          while (cc < C - 1 && g >= off + peer_cnt[cc]) off += peer_cnt[cc++];
          candall[g] = cluster.map_shared_rank(cand, cc)[g - off];
        }
        __syncthreads();
        for (int i = tid; i < cnt_s; i += kCsThreads) {
          const uint2 me = cand[i];
          int r = 0;
          for (int g = 0; g < cnt; ++g) {
            const uint2 o = candall[g];
            r += (o.x > me.x) || (o.x == me.x && o.y < me.y);
          }
          st[me.y - pos_lo] = r < need2 ? 2 : 0;
        }
        __syncthreads();
        break;
      }
      need = need2;  // refine inside the threshold bin
    }
    // this CTA's selected pages in page order, as physical ids
    {
      const int ch = (nloc + kCsThreads - 1) / kCsThreads;
      const int i0 = min(nloc, tid * ch), i1 = min(nloc, i0 + ch);
      int m = 0;
      for (int i = i0; i < i1; ++i) m += st[i] == 2;
      int tot_sel;
      int w = cs_block_scan(m, &tot_sel);
      for (int i = i0; i < i1; ++i) {
        if (st[i] != 2) continue;
        int pid = __ldcg(a.kv_indices + pos_lo + i);
        if (pid < 0 || pid >= a.kv_cap) {
          raise_dev_error(a.err, AOAKV_DEV_ERR_BAD_PAGE);
          pid = -1;
        }
        sel[w++] = pid;
      }
      if (tid == 0) xs.n_sel = tot_sel;
    }
    __syncthreads();
    cluster.sync();  // selections published
    if (warp == 0) {
      int v = lane < C ? cluster.map_shared_rank(&xs, lane)->n_sel : 0;
      int x = v;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, x, o);
        if (lane >= o) x += y;
      }
      if (lane < C) peer_off[lane] = x - v;
      if (lane == C - 1) peer_off[C] = x;
    }
    __syncthreads();
  }

  // ------------------------------------------------------------- 3 decode
  // slots: the selected pages (in page order), then the last page
  const int T = sparse ? k : (N <= k ? N : 1);
  const int last_pid = __ldcg(a.kv_indices + N - 1);
  if (a.selected_out) {
    int32_t* row = a.selected_out + static_cast<size_t>(h) * a.sel_cols;
    if (sparse) {
      for (int i = tid; i < xs.n_sel; i += kCsThreads)
        if (peer_off[c] + i < T - 1) row[peer_off[c] + i] = sel[i];
    } else if (c == 0) {
      for (int i = tid; i < T - 1; i += kCsThreads) row[i] = __ldcg(a.kv_indices + i);
    }
    if (c == C - 1)
      for (int i = T - 1 + tid; i < a.sel_cols; i += kCsThreads) row[i] = i == T - 1 ? last_pid : -1;
  }
  const int s_lo = (c * T) / C, s_hi = ((c + 1) * T) / C;
  float qs[CPL];
#pragma unroll
  for (int i = 0; i < CPL; ++i) qs[i] = qv[i] * a.scale_log2;
  float m = -INFINITY, l = 0.f, o[CPL];
#pragma unroll
  for (int i = 0; i < CPL; ++i) o[i] = 0.f;
  for (int s = s_lo + warp; s < s_hi; s += kCsWarps) {
    int ntok = 0;
    if (lane == 0) {
      int pid = -1;
      if (s == T - 1) {
        pid = last_pid;
        ntok = a.last_len;
      } else if (sparse) {
        int cc = 0;
        while (cc < C - 1 && s >= peer_off[cc + 1]) ++cc;
        if (s < peer_off[C]) pid = cluster.map_shared_rank(sel, cc)[s - peer_off[cc]];
        ntok = P;
      } else {
        pid = __ldcg(a.kv_indices + s);
        ntok = P;
      }
      if (pid < 0 || pid >= a.kv_cap) {
        raise_dev_error(a.err, AOAKV_DEV_ERR_BAD_PAGE);
        ntok = 0;
      }
      if (ntok > 0) {
        fence_proxy_async_smem();
        mbar_arrive_expect_tx(bar, 2u * tile_bytes);
        tma_load_3d(slot, &kv_map, 0, h, pid * 2 * P, bar);
        tma_load_3d(slot + tile_bytes, &kv_map, 0, h, pid * 2 * P + P, bar);
      }
    }
    ntok = __shfl_sync(0xffffffffu, ntok, 0);
    if (ntok > 0) {
      const bool got = mbar_wait_bounded(bar, par, a.err);
      par ^= 1u;
      if (got) {
        const __half* Kt = reinterpret_cast<const __half*>(slot);
        for (int t0 = 0; t0 < ntok; t0 += 8) attend8<D>(Kt, Kt + P * D, t0, ntok, P, qs, m, l, o);
      }
    }
    __syncwarp();
  }
  // merge the warps of this CTA
  {
    float* mw = mrg + warp * (D + 2);
#pragma unroll
    for (int i = 0; i < CPL; ++i) mw[lane * CPL + i] = o[i];
    if (lane == 0) {
      mw[D] = m;
      mw[D + 1] = l;
    }
  }
  __syncthreads();
  if (tid < D) {
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < kCsWarps; ++w) M = fmaxf(M, mrg[w * (D + 2) + D]);
    float Ls = 0.f, O = 0.f;
    if (M != -INFINITY) {
#pragma unroll
      for (int w = 0; w < kCsWarps; ++w) {
        const float f = fast_exp2(mrg[w * (D + 2) + D] - M);
        Ls += f * mrg[w * (D + 2) + D + 1];
        O += f * mrg[w * (D + 2) + tid];
      }
    }
    xo[tid] = O;
    if (tid == 0) {
      xs.M = M;
      xs.L = Ls;
    }
  }
  __syncthreads();
  cluster.sync();  // partial states published
  constexpr int DPC = D / C;
  if (tid < DPC) {
    const int d = c * DPC + tid;
    float MM = -INFINITY;
#pragma unroll
    for (int cc = 0; cc < C; ++cc) MM = fmaxf(MM, cluster.map_shared_rank(&xs, cc)->M);
    float LL = 0.f, OO = 0.f;
    if (MM != -INFINITY) {
#pragma unroll
      for (int cc = 0; cc < C; ++cc) {
        const CsXchg* px = cluster.map_shared_rank(&xs, cc);
        const float f = fast_exp2(px->M - MM);
        LL += f * px->L;
        OO += f * cluster.map_shared_rank(xo, cc)[d];
      }
    }
    a.o[static_cast<size_t>(h) * D + d] = __float2half_rn(LL > 0.f ? OO / LL : 0.f);
  }
  cluster.sync();  // no CTA leaves while a peer still reads its shared memory
}

using KernelFn = void (*)(CUtensorMap, CUtensorMap, ClusterStepArgs, int);

template <int D>
const void* kernel_for(int C) {
  switch (C) {
    case 1: return reinterpret_cast<const void*>(cluster_step_kernel<D, 1>);
    case 2: return reinterpret_cast<const void*>(cluster_step_kernel<D, 2>);
    case 4: return reinterpret_cast<const void*>(cluster_step_kernel<D, 4>);
    default: return reinterpret_cast<const void*>(cluster_step_kernel<D, 8>);
  }
}

const void* kernel_ptr(int D, int C) { return D == 128 ? kernel_for<128>(C) : kernel_for<64>(C); }

// Per (device, D, C): the dynamic shared memory the kernel attribute allows
// and the clusters that fit at once at that size.
struct FnState {
  size_t smem_set = 0;
  int max_clusters = 0;
};
std::mutex g_fn_mu;
std::map<std::tuple<int, int, int>, FnState> g_fn_state;

// -1 unknown, 0 the driver rejected programmatic serialization with
// clusters, 1 accepted (learnt on the first launch outside stream capture)
std::atomic<int> g_cluster_pdl{-1};

}  // namespace

int cluster_step_plan(int H, int D, int P, int max_pages, ClusterPlan* plan) {
  if ((D != 64 && D != 128) || P < 1 || P > kCsMaxPage || H < 1 || H > 65535 || max_pages < 1)
    return 0;
  const int sms = num_sms();
  int C = 8;
  while (C > 1 && H * C > sms) C >>= 1;
  int n_st = (max_pages - 1 + P - 1) / P;
  if (n_st < 1) n_st = 1;
  int max_local = (n_st + C - 1) / C * P;
  size_t smem = static_cast<size_t>(cs_layout(D, P, max_local).total) + 128;
  while (smem > 200 * 1024 && C < 8) {  // long sequences: more CTAs per head
    C <<= 1;
    max_local = (n_st + C - 1) / C * P;
    smem = static_cast<size_t>(cs_layout(D, P, max_local).total) + 128;
  }
  if (smem > 200 * 1024) return 0;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 0;
  const void* fn = kernel_ptr(D, C);
  std::lock_guard<std::mutex> lk(g_fn_mu);
  FnState& fs = g_fn_state[std::make_tuple(dev, D, C)];
  if (fs.smem_set < smem) {
    if (cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(smem)) != cudaSuccess) {
      (void)cudaGetLastError();
      return 0;
    }
    fs.smem_set = smem;
    fs.max_clusters = 0;
  }
  if (fs.max_clusters == 0) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(C, H);
    cfg.blockDim = dim3(kCsThreads);
    cfg.dynamicSmemBytes = fs.smem_set;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = C;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    int ncl = 0;
    if (cudaOccupancyMaxActiveClusters(&ncl, fn, &cfg) != cudaSuccess || ncl < 1) {
      (void)cudaGetLastError();
      return 0;
    }
    fs.max_clusters = ncl;
  }
  plan->cluster = C;
  plan->max_local = max_local;
  plan->smem = fs.smem_set;
  plan->waves = (H + fs.max_clusters - 1) / fs.max_clusters;
  return 1;
}

int launch_cluster_step(const ClusterStepArgs& a, const CUtensorMap& kv_map,
                        const CUtensorMap& meta_map, int D, const ClusterPlan& plan,
                        cudaStream_t s) {
  const int C = plan.cluster;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(C, a.H);
  cfg.blockDim = dim3(kCsThreads);
  cfg.dynamicSmemBytes = plan.smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = C;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  const KernelFn fn = reinterpret_cast<KernelFn>(const_cast<void*>(kernel_ptr(D, C)));
  int pdl = g_cluster_pdl.load();
  if (pdl == -1) {
    cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
    if (cudaStreamIsCapturing(s, &cs) != cudaSuccess || cs != cudaStreamCaptureStatusNone)
      pdl = 0;  // learn outside capture only: a failed launch would end the capture
  }
  if (pdl != 0) {
    cfg.numAttrs = 2;
    const cudaError_t e = cudaLaunchKernelEx(&cfg, fn, kv_map, meta_map, a, plan.max_local);
    if (e == cudaSuccess) {
      g_cluster_pdl.store(1);
      return AOAKV_OK;
    }
    if (pdl == 1) AOAKV_CUDA_TRY(e, "cluster step launch");
    (void)cudaGetLastError();
    g_cluster_pdl.store(0);
  }
  cfg.numAttrs = 1;
  AOAKV_CUDA_TRY(cudaLaunchKernelEx(&cfg, fn, kv_map, meta_map, a, plan.max_local),
                 "cluster step launch");
  return AOAKV_OK;
}

}  // namespace aoakv
