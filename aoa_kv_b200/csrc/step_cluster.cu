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
#include "step_cluster.h"

namespace cg = cooperative_groups;

namespace aoakv {
namespace {

constexpr int kCsThreads = 512;
constexpr int kCsWarps = kCsThreads / 32;
constexpr int kCsBins = 2048;             // 0 NaN, 1 -inf, 2..2046 linear, 2047 +inf
constexpr int kCsLinBins = kCsBins - 3;
constexpr int kCsBinsPerThread = kCsBins / kCsThreads;
constexpr int kCsMaxCand = 512;           // fallback: exact ranking of the threshold bin
constexpr int kCsGather = 2048;           // candidates gathered from the whole cluster
constexpr int kCsMaxLevels = 6;
constexpr int kCsMaxPage = 16;
static_assert(kCsBinsPerThread == 4, "one uint4 of bins per thread");

struct CsLayout {
  int ring, scores, state, pidl, hist, cand, lst, gkey, gpos, items, mrg, xo, total;
};

__host__ __device__ inline int cs_up(int x) { return (x + 127) / 128 * 128; }
// One ring slot: a metadata page's max and min tiles (scoring) or a KV page's
// K and V as D/64 swizzled 16-row tiles of 128-byte rows (decode), 1024-byte
// aligned (the 128-byte swizzle repeats every 8 rows).
constexpr int kCsSubTile = 16 * 128;
__host__ __device__ inline int cs_slot_bytes(int D, int P) {
  const int score = 2 * P * D * 2, dec = 2 * (D / 64) * kCsSubTile;
  const int b = score > dec ? score : dec;
  return (b + 1023) / 1024 * 1024;
}
// Local candidates one CTA may publish: its share of the gathered lists,
// but no more than twice the attended slots (at least kCsMaxCand), so a
// small cluster does not spend shared memory on lists it cannot fill.
__host__ __device__ inline int cs_capl(int C, int max_slots) {
  const int want = 2 * max_slots > kCsMaxCand ? 2 * max_slots : kCsMaxCand;
  return kCsGather / C < want ? kCsGather / C : want;
}
__host__ __device__ inline int cs_max_items(int C, int max_slots) {
  const int a = cs_capl(C, max_slots) + 2, b = (max_slots + C - 1) / C;
  return a > b ? a : b;
}

__host__ __device__ inline CsLayout cs_layout(int D, int P, int C, int max_local,
                                              int max_slots) {
  CsLayout L;
  const int capl = cs_capl(C, max_slots);
  const int capx = capl > kCsMaxCand ? capl : kCsMaxCand;
  int off = 0;
  L.ring = off;  // one TMA slot per warp: metadata pages, then K/V pages
  off += kCsWarps * cs_slot_bytes(D, P);
  L.scores = off;
  off += cs_up(max_local * 4);
  L.state = off;
  off += cs_up(max_local);
  L.pidl = off;  // page ids of the scored pages; the fallback's selection list
  off += cs_up(max_local * 4);
  L.hist = off;
  off += kCsBins * 4;
  L.cand = off;  // local candidates {key, page, id}; the fallback's threshold bin
  off += capx * 16;
  L.lst = off;  // the same sorted by (score desc, page asc): read by peers
  off += cs_up(capl * 16);
  L.gkey = off;  // keys and pages of every CTA's sorted list, CTA after CTA
  off += kCsGather * 4;
  L.gpos = off;
  off += kCsGather * 4;
  L.items = off;  // page ids this CTA attends
  off += cs_up(cs_max_items(C, max_slots) * 4);
  L.mrg = off;
  off += cs_up(kCsWarps * (D + 2) * 4);
  L.xo = off;  // CTA 0: every CTA's partial state (D numerators, max, sum)
  off += cs_up(C * (D + 2) * 4);
  L.total = off;
  return L;
}

// What peer CTAs read from this CTA's shared memory besides the arrays.
struct CsXchg {
  int m, ovf;        // local candidates published in `lst`; more than fit
  float fmin, fmax;  // fallback: finite score range of this CTA's candidates
  int n_sel;         // fallback: selected pages in the `sel` array
};

// ---------------------------------------------------------- cluster PTX
__device__ __forceinline__ void cluster_arrive_release() {
  asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
}
// Arrival that orders nothing: for barriers that only mark "done reading
// peers' shared memory" (the values read are already consumed).
__device__ __forceinline__ void cluster_arrive_relaxed() {
  asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory");
}
__device__ __forceinline__ void cluster_wait_acquire() {
  asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// Arrives (release, cluster scope) on the mbarrier at the same shared
// memory offset as `bar` in CTA `rank` of the cluster.
__device__ __forceinline__ void mbar_arrive_remote(uint64_t* bar, uint32_t rank) {
  uint32_t remote;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(remote) : "r"(smem_addr(bar)), "r"(rank));
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(remote)
               : "memory");
}
__device__ __forceinline__ bool mbar_try_wait_cluster(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_addr(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
// L2 prefetch of one TMA box (no completion, no effect on correctness).
__device__ __forceinline__ void tma_prefetch_l2_3d(const CUtensorMap* map, int c0, int c1,
                                                   int c2) {
  asm volatile("cp.async.bulk.prefetch.tensor.3d.L2.global.tile [%0, {%1, %2, %3}];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(c0), "r"(c1), "r"(c2)
               : "memory");
}

// (key, page) of `a` ranks above that of `b`: higher score, then lower page.
__device__ __forceinline__ bool cs_beats(uint32_t ka, uint32_t pa, uint32_t kb, uint32_t pb) {
  return ka > kb || (ka == kb && pa < pb);
}

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

// The same order-preserving binning with a precomputed scale (kCsLinBins /
// range, 0 when the range is zero, infinite or overflows): monotone but not
// identical to cs_bin, so it is used only where a superset suffices.
__device__ __forceinline__ int cs_bin_mul(float x, float gmin, float scale) {
  if (isnan(x)) return 0;
  if (x == -INFINITY) return 1;
  if (x == INFINITY) return kCsBins - 1;
  const float t = (x - gmin) * scale;
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

// ------------------------------------------------ tensor-core page attention
__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2,
                                        uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr)
               : "memory");
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2,
                                          uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr)
               : "memory");
}
// d += a (16x16 fp16, row) * b (16x8 fp16, col), fp32 accumulate
__device__ __forceinline__ void mma16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                         uint32_t a3, uint32_t b0, uint32_t b1) {
  asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
// Byte offset of 16-byte unit `unit` of row `row` in a 1024-byte-aligned tile
// of 128-byte rows written by TMA with the 128-byte swizzle.
__device__ __forceinline__ uint32_t sw128(int row, int unit) {
  return static_cast<uint32_t>(row * 128 + ((unit ^ (row & 7)) << 4));
}
// Shared-memory byte offset of the lane's CPL channels in row `row` of a
// page's K (or V) tiles (D/64 tiles of kCsSubTile bytes).
template <int D>
__device__ __forceinline__ uint32_t sw_lane_off(int row) {
  constexpr int CPL = D / 32;
  const int ch = (threadIdx.x & 31) * CPL;
  return static_cast<uint32_t>((ch >> 6) * kCsSubTile) + sw128(row, (ch & 63) >> 3) +
         static_cast<uint32_t>((ch & 7) * 2);
}

// One warp attends one page (ntok valid rows) on the tensor cores:
// S^T = K q^T (M = 16 tokens, K = D channels; q is column 0 of B) and
// O^T += V^T P^T (M = 16 channels per tile, K = 16 tokens; P is column 0 of
// B, rounded to fp16 — the softmax sum adds the same rounded values).
// Online softmax in the log2 domain. Only column 0 of every C fragment is
// meaningful: lane 4g holds tokens g, g+8 (S) and channels 16mm+g, 16mm+g+8
// (acc[mm][0], acc[mm][2]). Rows >= ntok of V must hold finite values (the
// caller zeroes them).
template <int D>
__device__ __forceinline__ void cs_attend_page_tc(uint32_t kb, uint32_t vb, int ntok,
                                                  const uint32_t (&qb)[D / 16][2],
                                                  float scale_log2, float& m, float& l,
                                                  float (&acc)[D / 16][4]) {
  constexpr int NK = D / 16;
  const int lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3, mi = lane >> 3, r8 = lane & 7;
  float s4[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
  for (int kk = 0; kk < NK; ++kk) {
    uint32_t a0, a1, a2, a3;
    ldsm_x4(kb + (kk >> 2) * kCsSubTile + sw128((mi & 1) * 8 + r8, (kk & 3) * 2 + (mi >> 1)), a0,
            a1, a2, a3);
    mma16816(s4, a0, a1, a2, a3, qb[kk][0], qb[kk][1]);
  }
  const bool v0 = t == 0 && g < ntok, v1 = t == 0 && g + 8 < ntok;
  const float x0 = v0 ? s4[0] * scale_log2 : -INFINITY;
  const float x1 = v1 ? s4[2] * scale_log2 : -INFINITY;
  float mx = fmaxf(x0, x1);
#pragma unroll
  for (int off = 4; off < 32; off <<= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
  mx = __shfl_sync(0xffffffffu, mx, 0);
  const float m_new = fmaxf(m, mx);  // finite: token 0 is valid
  const float alpha = fast_exp2(m - m_new);
  const float p0 = v0 ? __half2float(__float2half_rn(fast_exp2(x0 - m_new))) : 0.f;
  const float p1 = v1 ? __half2float(__float2half_rn(fast_exp2(x1 - m_new))) : 0.f;
  float ps = p0 + p1;
#pragma unroll
  for (int off = 4; off < 32; off <<= 1) ps += __shfl_xor_sync(0xffffffffu, ps, off);
  ps = __shfl_sync(0xffffffffu, ps, 0);
  l = l * alpha + ps;
  // P^T as B: lane t (group 0) holds tokens 2t, 2t+1 and 2t+8, 2t+9
  const float pa = __shfl_sync(0xffffffffu, p0, 8 * t), pb = __shfl_sync(0xffffffffu, p0, 8 * t + 4);
  const float pc = __shfl_sync(0xffffffffu, p1, 8 * t), pd = __shfl_sync(0xffffffffu, p1, 8 * t + 4);
  uint32_t b0 = 0u, b1 = 0u;
  if (g == 0) {
    const __half2 h01 = __floats2half2_rn(pa, pb), h89 = __floats2half2_rn(pc, pd);
    b0 = *reinterpret_cast<const uint32_t*>(&h01);
    b1 = *reinterpret_cast<const uint32_t*>(&h89);
  }
#pragma unroll
  for (int mm = 0; mm < NK; ++mm) {
#pragma unroll
    for (int i = 0; i < 4; ++i) acc[mm][i] *= alpha;
    uint32_t a0, a1, a2, a3;
    ldsm_x4_t(vb + (mm >> 2) * kCsSubTile + sw128((mi >> 1) * 8 + r8, (mm & 3) * 2 + (mi & 1)), a0,
              a1, a2, a3);
    mma16816(acc[mm], a0, a1, a2, a3, b0, b1);
  }
  m = m_new;
}

// One warp: the bin b of hist (kCsBins counts) with above(b) < need <=
// above(b) + hist[b]; bc = {b, above(b), hist[b]}. Two levels of suffix sums
// over the lanes (64 bins per lane, then 2), no block barrier.
__device__ __forceinline__ void cs_threshold_warp(const uint32_t* hist, int need, int* bc) {
  const int lane = threadIdx.x & 31;
  const uint4* h4 = reinterpret_cast<const uint4*>(hist);
  int sl = 0;
#pragma unroll
  for (int j = 0; j < 16; ++j) {
    const uint4 v = h4[lane * 16 + ((j + lane) & 15)];  // rotated: no bank conflicts
    sl += static_cast<int>(v.x + v.y + v.z + v.w);
  }
  int inc = sl;  // sum over this lane and the higher ones
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_down_sync(0xffffffffu, inc, o);
    if (lane + o < 32) inc += y;
  }
  const int above1 = inc - sl;
  const unsigned f1 = __ballot_sync(0xffffffffu, above1 < need && need <= above1 + sl);
  const int L1 = __ffs(f1) - 1;
  const int a1 = __shfl_sync(0xffffffffu, above1, L1);
  const uint2 v2 = reinterpret_cast<const uint2*>(hist)[L1 * 32 + lane];
  const int s2 = static_cast<int>(v2.x + v2.y);
  int inc2 = s2;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_down_sync(0xffffffffu, inc2, o);
    if (lane + o < 32) inc2 += y;
  }
  const int above2 = a1 + inc2 - s2;
  const int hi = static_cast<int>(v2.y), lo = static_cast<int>(v2.x);
  int b = -1, ab = 0, cnt = 0;
  if (above2 < need && need <= above2 + hi) {
    b = L1 * 64 + 2 * lane + 1;
    ab = above2;
    cnt = hi;
  } else if (above2 + hi < need && need <= above2 + hi + lo) {
    b = L1 * 64 + 2 * lane;
    ab = above2 + hi;
    cnt = lo;
  }
  const unsigned f2 = __ballot_sync(0xffffffffu, b >= 0);
  if (lane == __ffs(f2) - 1) {
    bc[0] = b;
    bc[1] = ab;
    bc[2] = cnt;
  }
}

template <int CPL>
struct LaneVec;  // the lane's CPL fp16 channels of one row
template <>
struct LaneVec<4> {
  using T = uint2;
};
template <>
struct LaneVec<2> {
  using T = uint32_t;
};

// A lane's CPL fp16 channels packed in LaneVec words, handled by value
// (taking a register's address would move it to local memory): to and
// from floats, per-half max / min, and a repeated half2 pattern.
__device__ __forceinline__ __half2 u32_h2(uint32_t u) {
  return __halves2half2(__ushort_as_half(static_cast<unsigned short>(u & 0xffffu)),
                        __ushort_as_half(static_cast<unsigned short>(u >> 16)));
}
__device__ __forceinline__ uint32_t h2_u32(__half2 h) {
  return static_cast<uint32_t>(__half_as_ushort(__low2half(h))) |
         (static_cast<uint32_t>(__half_as_ushort(__high2half(h))) << 16);
}
template <int CPL>
__device__ __forceinline__ void vec_to_float(typename LaneVec<CPL>::T v, float f[CPL]) {
  if constexpr (CPL == 4) {
    const float2 a = __half22float2(u32_h2(v.x)), b = __half22float2(u32_h2(v.y));
    f[0] = a.x; f[1] = a.y; f[2] = b.x; f[3] = b.y;
  } else {
    const float2 a = __half22float2(u32_h2(v));
    f[0] = a.x; f[1] = a.y;
  }
}
template <int CPL>
__device__ __forceinline__ typename LaneVec<CPL>::T float_to_vec(const float f[CPL]) {
  if constexpr (CPL == 4) {
    return make_uint2(h2_u32(__floats2half2_rn(f[0], f[1])), h2_u32(__floats2half2_rn(f[2], f[3])));
  } else {
    return h2_u32(__floats2half2_rn(f[0], f[1]));
  }
}
template <int CPL>
__device__ __forceinline__ typename LaneVec<CPL>::T vec_hmax(typename LaneVec<CPL>::T a,
                                                              typename LaneVec<CPL>::T b) {
  if constexpr (CPL == 4) {
    return make_uint2(h2_u32(__hmax2(u32_h2(a.x), u32_h2(b.x))),
                      h2_u32(__hmax2(u32_h2(a.y), u32_h2(b.y))));
  } else {
    return h2_u32(__hmax2(u32_h2(a), u32_h2(b)));
  }
}
template <int CPL>
__device__ __forceinline__ typename LaneVec<CPL>::T vec_hmin(typename LaneVec<CPL>::T a,
                                                              typename LaneVec<CPL>::T b) {
  if constexpr (CPL == 4) {
    return make_uint2(h2_u32(__hmin2(u32_h2(a.x), u32_h2(b.x))),
                      h2_u32(__hmin2(u32_h2(a.y), u32_h2(b.y))));
  } else {
    return h2_u32(__hmin2(u32_h2(a), u32_h2(b)));
  }
}
template <int CPL>
__device__ __forceinline__ typename LaneVec<CPL>::T vec_fill(uint32_t pattern) {
  if constexpr (CPL == 4) {
    return make_uint2(pattern, pattern);
  } else {
    return pattern;
  }
}

// RoPE of the lane's CPL channels of one row held as floats (channel
// lane * CPL + t); the partner of a channel (j <-> j + D/2) sits 16 lanes
// away. The values come back rounded to fp16, as the stand-alone kernel
// stores them. Every lane of the warp takes part.
template <int CPL>
__device__ __forceinline__ void cs_rope_lane(float v[CPL], int lane, int D, float pos,
                                             float rcp_scale, float log2_rcp_theta) {
  float p[CPL];
#pragma unroll
  for (int t = 0; t < CPL; ++t) p[t] = __shfl_xor_sync(0xffffffffu, v[t], 16);
  const bool lo = lane < 16;
#pragma unroll
  for (int t = 0; t < CPL; ++t) {
    __half o0, o1;
    rope_pair(lo ? v[t] : p[t], lo ? p[t] : v[t], (lane & 15) * CPL + t, D, pos, rcp_scale,
              log2_rcp_theta, &o0, &o1);
    v[t] = __half2float(lo ? o0 : o1);
  }
}

template <int D, int C>
__global__ void __launch_bounds__(kCsThreads, 1)
    cluster_step_kernel(const __grid_constant__ CUtensorMap kv_map,
                        const __grid_constant__ CUtensorMap meta_map, ClusterStepArgs a_in,
                        CsShape shp) {
  constexpr int CPL = D / 32;           // channels per lane
  const int CAPL = cs_capl(C, shp.max_slots);  // local candidates one CTA may publish
  using Vec = typename LaneVec<CPL>::T;
  extern __shared__ uint8_t smem_raw[];
  // (rounded as an integer: measured faster here than align_smem's shared-
  // window pointer, 22.0 vs 22.8 us per layer-step at the headline shape)
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  __shared__ uint64_t bars[kCsWarps];
  __shared__ uint64_t merge_bar;  // CTA 0: the other CTAs' partial states are in
  __shared__ CsXchg xs;
  __shared__ int bc[3];  // threshold bin, count above it, count in it
  __shared__ int peer_cnt[C], peer_off[C + 1];
  __shared__ float gsh[2];
  __shared__ uint32_t kmin_s, kmax_s;     // key range of this CTA's ranked scores
  __shared__ int cnt_s;
  __shared__ int peer_m[C], peer_ovf[C];  // every CTA's candidate count and overflow flag
  __shared__ __align__(16) __half q_rot[128];  // head h's q (after RoPE when fused)

  cg::cluster_group cluster = cg::this_cluster();
  const int c = static_cast<int>(cluster.block_rank());
  const int h = blockIdx.y;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int P = a_in.P, H = a_in.H;
  const CsLayout lay = cs_layout(D, P, C, shp.max_local, shp.max_slots);
  uint8_t* slot = smem + lay.ring + warp * cs_slot_bytes(D, P);
  float* sc = reinterpret_cast<float*>(smem + lay.scores);
  uint8_t* st = smem + lay.state;
  int* pidl = reinterpret_cast<int*>(smem + lay.pidl);
  uint32_t* hist = reinterpret_cast<uint32_t*>(smem + lay.hist);
  uint4* cand = reinterpret_cast<uint4*>(smem + lay.cand);
  uint4* lst = reinterpret_cast<uint4*>(smem + lay.lst);
  uint32_t* gkey = reinterpret_cast<uint32_t*>(smem + lay.gkey);
  uint32_t* gpos = reinterpret_cast<uint32_t*>(smem + lay.gpos);
  int* items = reinterpret_cast<int*>(smem + lay.items);
  float* mrg = reinterpret_cast<float*>(smem + lay.mrg);
  float* xo = reinterpret_cast<float*>(smem + lay.xo);
  uint64_t* bar = &bars[warp];
  const uint32_t tile_bytes = static_cast<uint32_t>(P * D * 2);

  if (tid == 0) {
    for (int i = 0; i < kCsWarps; ++i) mbar_init(&bars[i], 1);
    mbar_init(&merge_bar, C > 1 ? C - 1 : 1);
    fence_mbar_init();
    tma_prefetch_desc(&kv_map);
    tma_prefetch_desc(&meta_map);
    kmin_s = 0xffffffffu;
    kmax_s = 0u;
    cnt_s = 0;
  }
  for (int b = tid; b < kCsBins; b += kCsThreads) hist[b] = 0u;
  __syncthreads();
  cluster_arrive_relaxed();  // merge_bar initialised (fence.mbarrier_init above; waited for
                             // before any remote access)
  // Everything in global memory may be written by the previous kernel on
  // the stream (under programmatic dependent launch it can still be
  // running), so every global read comes after this wait.
  pdl_wait();
  pdl_launch_dependents();

  // The arguments stay in parameter space (a copy of the whole struct would
  // live in local memory); the fields a batched launch moves per request
  // are copied into registers.
  const ClusterStepArgs& a = a_in;
  const __half* q_in = a.q;
  const __half* kn_in = a.k_new;
  const __half* vn_in = a.v_new;
  __half* o_out = a.o;
  const int32_t* kv_idx = a.kv_indices;
  const int32_t* meta_idx = a.meta_indices;
  int n_pages = a.n_pages, last_len = a.last_len, k_slots = a.k_slots;
  int32_t* sel_out = a.selected_out;
  if (a.kv_indptr) {  // batched: request blockIdx.z of a shared page pool
    const int r = blockIdx.z;
    const int p0 = __ldcg(a.kv_indptr + r);
    const int m0 = __ldcg(a.meta_indptr + r);
    n_pages = __ldcg(a.kv_ends ? a.kv_ends + r : a.kv_indptr + r + 1) - p0;
    last_len = __ldcg(a.last_lens + r);
    if (a.kv_ends && n_pages == 0) return;  // an empty page-table slot
    // every CTA of the cluster reads the same values, so all leave together
    // (no cluster barrier is pending: the arrival above needs no wait)
    if (p0 < 0 || m0 < 0 || n_pages < 1 || n_pages > a.max_pages || last_len < 1 ||
        last_len > P) {
      if (tid == 0) raise_dev_error(a.err, AOAKV_DEV_ERR_BAD_PAGE);
      return;
    }
    kv_idx += p0;
    meta_idx += m0;
    const int kp = a.sink ? max(3, a.budget) : a.budget;
    k_slots = min(kp, n_pages);
    const size_t qo = static_cast<size_t>(r) * H * D;
    q_in += qo;
    kn_in += qo;
    vn_in += qo;
    o_out += qo;
    if (sel_out) sel_out += static_cast<size_t>(r) * H * a.sel_cols;
  }
  const int N = n_pages, n = N - 1;
  const int k = k_slots;
  const int shard = a.shard;
  // propose scores and ranks every local page (even when they are <= k);
  // finish scores nothing
  const bool sparse = shard == kShardPropose ? n >= 1 : (shard == kShardNone && N > k && k > 1);
  const bool aoa = a.mode == AOAKV_SCORE_AOAKV;
  const int n_st = sparse ? (n + P - 1) / P : 0;  // metadata pages holding scored pages
  const int st_lo = (c * n_st) / C, st_hi = ((c + 1) * n_st) / C;
  const int pos_lo = st_lo * P;
  const int nloc = sparse ? max(0, min(n, st_hi * P) - pos_lo) : 0;
  const int r_lo = a.sink ? 1 : 0;
  // attended slots: the selected pages, then the last page; CTA c decodes
  // slots [s_lo, s_hi), so the last page falls to CTA C-1
  const int T = sparse ? k : (N <= k ? N : 1);
  const int s_lo = (c * T) / C, s_hi = ((c + 1) * T) / C;
  // ids of the last page (attended by CTA C-1, which also appends to it);
  // a propose pass, or a finish pass on a GPU without it, has none
  const bool has_last = shard == kShardNone || (shard == kShardFinish && a.owns_last);
  const int w_last = (c == C - 1 && has_last) ? (shard ? 0 : (T - 1 - s_lo) % kCsWarps) : -1;
  const int last_pid = has_last ? __ldcg(kv_idx + N - 1) : -1;
  const int app_mpid = (c == C - 1 && has_last) ? __ldcg(meta_idx + (N - 1) / P) : 0;
  if (warp == w_last && lane == 0 && last_pid >= 0 && last_pid < a.kv_cap) {  // warm L2
#pragma unroll
    for (int sub = 0; sub < D / 64; ++sub) {
      tma_prefetch_l2_3d(&kv_map, 64 * sub, h, last_pid * 2 * P);
      tma_prefetch_l2_3d(&kv_map, 64 * sub, h, last_pid * 2 * P + P);
    }
  }

  float qv[CPL];
  load_row<CPL>(q_in + static_cast<size_t>(h) * D + lane * CPL, qv);
  const float rope_pos = static_cast<float>(a.rope_pos >= 0 ? a.rope_pos
                                                            : (N - 1) * P + last_len - 1);
  // every warp rotates its copy (RoPE fused); warp 0 keeps q in shared
  // memory for the decode
  if (a.rope) cs_rope_lane<CPL>(qv, lane, D, rope_pos, a.rope_rcp_scale, a.rope_log2_rcp_theta);
  if (warp == 0)
#pragma unroll
    for (int t = 0; t < CPL; ++t) q_rot[lane * CPL + t] = __float2half_rn(qv[t]);
  uint32_t msk[CPL / 2];
#pragma unroll
  for (int i = 0; i < CPL / 2; ++i)
    msk[i] = (qv[2 * i] > 0.f ? 0x0000ffffu : 0u) | (qv[2 * i + 1] > 0.f ? 0xffff0000u : 0u);
  uint32_t par = 0;  // phase of this warp's ring-slot barrier

  // ------------------------------------------------------------ 1 scoring
  if (sparse) {
    const int jp = (lane >> 1) & 15;           // page of the stage this lane scores
    const bool writer = (lane & 1) == 0 && jp < P;
    // the metadata page of stage t and the lane's page id / v_log_norm
    auto meta_of = [&](int t) -> int { return lane == 0 ? __ldcg(meta_idx + t) : 0; };
    auto page_of = [&](int t, float* vlo) -> int {
      const int pos = t * P + jp;
      *vlo = 0.f;
      if (!writer || pos >= n) return -1;
      const int pid = __ldcg(kv_idx + pos);
      if (pid < 0 || pid >= a.kv_cap) {
        raise_dev_error(a.err, AOAKV_DEV_ERR_BAD_PAGE);
        *vlo = NAN;
        return -1;
      }
      if (aoa) *vlo = __half2float(__ldcg(a.vlog + static_cast<size_t>(pid) * H + h));
      return pid;
    };
    auto issue = [&](int mp) -> bool {
      int ok = 0;
      if (lane == 0) {
        if (mp >= 0 && mp < a.meta_cap) {
          ok = 1;
          mbar_arrive_expect_tx(bar, 2u * tile_bytes);
          tma_load_3d(slot, &meta_map, 0, h, mp * 2 * P, bar);
          tma_load_3d(slot + tile_bytes, &meta_map, 0, h, mp * 2 * P + P, bar);
        } else {
          raise_dev_error(a.err, AOAKV_DEV_ERR_BAD_PAGE);
        }
      }
      return __shfl_sync(0xffffffffu, ok, 0) != 0;
    };
    uint32_t kmin_l = 0xffffffffu, kmax_l = 0u;
    int t = st_lo + warp;
    bool ok = false;
    float vl = 0.f;
    int pg = -1;
    int mp_next = 0;
    if (t < st_hi) {
      ok = issue(meta_of(t));
      pg = page_of(t, &vl);
      if (t + kCsWarps < st_hi) mp_next = meta_of(t + kCsWarps);  // one stage ahead
    }
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
      const int pg_t = pg;
      const int pos = t * P + jp;
      // Every lane has consumed the slot (its values are in `part`) before
      // lane 0 refills it: the TMA write cannot overtake these reads.
      __syncwarp();
      const int tn = t + kCsWarps;
      if (tn < st_hi) {
        ok = issue(mp_next);
        pg = page_of(tn, &vl);
        if (tn + kCsWarps < st_hi) mp_next = meta_of(tn + kCsWarps);
      }
      if (writer && pos < n) {
        const float score = !got ? NAN : (aoa ? a.two_rsqrt_d * s + 2.f * vl_t : s);
        const int i = pos - pos_lo;
        sc[i] = score;
        pidl[i] = pg_t;
        const uint8_t s0 = pos >= r_lo ? 1 : 2;  // the sink page is forced
        st[i] = s0;
        if (s0 == 1 && isfinite(score)) {
          const uint32_t kk = float_to_key(score);
          kmin_l = min(kmin_l, kk);
          kmax_l = max(kmax_l, kk);
        }
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      kmin_l = min(kmin_l, __shfl_xor_sync(0xffffffffu, kmin_l, o));
      kmax_l = max(kmax_l, __shfl_xor_sync(0xffffffffu, kmax_l, o));
    }
    if (lane == 0 && kmin_l <= kmax_l) {
      atomicMin(&kmin_s, kmin_l);
      atomicMax(&kmax_s, kmax_l);
    }
  }
  __syncthreads();
  cluster_wait_acquire();  // every CTA's merge_bar is initialised

  // ---------------------------------------------------------- 2 selection
  // Fast path: each CTA sorts its local candidates — every ranked page whose
  // score reaches the bin of the CTA's K-th largest, a superset of its share
  // of the global top-K — by (score desc, page asc); its winners are a
  // prefix of that list. Before the one cluster barrier it starts the TMA
  // loads of its first candidates' K/V pages into the ring (and warms L2
  // with a few more); after it, each CTA copies the other lists and ranks
  // its own candidates by binary search in them: a rank below K is a
  // winner, attended by this CTA. A CTA with more than CAPL candidates
  // (many equal scores) sends the whole cluster to the level-by-level
  // fallback, whose winners are spread evenly over the cluster.
  int32_t* sel_row =
      sel_out ? sel_out + static_cast<size_t>(h) * a.sel_cols : nullptr;
  const bool sink_owner = sparse && a.sink && st_lo == 0 && st_hi > 0;
  // pages attended whatever the selection: the last page (CTA C-1, first),
  // the sink page (its owner)
  const int n_special = (c == C - 1 ? 1 : 0) + (sink_owner ? 1 : 0);
  int n_spec = 0;    // items whose pages were loaded before the selection ended
  int n_items = 0;   // pages this CTA attends
  int last_item = -1;
  bool spec_issued = false;  // this warp's slot holds a speculative load
  bool fast = true;
  auto load_page = [&](int pid) {  // lane 0: the page's K and V tiles into the warp's slot
    fence_proxy_async_smem();  // the slot may hold rows written by this warp (the append)
    mbar_arrive_expect_tx(bar, 2u * tile_bytes);
#pragma unroll
    for (int sub = 0; sub < D / 64; ++sub) {
      tma_load_3d(slot + sub * kCsSubTile, &kv_map, 64 * sub, h, pid * 2 * P, bar);
      tma_load_3d(slot + (D / 64 + sub) * kCsSubTile, &kv_map, 64 * sub, h, pid * 2 * P + P, bar);
    }
  };
  auto warm_page = [&](int pid) {  // L2 prefetch of a page's K and V
#pragma unroll
    for (int sub = 0; sub < D / 64; ++sub) {
      tma_prefetch_l2_3d(&kv_map, 64 * sub, h, pid * 2 * P);
      tma_prefetch_l2_3d(&kv_map, 64 * sub, h, pid * 2 * P + P);
    }
  };
  int n_out = 0;  // propose: entries of this head's cand_out written, best first
  if (shard == kShardFinish) {
    // This GPU's list holds its best pages, best first: rank each entry
    // against the other GPUs' lists; the winners are a prefix of the list.
    const int np = a.n_prop, G = a.world, me = a.rank;
    const int n_mine = N - (a.owns_last ? 1 : 0);  // local pages besides the last
    int w = 0;
    if (np > 0) {
      if (a.p2p) {  // every GPU's list, from this GPU's mailbox, once tagged with this epoch
        const uint32_t epoch =
            __ldcg(reinterpret_cast<const uint32_t*>(a.mail.base[me] + a.mail.ep_off)) + 1u;
        const uint64_t* box = reinterpret_cast<const uint64_t*>(a.mail.base[me] + a.mail.cand_off);
        for (int g = tid; g < G * np; g += kCsThreads) {
          const int gg = g / np, i = g - gg * np;
          const uint2 e =
              tagged_wait2_sys(box + ((static_cast<size_t>(gg) * H + h) * np + i) * 2, epoch, a.err);
          gkey[g] = e.x;
          gpos[g] = e.y;
        }
      } else {
        for (int g = tid; g < G * np; g += kCsThreads) {
          const int gg = g / np, i = g - gg * np;
          const uint2 e = __ldcg(a.cand_in + (static_cast<size_t>(gg) * H + h) * np + i);
          gkey[g] = e.x;
          gpos[g] = e.y;
        }
      }
      __syncthreads();
      // global rank of entry i of list g: i plus, in every other list, the
      // entries that beat it (a prefix: binary search)
      auto rank_of = [&](int g, int i) -> int {
        const uint32_t mk = gkey[g * np + i], mp = gpos[g * np + i];
        int r = i;
        for (int gg = 0; gg < G; ++gg) {
          if (gg == g) continue;
          int lo = gg * np, hi = lo + np;
          while (lo < hi) {
            const int mid = (lo + hi) >> 1;
            if (cs_beats(gkey[mid], gpos[mid], mk, mp)) lo = mid + 1;
            else hi = mid;
          }
          r += lo - gg * np;
        }
        return r;
      };
      bool win = false;
      if (tid < np) win = gpos[me * np + tid] != 0xffffffffu && rank_of(me, tid) < np;
      w = __syncthreads_count(win);
      if (sel_row)  // every list's winners, by rank (lists c, c + C, ... here)
        for (int g = c; g < G; g += C)
          for (int i = tid; i < np; i += kCsThreads)
            if (gpos[g * np + i] != 0xffffffffu) {
              const int r = rank_of(g, i);
              if (r < np) sel_row[r] = static_cast<int>(gpos[g * np + i]);
            }
    }
    // attended here: the winners (or every local page when dense), then
    // the last page on its owner; CTA c takes slots [lo_s, hi_s)
    const int Tl = (np > 0 ? w : (a.dense ? n_mine : 0)) + (a.owns_last ? 1 : 0);
    const int lo_s = (c * Tl) / C, hi_s = ((c + 1) * Tl) / C;
    for (int j = lo_s + tid; j < hi_s; j += kCsThreads) {
      int pid = -1;
      if (a.owns_last && j == Tl - 1) {
        pid = last_pid;
      } else if (np > 0) {
        const int li = static_cast<int>(gpos[me * np + j]) - a.page_lo;
        if (li >= 0 && li < n_mine) pid = __ldcg(kv_idx + li);  // else BAD_PAGE below
      } else {
        pid = __ldcg(kv_idx + j);
      }
      items[j - lo_s] = pid;
    }
    n_items = hi_s - lo_s;
    last_item = (a.owns_last && c == C - 1) ? Tl - 1 - lo_s : -1;
  }
  if (sparse) {
    const int K = (k - 1) - r_lo;  // pages to choose among the ranked ones (>= 1)
    const int rk0 = min(nloc, max(0, r_lo - pos_lo));  // first ranked local index
    const int n_rank = nloc - rk0;
    int lb = -1;  // local threshold bin; -1: every ranked page is a candidate
    float lmin = 0.f, lscale = 0.f;
    if (n_rank > K) {
      if (kmin_s <= kmax_s) {
        lmin = key_to_float(kmin_s);
        const float lmax = key_to_float(kmax_s);
        const float r = lmax - lmin;
        const float sc0 = static_cast<float>(kCsLinBins) / r;
        lscale = (r > 0.f && r < INFINITY && sc0 < INFINITY) ? sc0 : 0.f;
      }
      for (int i = rk0 + tid; i < nloc; i += kCsThreads)
        atomicAdd(&hist[cs_bin_mul(sc[i], lmin, lscale)], 1u);
      __syncthreads();
      if (warp == 0) cs_threshold_warp(hist, K, bc);
      __syncthreads();
      lb = bc[0];
    }
    for (int i0 = rk0 + warp * 32; i0 < nloc; i0 += kCsThreads) {  // one atomic per warp
      const int i = i0 + lane;
      const bool in = i < nloc && (lb < 0 || cs_bin_mul(sc[i], lmin, lscale) >= lb);
      const unsigned bal = __ballot_sync(0xffffffffu, in);
      int base = 0;
      if (lane == 0 && bal) base = atomicAdd(&cnt_s, __popc(bal));
      base = __shfl_sync(0xffffffffu, base, 0);
      const int j = base + __popc(bal & ((1u << lane) - 1u));
      if (in && j < CAPL)
        cand[j] = make_uint4(float_to_key(sc[i]), static_cast<uint32_t>(pos_lo + i),
                             static_cast<uint32_t>(pidl[i]), 0u);
    }
    __syncthreads();
    const int m_c = cnt_s;
    if (m_c <= CAPL) {
      // sort by counting, TPC threads per candidate
      int m2 = 1;
      while (m2 < m_c) m2 <<= 1;
      const int tpc = m2 >= kCsThreads ? 1 : (kCsThreads / m2 > 32 ? 32 : kCsThreads / m2);
      for (int base = 0; base < m_c; base += kCsThreads / tpc) {
        const int i = base + tid / tpc, sub = tid % tpc;
        int r = 0;
        uint4 me = make_uint4(0u, 0u, 0u, 0u);
        if (i < m_c) {
          me = cand[i];
          int j = sub;
          for (; j + 3 * tpc < m_c; j += 4 * tpc) {  // four independent loads in flight
            const uint4 o0 = cand[j], o1 = cand[j + tpc], o2 = cand[j + 2 * tpc],
                        o3 = cand[j + 3 * tpc];
            r += cs_beats(o0.x, o0.y, me.x, me.y) + cs_beats(o1.x, o1.y, me.x, me.y) +
                 cs_beats(o2.x, o2.y, me.x, me.y) + cs_beats(o3.x, o3.y, me.x, me.y);
          }
          for (; j < m_c; j += tpc) {
            const uint4 o = cand[j];
            r += cs_beats(o.x, o.y, me.x, me.y);
          }
        }
        for (int off = tpc >> 1; off > 0; off >>= 1) r += __shfl_xor_sync(0xffffffffu, r, off);
        if (i < m_c && sub == 0) lst[r] = me;
      }
    }
    // Peers read the first K entries of this list (K * C <= kCsGather, else
    // the cluster takes the fallback): slots past the candidates hold an
    // entry that beats nothing and never wins.
    const bool gatherable = K * C <= kCsGather;
    if (tid == 0) {
      xs.m = m_c;
      xs.ovf = m_c > CAPL || !gatherable;
    }
    if (gatherable && m_c < K)
      for (int j = m_c + tid; j < K; j += kCsThreads)
        lst[j] = make_uint4(0u, 0xffffffffu, 0xffffffffu, 0u);
    __syncthreads();
    // Publish (release) first, then start the likely winners' loads, so the
    // release never waits for them: K/V of the first candidates into the
    // ring, a few more warmed in L2.
    cluster_arrive_release();
    if (m_c <= CAPL && shard == kShardNone) {
      n_spec = min(kCsWarps, n_special + m_c);
      if (warp < n_spec) {
        const int pid = warp < n_special
                            ? ((c == C - 1 && warp == 0) ? last_pid : __ldcg(kv_idx))
                            : static_cast<int>(lst[warp - n_special].z);
        spec_issued = pid >= 0 && pid < a.kv_cap;
        if (lane == 0 && spec_issued) load_page(pid);
      }
      const int npf = min(m_c, (5 * K + 4 * C - 1) / (4 * C) + 2);
      const int j0 = kCsWarps - n_special;
      if (tid + j0 < npf) {
        const int pid = static_cast<int>(lst[tid + j0].z);
        if (pid >= 0) warm_page(pid);
      }
    }
    cluster_wait_acquire();  // local candidate lists published
    // One round of distributed shared memory: every CTA's count, overflow
    // flag and first K entries (a winner ranks below K in its own list).
    if (tid < C) {
      const CsXchg* px = cluster.map_shared_rank(&xs, tid);
      peer_m[tid] = px->m;
      peer_ovf[tid] = px->ovf;
    }
    uint2* gkp = reinterpret_cast<uint2*>(gkey);  // {key, page} pairs: gkey and gpos regions
    if (gatherable)
      for (int g = tid; g < C * K; g += kCsThreads) {
        const int cc = g / K;
        const uint4 e = cluster.map_shared_rank(lst, cc)[g - cc * K];
        gkp[g] = make_uint2(e.x, e.y);
      }
    __syncthreads();
#pragma unroll
    for (int cc = 0; cc < C; ++cc) fast = fast && peer_ovf[cc] == 0;
    if (fast) {
      int M = 0;
#pragma unroll
      for (int cc = 0; cc < C; ++cc) M += min(peer_m[cc], K);
      n_out = r_lo + min(K, M);
      const int mine = min(m_c, K);
      // rank of own entry i: i plus the entries of the other lists that beat
      // it. Few entries: tpc threads count them in parallel; many: one
      // thread binary-searches each list.
      int k2 = 1;
      while (k2 < K) k2 <<= 1;
      const int tpc = k2 >= kCsThreads ? 1 : (kCsThreads / k2 > 32 ? 32 : kCsThreads / k2);
      const bool count = (C - 1) * K <= 64 * tpc;
      bool win = false;
      int i = tid, r = 0;
      if (count) {
        i = tid / tpc;
        const int sub = tid - i * tpc;
        if (i < mine) {
          const uint2 me = gkp[c * K + i];
#pragma unroll
          for (int cc = 0; cc < C; ++cc) {
            if (cc == c) continue;
#pragma unroll 4
            for (int g = cc * K + sub; g < (cc + 1) * K; g += tpc) {
              const uint2 e = gkp[g];
              r += cs_beats(e.x, e.y, me.x, me.y);
            }
          }
        }
        for (int off = tpc >> 1; off > 0; off >>= 1) r += __shfl_xor_sync(0xffffffffu, r, off);
        r += i;
        win = i < mine && sub == 0 && r < K;
      } else if (i < mine) {
        const uint32_t mk = gkp[c * K + i].x, mpos = gkp[c * K + i].y;
        int lo[C], hi[C];  // binary searches of all lists in lockstep
#pragma unroll
        for (int cc = 0; cc < C; ++cc) {
          lo[cc] = cc * K;
          hi[cc] = cc == c ? cc * K : cc * K + min(peer_m[cc], K);
        }
        bool more = true;
        while (more) {
          more = false;
#pragma unroll
          for (int cc = 0; cc < C; ++cc) {
            if (lo[cc] < hi[cc]) {
              const int mid = (lo[cc] + hi[cc]) >> 1;
              const uint2 e = gkp[mid];
              if (cs_beats(e.x, e.y, mk, mpos)) lo[cc] = mid + 1;
              else hi[cc] = mid;
              more = true;
            }
          }
        }
        r = i;
#pragma unroll
        for (int cc = 0; cc < C; ++cc)
          if (cc != c) r += lo[cc] - cc * K;
        win = r < K;
      }
      if (win && sel_row) sel_row[r + r_lo] = static_cast<int>(lst[i].z);
      if (win && shard == kShardPropose)
        a.cand_out[static_cast<size_t>(h) * a.n_prop + r + r_lo] =
            make_uint2(lst[i].x, static_cast<uint32_t>(a.page_lo) + lst[i].y);
      const int w_c = __syncthreads_count(win);  // the winners are lst[0, w_c)
      n_items = n_special + w_c;
      for (int j = tid; j < n_items; j += kCsThreads)
        items[j] = j < n_special ? ((c == C - 1 && j == 0) ? last_pid : __ldcg(kv_idx))
                                 : static_cast<int>(lst[j - n_special].z);
      if (c == C - 1) last_item = 0;
      if (sel_row && tid == 0) {
        if (sink_owner) sel_row[0] = __ldcg(kv_idx);
        if (c == C - 1) sel_row[T - 1] = last_pid;
      }
    } else {
      // ---- fallback: exact selection by levels over the whole cluster
      uint2* candall = reinterpret_cast<uint2*>(gkey);  // gkey and gpos: 2 * kCsGather words
      uint2* cand2 = reinterpret_cast<uint2*>(cand);
      int* sel = pidl;  // this CTA's selected pages (positions), page order
      int need = K;
      for (int level = 0; need > 0; ++level) {
        // A: finite range of the candidates (state 1), cluster-wide
        float lo = INFINITY, hi = -INFINITY;
        for (int i = tid; i < nloc; i += kCsThreads) {
          if (st[i] != 1) continue;
          const float x = sc[i];
          if (isfinite(x)) {
            lo = fminf(lo, x);
            hi = fmaxf(hi, x);
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
              cand2[atomicAdd(&cnt_s, 1)] =
                  make_uint2(float_to_key(sc[i]), static_cast<uint32_t>(pos_lo + i));
          __syncthreads();
          cluster.sync();  // candidate lists published
          for (int g = tid; g < cnt; g += kCsThreads) {
            int cc = 0, off = 0;
            while (cc < C - 1 && g >= off + peer_cnt[cc]) off += peer_cnt[cc++];
            candall[g] = cluster.map_shared_rank(cand2, cc)[g - off];
          }
          __syncthreads();
          for (int i = tid; i < cnt_s; i += kCsThreads) {
            const uint2 me = cand2[i];
            int r = 0;
            for (int g = 0; g < cnt; ++g) {
              const uint2 o = candall[g];
              r += cs_beats(o.x, o.y, me.x, me.y);
            }
            st[me.y - pos_lo] = r < need2 ? 2 : 0;
          }
          __syncthreads();
          break;
        }
        need = need2;  // refine inside the threshold bin
      }
      {  // this CTA's selected pages in page order (sink page 0 included)
        const int ch = (nloc + kCsThreads - 1) / kCsThreads;
        const int i0 = min(nloc, tid * ch), i1 = min(nloc, i0 + ch);
        int m = 0;
        for (int i = i0; i < i1; ++i) m += st[i] == 2;
        int tot_sel;
        int w = cs_block_scan(m, &tot_sel);
        for (int i = i0; i < i1; ++i)
          if (st[i] == 2) sel[w++] = pos_lo + i;
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
      if (shard == kShardPropose) {
        // the selected pages of every CTA with their keys (the sink page
        // above all), each CTA ranking its own by (key, page)
        const int own = peer_off[c + 1] - peer_off[c], total = peer_off[C];
        for (int j = tid; j < own; j += kCsThreads) {
          const int pos = sel[j];
          const uint32_t key =
              (a.sink && pos == 0) ? 0xffffffffu : float_to_key(sc[pos - pos_lo]);
          cand2[j] = make_uint2(key, static_cast<uint32_t>(pos));
        }
        __syncthreads();
        cluster.sync();  // keyed lists published
        for (int g = tid; g < total; g += kCsThreads) {
          int cc = 0;
          while (cc < C - 1 && g >= peer_off[cc + 1]) ++cc;
          candall[g] = cluster.map_shared_rank(cand2, cc)[g - peer_off[cc]];
        }
        __syncthreads();
        for (int j = tid; j < own; j += kCsThreads) {
          const uint2 me = cand2[j];
          int r = 0;
          for (int g = 0; g < total; ++g) r += cs_beats(candall[g].x, candall[g].y, me.x, me.y);
          a.cand_out[static_cast<size_t>(h) * a.n_prop + r] =
              make_uint2(me.x, static_cast<uint32_t>(a.page_lo) + me.y);
        }
        n_out = total;
      } else {
        // the page ids of this CTA's decode slots, from the owners' lists
        for (int sl = s_lo + tid; sl < min(s_hi, T - 1); sl += kCsThreads) {
          int pid = -1;
          if (sl < peer_off[C]) {
            int cc = 0;
            while (cc < C - 1 && sl >= peer_off[cc + 1]) ++cc;
            const int pos = cluster.map_shared_rank(sel, cc)[sl - peer_off[cc]];
            if (pos >= 0 && pos < N) pid = __ldcg(kv_idx + pos);
          }
          items[sl - s_lo] = pid;
          if (sel_row) sel_row[sl] = pid;
        }
      }
    }
  } else if (shard == kShardNone) {
    for (int sl = s_lo + tid; sl < min(s_hi, T - 1); sl += kCsThreads) {  // every page
      const int pid = __ldcg(kv_idx + sl);
      items[sl - s_lo] = pid;
      if (sel_row) sel_row[sl] = pid;
    }
  }
  if (shard == kShardNone && (!sparse || !fast)) {
    n_items = s_hi - s_lo;
    if (c == C - 1) {
      last_item = T - 1 - s_lo;
      if (tid == 0) {
        items[last_item] = last_pid;
        if (sel_row) sel_row[T - 1] = last_pid;
      }
    }
  }
  if (sel_row && c == C - 1 && shard == kShardNone)
    for (int i = T + tid; i < a.sel_cols; i += kCsThreads) sel_row[i] = -1;
  if (shard == kShardPropose && c == 0) {  // the sink page first; unused entries last
    uint2* out = a.cand_out + static_cast<size_t>(h) * a.n_prop;
    if (sink_owner && tid == 0) out[0] = make_uint2(0xffffffffu, static_cast<uint32_t>(a.page_lo));
    for (int i = n_out + tid; i < a.n_prop; i += kCsThreads) out[i] = make_uint2(0u, 0xffffffffu);
  }
  __syncthreads();
  if (shard == kShardPropose) {
    // No decode. The barrier also makes every CTA's entries of cand_out
    // visible to CTA 0, which (with mailboxes) forwards the head's list to
    // every other GPU and raises fc there.
    cluster_arrive_release();
    cluster_wait_acquire();
    if (a.p2p && c == 0) {  // the head's list, tagged, into every GPU's mailbox
      const int np = a.n_prop;
      const uint32_t epoch =
          __ldcg(reinterpret_cast<const uint32_t*>(a.mail.base[a.rank] + a.mail.ep_off)) + 1u;
      const uint2* src = a.cand_out + static_cast<size_t>(h) * np;
      for (int i = tid; i < np; i += kCsThreads) {
        const uint2 e = __ldcg(src + i);
        for (int g = 0; g < a.world; ++g) {
          uint64_t* w = reinterpret_cast<uint64_t*>(a.mail.base[g] + a.mail.cand_off) +
                        ((static_cast<size_t>(a.rank) * H + h) * np + i) * 2;
          tagged_store2_sys(w, e.x, e.y, epoch);
        }
      }
    }
    return;
  }
  // no shared memory of a peer is read after this point (the values read are
  // consumed), so the arrival need not order anything
  cluster_arrive_relaxed();

  // ------------------------------------------------------------- 3 decode
  // q as column 0 of the B operand of S^T = K q^T (lanes 0..3: channels
  // 16kk + 2t, +1 and 16kk + 2t + 8, +9)
  constexpr int NK = D / 16;
  uint32_t qb[NK][2];
#pragma unroll
  for (int kk = 0; kk < NK; ++kk) {
    qb[kk][0] = qb[kk][1] = 0u;
    if (lane < 4) {
      const uint32_t* qw = reinterpret_cast<const uint32_t*>(q_rot);
      qb[kk][0] = qw[kk * 8 + lane];
      qb[kk][1] = qw[kk * 8 + 4 + lane];
    }
  }
  float m = -INFINITY, l = 0.f, acc[NK][4];
#pragma unroll
  for (int mm = 0; mm < NK; ++mm)
#pragma unroll
    for (int i = 0; i < 4; ++i) acc[mm][i] = 0.f;
  const uint32_t kb = smem_addr(slot), vb = kb + (D / 64) * kCsSubTile;
  const size_t HD = static_cast<size_t>(H) * D;
  const size_t col = static_cast<size_t>(h) * D + lane * CPL;
  const bool preloaded = sparse && fast;  // items [0, n_spec) sit in the warps' slots
  if (spec_issued && (!preloaded || warp >= n_items)) {  // loaded but not attended: drain
    mbar_wait_bounded(bar, par, a.err);
    par ^= 1u;
  }
  for (int j = warp; j < n_items; j += kCsWarps) {
    const bool is_last = j == last_item;
    int pid = items[j];
    if (pid < 0 || pid >= a.kv_cap) {
      if (lane == 0) raise_dev_error(a.err, AOAKV_DEV_ERR_BAD_PAGE);
      continue;
    }
    if (!(preloaded && j < n_spec)) {  // (a preloaded item's load is spec_issued)
      if (lane == 0) load_page(pid);
      __syncwarp();
    }
    const int ntok = is_last ? last_len : P;
    // the new token (a1, decode_page.cuh:392-506) and the last page's
    // running key max/min, read while the tiles are in flight
    Vec kn, vn, mxo, mno;
    const int entry = last_len - 1, mentry = (N - 1) % P;
    const bool meta_ok = app_mpid >= 0 && app_mpid < a.meta_cap;
    __half* mk = a.meta + ((static_cast<size_t>(app_mpid) * 2 + 0) * P + mentry) * HD + col;
    __half* mv = a.meta + ((static_cast<size_t>(app_mpid) * 2 + 1) * P + mentry) * HD + col;
    if (is_last) {
      kn = *reinterpret_cast<const Vec*>(kn_in + col);
      if (a.rope) {  // rotate the new key; the rotated key also goes back in place
        float kf[CPL];
        vec_to_float<CPL>(kn, kf);
        cs_rope_lane<CPL>(kf, lane, D, rope_pos, a.rope_rcp_scale, a.rope_log2_rcp_theta);
        kn = float_to_vec<CPL>(kf);
        *reinterpret_cast<Vec*>(const_cast<__half*>(kn_in) + col) = kn;
      }
      vn = *reinterpret_cast<const Vec*>(vn_in + col);
      if (entry > 0 && meta_ok) {
        mxo = *reinterpret_cast<const Vec*>(mk);
        mno = *reinterpret_cast<const Vec*>(mv);
      }
    }
    const bool got = mbar_wait_bounded(bar, par, a.err);
    par ^= 1u;
    if (!got) continue;
    uint8_t* Kt = slot;
    uint8_t* Vt = slot + (D / 64) * kCsSubTile;
    if (is_last) {  // the new token is row `entry` of the page
      *reinterpret_cast<Vec*>(Kt + sw_lane_off<D>(entry)) = kn;
      *reinterpret_cast<Vec*>(Vt + sw_lane_off<D>(entry)) = vn;
    }
    for (int r = ntok; r < 16; ++r) {  // rows past the page's tokens: finite zeros
      *reinterpret_cast<Vec*>(Vt + sw_lane_off<D>(r)) = Vec{};
    }
    __syncwarp();
    cs_attend_page_tc<D>(kb, vb, ntok, qb, a.scale_log2, m, l, acc);
    if (is_last) {
      // write the token, the max/min (init -+65504 on a new page) and, when
      // the token fills the page, v_log_norm = log(||mean_t V||_2 + 1e-6)
      *reinterpret_cast<Vec*>(a.kv + (static_cast<size_t>(pid) * 2 * P + entry) * HD + col) = kn;
      *reinterpret_cast<Vec*>(a.kv + ((static_cast<size_t>(pid) * 2 + 1) * P + entry) * HD +
                              col) = vn;
      if (meta_ok) {
        if (entry == 0) {  // a new page: max from -65504, min from +65504
          mxo = vec_fill<CPL>(0xfbfffbffu);
          mno = vec_fill<CPL>(0x7bff7bffu);
        }
        *reinterpret_cast<Vec*>(mk) = vec_hmax<CPL>(mxo, kn);
        *reinterpret_cast<Vec*>(mv) = vec_hmin<CPL>(mno, kn);
      } else if (lane == 0) {
        raise_dev_error(a.err, AOAKV_DEV_ERR_BAD_PAGE);
      }
      if (entry + 1 == P) {
        float sum[CPL];
#pragma unroll
        for (int i = 0; i < CPL; ++i) sum[i] = 0.f;
        for (int t = 0; t < P; ++t) {
          float f[CPL];
          load_row<CPL>(reinterpret_cast<const __half*>(Vt + sw_lane_off<D>(t)), f);
#pragma unroll
          for (int i = 0; i < CPL; ++i) sum[i] += f[i];
        }
        const float inv = 1.f / P;
        float l2 = 0.f;
#pragma unroll
        for (int i = 0; i < CPL; ++i) l2 += (sum[i] * inv) * (sum[i] * inv);
#pragma unroll
        for (int off = 16; off > 0; off >>= 1) l2 += __shfl_xor_sync(0xffffffffu, l2, off);
        if (lane == 0)
          a.vlog[static_cast<size_t>(pid) * H + h] = __float2half_rn(logf(sqrtf(l2) + 1e-6f));
      }
    }
    __syncwarp();  // the slot is consumed before this warp's next load
  }
  // merge the warps of this CTA, then push the CTA's state to CTA 0
  {
    float* mw = mrg + warp * (D + 2);
    if ((lane & 3) == 0) {  // column 0 of the O^T fragments
#pragma unroll
      for (int mm = 0; mm < NK; ++mm) {
        mw[mm * 16 + (lane >> 2)] = acc[mm][0];
        mw[mm * 16 + (lane >> 2) + 8] = acc[mm][2];
      }
    }
    if (lane == 0) {
      mw[D] = m;
      mw[D + 1] = l;
    }
  }
  __syncthreads();
  float* xo0 = cluster.map_shared_rank(xo, 0) + c * (D + 2);
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
    xo0[tid] = O;
    if (tid == 0) {
      xo0[D] = M;
      xo0[D + 1] = Ls;
    }
  }
  __syncthreads();
  if (c != 0) {
    if (tid == 0) {
      asm volatile("fence.acq_rel.cluster;" ::: "memory");
      mbar_arrive_remote(&merge_bar, 0);
    }
  } else {
    if (C > 1) {  // bounded wait for the other CTAs' states
      bool arrived = false;
      for (uint32_t i = 0; i < (1u << 26) && !arrived; ++i) {
        arrived = mbar_try_wait_cluster(&merge_bar, 0u);
        if (!arrived && i > 64) __nanosleep(32);
      }
      if (!arrived && tid == 0) raise_dev_error(a.err, AOAKV_DEV_ERR_TIMEOUT);
    }
    if (tid < D) {
      float MM = -INFINITY;
#pragma unroll
      for (int cc = 0; cc < C; ++cc) MM = fmaxf(MM, xo[cc * (D + 2) + D]);
      float LL = 0.f, OO = 0.f;
      if (MM != -INFINITY) {
#pragma unroll
        for (int cc = 0; cc < C; ++cc) {
          const float f = fast_exp2(xo[cc * (D + 2) + D] - MM);
          LL += f * xo[cc * (D + 2) + D + 1];
          OO += f * xo[cc * (D + 2) + tid];
        }
      }
      if (shard == kShardFinish) {  // this GPU's partial state
        const float ov = LL > 0.f ? OO / LL : 0.f;
        const float lse = LL > 0.f ? (MM + log2f(LL)) * 0.6931471805599453f : -INFINITY;
        const size_t at = static_cast<size_t>(h) * (D + 1);
        if (!a.p2p) {
          a.state_out[at + tid] = ov;
          if (tid == 0) a.state_out[at + D] = lse;
        } else {  // tagged, into every GPU's mailbox, this GPU's row
          const uint32_t epoch =
              __ldcg(reinterpret_cast<const uint32_t*>(a.mail.base[a.rank] + a.mail.ep_off) +
                     1) + 1u;
          for (int g = 0; g < a.world; ++g) {
            uint64_t* so = reinterpret_cast<uint64_t*>(a.mail.base[g] + a.mail.state_off) +
                           static_cast<size_t>(a.rank) * H * (D + 1) + at;
            tagged_store_sys(so + tid, __float_as_uint(ov), epoch);
            if (tid == 0) tagged_store_sys(so + D, __float_as_uint(lse), epoch);
          }
        }
      } else {
        o_out[static_cast<size_t>(h) * D + tid] = __float2half_rn(LL > 0.f ? OO / LL : 0.f);
      }
    }
  }
  cluster_wait_acquire();  // every peer is past its last read of this CTA's memory
  // the rotated q in place, once every CTA of the cluster has read the input
  if (a.rope && c == 0 && tid < D) const_cast<__half*>(q_in)[static_cast<size_t>(h) * D + tid] = q_rot[tid];
}

using KernelFn = void (*)(CUtensorMap, CUtensorMap, ClusterStepArgs, CsShape);

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

int cluster_step_plan(int H, int D, int P, int max_pages, int max_slots, int max_ctas,
                      ClusterPlan* plan, bool slots_beyond_pages) {
  if ((D != 64 && D != 128) || P < 1 || P > kCsMaxPage || H < 1 || H > 65535 || max_pages < 1 ||
      max_slots < 1)
    return 0;
  if (max_slots > max_pages && !slots_beyond_pages) max_slots = max_pages;
  const int ctas = max_ctas > 0 ? max_ctas : num_sms();
  int C = 8;
  while (C > 1 && H * C > ctas) C >>= 1;
  int n_st = (max_pages - 1 + P - 1) / P;
  if (n_st < 1) n_st = 1;
  auto smem_for = [&](int cl) {
    const int ml = (n_st + cl - 1) / cl * P;
    return static_cast<size_t>(cs_layout(D, P, cl, ml, max_slots).total) + 1024;  // + alignment
  };
  size_t smem = smem_for(C);
  while (smem > 200 * 1024 && C < 8) {  // long sequences: more CTAs per head
    C <<= 1;
    smem = smem_for(C);
  }
  if (smem > 200 * 1024) return 0;
  const int max_local = (n_st + C - 1) / C * P;
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
  plan->shape.max_local = max_local;
  plan->shape.max_slots = max_slots;
  plan->smem = fs.smem_set;
  plan->waves = (H + fs.max_clusters - 1) / fs.max_clusters;
  return 1;
}

int launch_cluster_step(const ClusterStepArgs& a, const CUtensorMap& kv_map,
                        const CUtensorMap& meta_map, int D, const ClusterPlan& plan,
                        cudaStream_t s, int num_requests) {
  const int C = plan.cluster;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(C, a.H, num_requests);
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
    const cudaError_t e = cudaLaunchKernelEx(&cfg, fn, kv_map, meta_map, a, plan.shape);
    if (e == cudaSuccess) {
      g_cluster_pdl.store(1);
      return AOAKV_OK;
    }
    if (pdl == 1) AOAKV_CUDA_TRY(e, "cluster step launch");
    (void)cudaGetLastError();
    g_cluster_pdl.store(0);
  }
  cfg.numAttrs = 1;
  AOAKV_CUDA_TRY(cudaLaunchKernelEx(&cfg, fn, kv_map, meta_map, a, plan.shape),
                 "cluster step launch");
  return AOAKV_OK;
}

}  // namespace aoakv
