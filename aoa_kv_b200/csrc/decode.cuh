// a5 split-KV sparse paged decode: one work unit = (head, chunk of page
// slots). Shared by the stand-alone decode entry point and the per-layer step.
//
// Reference: kernels/aoa_kv/kernels/include/decode/decode_attn.cuh:469-688
// (per-head gather of indices[h*page_budget + i] plus the shared last page,
// decode_page.cuh:325-351; online softmax in the log2 domain with
// sm_scale*log2e, :493, :77-120) and :937-1047 (split into chunks, then
// FlashInfer's VariableLengthMergeStates, whose math is the standard
// log-sum-exp combine of partial (m, l, o) states, restated here).
//
// Design: thread 0 issues one 3-D TMA box per K and V page tile (box
// {D, 1, P} over the view [rows = page*2*P + kv*P + entry][H][D]), every tile
// of the chunk up front, each completing on its own mbarrier. A warp owns one
// 8-token group of one page slot; lane l owns channels [l*D/32, (l+1)*D/32).
// The eight dot products finish with a 9-shuffle reduce-scatter (lane l ends
// with token (l >> 2) & 7), then one online-softmax update. Partial states
// merge across warps in shared memory and across chunks through a workspace;
// the last CTA of a head (atomic ticket) writes the output and re-arms the
// ticket, so no second launch and no host work is needed.
#pragma once

#include "common.cuh"

namespace aoakv {

constexpr int kDecThreads = 128;
constexpr int kDecWarps = kDecThreads / 32;
constexpr int kDecMaxChunk = 8;
constexpr int kDecHeader = 128;  // 8 mbarriers (64 B) + 8 token counts (32 B) + flag

struct DecodeArgs {
  const __half* q;             // [H, D]
  __half* o;                   // [H, D]
  const int32_t* indices;      // indices[h * idx_stride + slot], slot < n_sel
  int64_t idx_stride;
  int n_sel;                   // selected pages per head (excl. last page)
  int last_page, last_len;     // always-attended last page
  const int32_t* last_page_ptr;  // if set, the last page id is read from here
  int H, P, kv_cap;
  int chunk_pages, n_chunks;   // slots per unit, units per head
  float scale_log2;            // sm_scale * log2(e)
  float* ws_o;                 // [H, n_chunks, D] partial numerators
  float2* ws_ml;               // [H, n_chunks] partial (max, denominator)
  int* ws_cnt;                 // [H] arrival tickets, zero between calls
  int* err;
  float* o_f32;                // if set: fp32 output [H, D] instead of o
  float* lse;                  // if set: natural-log sum of exp of the scores [H]
  int group;                   // > 1: query head h reads KV head h / group (GQA):
                               // its page ids from row h / group, its K/V
                               // tiles from that head; q, o per query head
};

__host__ __device__ constexpr int dec_merge_bytes(int D, int nw = kDecWarps) {
  return nw * (D + 2) * 4;
}
__host__ __device__ constexpr int dec_tile_offset(int D, int nw = kDecWarps) {
  return (kDecHeader + dec_merge_bytes(D, nw) + 127) / 128 * 128;
}
__host__ __device__ constexpr size_t dec_smem_bytes(int D, int P, int chunk,
                                                   int nw = kDecWarps) {
  return static_cast<size_t>(dec_tile_offset(D, nw)) +
         static_cast<size_t>(chunk) * 2 * P * D * 2;
}

__device__ __forceinline__ float fast_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

template <int CPL>
__device__ __forceinline__ void load_row(const __half* p, float f[CPL]) {
  if constexpr (CPL == 4) {
    const uint2 u = *reinterpret_cast<const uint2*>(p);
    const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&u.x));
    const float2 b = __half22float2(*reinterpret_cast<const __half2*>(&u.y));
    f[0] = a.x; f[1] = a.y; f[2] = b.x; f[3] = b.y;
  } else {
    const float2 a = __half22float2(*reinterpret_cast<const __half2*>(p));
    f[0] = a.x; f[1] = a.y;
  }
}


// Issues the TMA loads of unit (h, c). Thread 0 only. Slot token counts land
// in tok[] (0 = skipped slot: bad page id or none). Selected page ids come
// from a.indices, or from the shared window win[slot - win_lo] when given.
__device__ __forceinline__ void decode_issue(const DecodeArgs& a,
                                             const CUtensorMap* tmap, int h,
                                             int c, uint64_t* bars, int* tok,
                                             __half* tiles, int D,
                                             const int* win = nullptr, int win_lo = 0) {
  if (a.group > 1) h /= a.group;  // the KV head this query head reads
  const int n_slots = a.n_sel + 1;
  const int s0 = c * a.chunk_pages;
  const int ns = min(n_slots, s0 + a.chunk_pages) - s0;
  const int tile = a.P * D;
  fence_proxy_async();  // prior generic smem/global accesses before async-proxy ones
  int pids[kDecMaxChunk];
#pragma unroll
  for (int j = 0; j < kDecMaxChunk; ++j) {  // all page ids first: one round trip
    const int slot = s0 + j;
    pids[j] = 0;
    if (j < ns) {
      if (slot < a.n_sel)
        pids[j] = win ? win[slot - win_lo]
                      : __ldcg(a.indices + static_cast<size_t>(h) * a.idx_stride + slot);
      else
        pids[j] = a.last_page_ptr ? __ldcg(a.last_page_ptr) : a.last_page;
    }
  }
#pragma unroll
  for (int j = 0; j < kDecMaxChunk; ++j) {
    if (j >= ns) break;
    const int slot = s0 + j;
    const int pid = pids[j];
    int nt = slot < a.n_sel ? a.P : a.last_len;
    if (pid == -1) {
      nt = 0;  // "no page here" (a shard that does not own this selected page)
    } else if (pid < 0 || pid >= a.kv_cap) {
      raise_dev_error(a.err, AOAKV_DEV_ERR_BAD_PAGE);
      nt = 0;
    }
    tok[j] = nt;
    if (nt > 0) {
      mbar_arrive_expect_tx(&bars[j], static_cast<uint32_t>(2 * tile * 2));
      tma_load_3d(tiles + (2 * j) * tile, tmap, 0, h, (pid * 2 + 0) * a.P, &bars[j]);
      tma_load_3d(tiles + (2 * j + 1) * tile, tmap, 0, h, (pid * 2 + 1) * a.P, &bars[j]);
    }
  }
}

// Final output of head h, channel d from the merged state (numerator O,
// denominator L, running max M in log2 units): o = O / L (fp16, or fp32 when
// a.o_f32 is set) and, if requested, lse = ln(sum exp(s)) = (M + log2 L) ln 2.
// A head with no tokens (L == 0) gets o = 0 and lse = -inf.
__device__ __forceinline__ void decode_write_out(const DecodeArgs& a, int h, int d, int D,
                                                 float O, float L, float M) {
  const float v = L > 0.f ? O / L : 0.f;
  const size_t i = static_cast<size_t>(h) * D + d;
  if (a.o_f32)
    a.o_f32[i] = v;
  else
    a.o[i] = __float2half_rn(v);
  if (a.lse && d == 0) a.lse[h] = L > 0.f ? (M + log2f(L)) * 0.6931471805599453f : -INFINITY;
}

// Online-softmax update of one warp's (m, l, o) with tokens [t0, t0+8) of
// the page tile K/V that hold nt valid tokens (rows >= nt are ignored).
template <int D>
__device__ __forceinline__ void attend8(const __half* K, const __half* V, int t0, int nt,
                                        int P, const float* qv, float& m, float& l,
                                        float* o) {
  constexpr int CPL = D / 32;
  const int lane = threadIdx.x & 31;
  float part[8];
#pragma unroll
  for (int u = 0; u < 8; ++u) {
    part[u] = 0.f;
    if (t0 + u < P) {
      float kf[CPL];
      load_row<CPL>(K + (t0 + u) * D + lane * CPL, kf);
#pragma unroll
      for (int i = 0; i < CPL; ++i) part[u] = fmaf(qv[i], kf[i], part[u]);
    }
  }
  // reduce-scatter 8 sums over 32 lanes: lane keeps token (lane>>2)&7
  const bool b4 = lane & 16, b3 = lane & 8, b2 = lane & 4;
  float r4[4], r2[2], r1;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float send = b4 ? part[i] : part[4 + i];
    const float keep = b4 ? part[4 + i] : part[i];
    r4[i] = keep + __shfl_xor_sync(0xffffffffu, send, 16);
  }
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    const float send = b3 ? r4[i] : r4[2 + i];
    const float keep = b3 ? r4[2 + i] : r4[i];
    r2[i] = keep + __shfl_xor_sync(0xffffffffu, send, 8);
  }
  {
    const float send = b2 ? r2[0] : r2[1];
    const float keep = b2 ? r2[1] : r2[0];
    r1 = keep + __shfl_xor_sync(0xffffffffu, send, 4);
  }
  r1 += __shfl_xor_sync(0xffffffffu, r1, 2);
  r1 += __shfl_xor_sync(0xffffffffu, r1, 1);
  const bool valid = t0 + ((lane >> 2) & 7) < nt;
  const float sv = valid ? r1 : -INFINITY;
  float gmax = fmaxf(sv, __shfl_xor_sync(0xffffffffu, sv, 4));
  gmax = fmaxf(gmax, __shfl_xor_sync(0xffffffffu, gmax, 8));
  gmax = fmaxf(gmax, __shfl_xor_sync(0xffffffffu, gmax, 16));
  const float m_new = fmaxf(m, gmax);  // finite: token t0 is valid
  const float alpha = fast_exp2(m - m_new);
  const float p = valid ? fast_exp2(sv - m_new) : 0.f;
  float ps = p + __shfl_xor_sync(0xffffffffu, p, 4);
  ps += __shfl_xor_sync(0xffffffffu, ps, 8);
  ps += __shfl_xor_sync(0xffffffffu, ps, 16);
  l = l * alpha + ps;
#pragma unroll
  for (int i = 0; i < CPL; ++i) o[i] *= alpha;
#pragma unroll
  for (int u = 0; u < 8; ++u) {
    const float pu = __shfl_sync(0xffffffffu, p, u * 4);
    if (t0 + u < nt) {  // never touch rows past the valid tokens (may be NaN)
      float vf[CPL];
      load_row<CPL>(V + (t0 + u) * D + lane * CPL, vf);
#pragma unroll
      for (int i = 0; i < CPL; ++i) o[i] = fmaf(pu, vf[i], o[i]);
    }
  }
  m = m_new;
}

// Computes unit (h, c) after decode_issue and a __syncthreads(), with NW
// warps (blockDim.x == 32 * NW). Work items are (slot, 8-token group) pairs.
// Barrier j completes the phase (phase_bits >> j) & 1. Writes the final
// output (single chunk) or a partial state and merges when last; the
// finishing CTA also zeroes *rearm (if given) for the next call.
template <int D, int NW>
__device__ __forceinline__ void decode_compute_multi(const DecodeArgs& a, int h, int c,
                                                     uint64_t* bars, const int* tok,
                                                     const __half* tiles, float* mrg,
                                                     int* flag_s, uint32_t phase_bits,
                                                     uint32_t* rearm) {
  constexpr int CPL = D / 32;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n_slots = a.n_sel + 1;
  const int s0 = c * a.chunk_pages;
  const int ns = min(n_slots, s0 + a.chunk_pages) - s0;
  const int tile = a.P * D;
  const int groups = (a.P + 7) / 8;

  float qv[CPL];
  load_row<CPL>(a.q + static_cast<size_t>(h) * D + lane * CPL, qv);
#pragma unroll
  for (int i = 0; i < CPL; ++i) qv[i] *= a.scale_log2;

  float m = -INFINITY, l = 0.f, o[CPL];
#pragma unroll
  for (int i = 0; i < CPL; ++i) o[i] = 0.f;

  for (int it = warp; it < ns * groups; it += NW) {
    const int j = it / groups, t0 = (it % groups) * 8;
    const int nt = tok[j];
    if (t0 >= nt) continue;
    if (!mbar_wait_bounded(&bars[j], (phase_bits >> j) & 1u, a.err)) continue;
    const __half* K = tiles + (2 * j) * tile;
    attend8<D>(K, K + tile, t0, nt, a.P, qv, m, l, o);
  }

  // ---- merge the warps of this CTA
  float* mw = mrg + warp * (D + 2);
#pragma unroll
  for (int i = 0; i < CPL; ++i) mw[lane * CPL + i] = o[i];
  if (lane == 0) {
    mw[D] = m;
    mw[D + 1] = l;
  }
  __syncthreads();
  float M = -INFINITY, Ls = 0.f, O = 0.f;
  const int d = threadIdx.x;
  if (d < D) {
#pragma unroll
    for (int w = 0; w < NW; ++w) M = fmaxf(M, mrg[w * (D + 2) + D]);
    if (M != -INFINITY) {
#pragma unroll
      for (int w = 0; w < NW; ++w) {
        const float sc = fast_exp2(mrg[w * (D + 2) + D] - M);
        Ls += sc * mrg[w * (D + 2) + D + 1];
        O += sc * mrg[w * (D + 2) + d];
      }
    }
  }
  if (a.n_chunks == 1) {
    if (d < D) decode_write_out(a, h, d, D, O, Ls, M);
    if (rearm && threadIdx.x == 0) *rearm = 0u;
    __syncthreads();
    return;
  }
  const size_t u = static_cast<size_t>(h) * a.n_chunks + c;
  if (d < D) a.ws_o[u * D + d] = O;
  if (d == 0) a.ws_ml[u] = make_float2(M, Ls);
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0)
    *flag_s = (atomicAdd(a.ws_cnt + h, 1) == a.n_chunks - 1);
  __syncthreads();
  if (*flag_s) {
    __threadfence();
    if (d < D) {
      const float2* ml = a.ws_ml + static_cast<size_t>(h) * a.n_chunks;
      const float* po = a.ws_o + static_cast<size_t>(h) * a.n_chunks * D;
      float MM = -INFINITY;
      for (int k = 0; k < a.n_chunks; ++k) MM = fmaxf(MM, __ldcg(&ml[k].x));
      float LL = 0.f, OO = 0.f;
      if (MM != -INFINITY) {
        for (int k = 0; k < a.n_chunks; ++k) {
          const float2 mlk = __ldcg(&ml[k]);
          const float sc = fast_exp2(mlk.x - MM);
          LL += sc * mlk.y;
          OO += sc * __ldcg(po + static_cast<size_t>(k) * D + d);
        }
      }
      decode_write_out(a, h, d, D, OO, LL, MM);
    }
    if (threadIdx.x == 0) {
      a.ws_cnt[h] = 0;
      if (rearm) *rearm = 0u;
    }
  }
  __syncthreads();
}

// The stand-alone decode: one unit per CTA of kDecWarps warps, phase 0.
template <int D>
__device__ __forceinline__ void decode_compute(const DecodeArgs& a, int h, int c,
                                               uint64_t* bars, const int* tok,
                                               const __half* tiles, float* mrg,
                                               int* flag_s, uint32_t parity) {
  decode_compute_multi<D, kDecWarps>(a, h, c, bars, tok, tiles, mrg, flag_s,
                                     parity ? 0xffffffffu : 0u, nullptr);
}

}  // namespace aoakv
