// a3 page scorer, shared by the stand-alone estimate entry point and the
// per-layer step.
//
// Reference: kernels/aoa_kv/kernels/include/decode/decode_attn.cuh:143-199
// (compute_max_possible: s = sum_i max(q_i*kmax_i, q_i*kmin_i), AOA score
// 2*s*rsqrt(d) + 2*v_log_norm, :193) and :263-443 (the kernel that streams
// the metadata cache, excluding the last page via last_page_len-1, :297-306);
// filtering/filter_util.py:968-1018 and :314-367 state the same quantity.
//
// Design: the metadata of one KV page for all heads is H*D fp16 contiguous
// (max slot) plus the same at +P*H*D (min slot), so a flat sweep over
// (page, head) rows reads HBM strictly sequentially. D/8 lanes own one row
// with one 16-byte streaming load per slot; U rows per thread are loaded
// before any arithmetic so every SM keeps ~100 KB in flight; a lane-group
// xor-shuffle finishes each dot product. Scores are fp32 internally.
#pragma once

#include "common.cuh"

namespace aoakv {

struct EstimateArgs {
  const __half* q;            // [H, D]
  const __half* meta;         // [meta_cap, 2, P, H, D]
  const int32_t* meta_indices;
  const int32_t* kv_indices;  // physical KV page of logical page p (AOA mode)
  const __half* vlog;         // [kv_cap, H]
  void* out;                  // out[h * out_stride + p]
  int64_t out_stride;
  int out_f32;
  int n_score;                // pages scored: N - 1
  int H, P;
  int meta_cap, kv_cap;
  int mode;                   // AOAKV_SCORE_*
  float two_rsqrt_d;
  int* err;
};

constexpr int kEstThreads = 256;
constexpr int kEstUnroll = 4;

// Rows row0, row0 + row_step, ... (each a sweep of U * THREADS/L rows) of the
// flattened (page, head) space; THREADS = blockDim.x.
template <int D, int THREADS>
__device__ __forceinline__ void estimate_rows_t(const EstimateArgs& a,
                                                const float* q_s, int row0,
                                                int row_step, int n_rows) {
  constexpr int L = D / 8;
  constexpr int RPS = THREADS / L;  // rows per sweep of the CTA
  const int lane = threadIdx.x % L;
  const int sub = threadIdx.x / L;
  const size_t HD = static_cast<size_t>(a.H) * D;
  const size_t slot = static_cast<size_t>(a.P) * HD;  // max slot -> min slot
  for (int base = row0; base < n_rows; base += row_step) {
    uint4 mx[kEstUnroll], mn[kEstUnroll];
    int hh[kEstUnroll], pp[kEstUnroll];
    bool ok[kEstUnroll];
#pragma unroll
    for (int u = 0; u < kEstUnroll; ++u) {
      const int r = base + u * RPS + sub;
      ok[u] = r < n_rows;
      const int p = ok[u] ? r / a.H : 0;
      const int h = ok[u] ? r - p * a.H : 0;
      pp[u] = p;
      hh[u] = h;
      int mpid = ok[u] ? __ldg(a.meta_indices + p / a.P) : 0;
      if (ok[u] && (mpid < 0 || mpid >= a.meta_cap)) {
        raise_dev_error(a.err, AOAKV_DEV_ERR_BAD_PAGE);
        ok[u] = false;
      }
      if (ok[u]) {
        const __half* row = a.meta + (static_cast<size_t>(mpid) * 2 * a.P + p % a.P) * HD +
                            static_cast<size_t>(h) * D + lane * 8;
        mx[u] = ld_stream_u4(row);
        mn[u] = ld_stream_u4(row + slot);
      } else {
        mx[u] = make_uint4(0, 0, 0, 0);
        mn[u] = make_uint4(0, 0, 0, 0);
      }
    }
#pragma unroll
    for (int u = 0; u < kEstUnroll; ++u) {
      float fa[8], fb[8];
      u4_to_f8(mx[u], fa);
      u4_to_f8(mn[u], fb);
      const float4 q0 = *reinterpret_cast<const float4*>(q_s + hh[u] * D + lane * 8);
      const float4 q1 = *reinterpret_cast<const float4*>(q_s + hh[u] * D + lane * 8 + 4);
      const float qv[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
      float s = 0.f;
#pragma unroll
      for (int i = 0; i < 8; ++i) s += fmaxf(qv[i] * fa[i], qv[i] * fb[i]);
#pragma unroll
      for (int off = L / 2; off > 0; off >>= 1) s += __shfl_xor_sync(0xffffffffu, s, off);
      if (ok[u] && lane == 0) {
        float score = s;
        if (a.mode == AOAKV_SCORE_AOAKV) {
          const int pid = a.kv_indices ? __ldg(a.kv_indices + pp[u]) : pp[u];
          float vl = 0.f;
          if (pid < 0 || pid >= a.kv_cap)
            raise_dev_error(a.err, AOAKV_DEV_ERR_BAD_PAGE);
          else
            vl = __half2float(a.vlog[static_cast<size_t>(pid) * a.H + hh[u]]);
          score = a.two_rsqrt_d * s + 2.f * vl;
        }
        const size_t o = static_cast<size_t>(hh[u]) * a.out_stride + pp[u];
        if (a.out_f32)
          static_cast<float*>(a.out)[o] = score;
        else
          static_cast<__half*>(a.out)[o] = __float2half_rn(score);
      }
    }
  }
}

template <int D>
__device__ __forceinline__ void estimate_rows(const EstimateArgs& a, const float* q_s,
                                              int row0, int row_step, int n_rows) {
  estimate_rows_t<D, kEstThreads>(a, q_s, row0, row_step, n_rows);
}

// Head-stationary sweep over the pages [p_begin, p_end), used when
// blockDim.x == H * D/8: thread t keeps head t/(D/8), channels
// 8*(t % (D/8)) .. +8, so q stays in registers. Because max(q*kmax, q*kmin)
// == q * (q > 0 ? kmax : kmin) whenever kmax >= kmin (which the append
// maintains), each channel costs one bit-select of the fp16 operand, one
// conversion and one FMA; the page's metadata rows, its v_log_norm and the
// page-table entries are all loaded before any arithmetic.
template <int D, int U>
__device__ __forceinline__ void estimate_pages_hs(const EstimateArgs& a, int p_begin,
                                                  int p_end) {
  constexpr int L = D / 8;
  const int h = threadIdx.x / L, lane = threadIdx.x % L;
  float qv[8];
  uint32_t msk[4];
  u4_to_f8(__ldg(reinterpret_cast<const uint4*>(a.q + static_cast<size_t>(h) * D + lane * 8)),
           qv);
#pragma unroll
  for (int i = 0; i < 4; ++i)
    msk[i] = (qv[2 * i] > 0.f ? 0x0000ffffu : 0u) | (qv[2 * i + 1] > 0.f ? 0xffff0000u : 0u);
  const bool aoa = a.mode == AOAKV_SCORE_AOAKV;
  const size_t HD = static_cast<size_t>(a.H) * D;
  const size_t slot = static_cast<size_t>(a.P) * HD;
  const size_t col = static_cast<size_t>(h) * D + lane * 8;
  for (int p0 = p_begin; p0 < p_end; p0 += U) {
    uint4 mx[U], mn[U];
    float vl[U];
    bool ok[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int p = p0 + u;
      ok[u] = p < p_end;
      int mpid = 0, pid = 0;
      if (ok[u]) {
        mpid = __ldg(a.meta_indices + p / a.P);
        pid = !aoa ? 0 : (a.kv_indices ? __ldg(a.kv_indices + p) : p);
        if (mpid < 0 || mpid >= a.meta_cap || pid < 0 || (aoa && pid >= a.kv_cap)) {
          raise_dev_error(a.err, AOAKV_DEV_ERR_BAD_PAGE);
          ok[u] = false;
        }
      }
      mx[u] = make_uint4(0, 0, 0, 0);
      mn[u] = make_uint4(0, 0, 0, 0);
      vl[u] = 0.f;
      if (ok[u]) {
        const __half* row = a.meta + (static_cast<size_t>(mpid) * 2 * a.P + p % a.P) * HD + col;
        mx[u] = ld_stream_u4(row);
        mn[u] = ld_stream_u4(row + slot);
        if (aoa) vl[u] = __half2float(a.vlog[static_cast<size_t>(pid) * a.H + h]);
      }
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      uint4 sel;
      sel.x = (mx[u].x & msk[0]) | (mn[u].x & ~msk[0]);
      sel.y = (mx[u].y & msk[1]) | (mn[u].y & ~msk[1]);
      sel.z = (mx[u].z & msk[2]) | (mn[u].z & ~msk[2]);
      sel.w = (mx[u].w & msk[3]) | (mn[u].w & ~msk[3]);
      float f[8];
      u4_to_f8(sel, f);
      float s0 = qv[0] * f[0], s1 = qv[1] * f[1];
#pragma unroll
      for (int i = 2; i < 8; i += 2) {
        s0 = fmaf(qv[i], f[i], s0);
        s1 = fmaf(qv[i + 1], f[i + 1], s1);
      }
      float s = s0 + s1;
#pragma unroll
      for (int off = L / 2; off > 0; off >>= 1) s += __shfl_xor_sync(0xffffffffu, s, off);
      if (ok[u] && lane == 0) {
        const float score = aoa ? a.two_rsqrt_d * s + 2.f * vl[u] : s;
        const size_t o = static_cast<size_t>(h) * a.out_stride + (p0 + u);
        if (a.out_f32)
          static_cast<float*>(a.out)[o] = score;
        else
          static_cast<__half*>(a.out)[o] = __float2half_rn(score);
      }
    }
  }
}

// ---------------------------------------------------------------------------
// Bulk-copy pipelined page scorer (blockDim.x == H * D/8, H % 8 == 0): the
// metadata of one page for all heads — its max block and min block, H*D fp16
// each, contiguous — and its v_log_norm row land in a shared-memory stage by
// three 1-D bulk copies issued by one thread; kEstStages stages keep the
// CTA's next pages in flight while the current one is scored, so HBM sees
// large contiguous reads with no register cost. The page-table entries of
// the CTA's whole range are fetched first in one round trip.
constexpr int kEstStages = 4;
constexpr int kEstMaxRange = 64;  // pages per CTA for this path

__host__ __device__ constexpr int est_stage_bytes(int H, int D) {
  return (2 * H * D * 2 + H * 2 + 127) / 128 * 128;
}

// ids_s: shared int[2 * kEstMaxRange]; bars: kEstStages mbarriers initialised
// to count 1 whose phases are tracked in *phase_bits (bit s = next parity).
template <int D>
__device__ __forceinline__ void estimate_pages_tma(const EstimateArgs& a, int p_begin, int p_end,
                                                   uint8_t* stages, uint64_t* bars, int* ids_s,
                                                   uint32_t* phase_bits) {
  constexpr int L = D / 8;
  const int h = threadIdx.x / L, lane = threadIdx.x % L;
  const int R = p_end - p_begin;
  const bool aoa = a.mode == AOAKV_SCORE_AOAKV;
  const int H = a.H;
  const size_t HD = static_cast<size_t>(H) * D;
  const int sb = est_stage_bytes(H, D);
  float qv[8];
  uint32_t msk[4];
  u4_to_f8(__ldg(reinterpret_cast<const uint4*>(a.q + static_cast<size_t>(h) * D + lane * 8)),
           qv);
#pragma unroll
  for (int i = 0; i < 4; ++i)
    msk[i] = (qv[2 * i] > 0.f ? 0x0000ffffu : 0u) | (qv[2 * i + 1] > 0.f ? 0xffff0000u : 0u);
  for (int t = threadIdx.x; t < R; t += blockDim.x) {
    const int p = p_begin + t;
    int mp = __ldg(a.meta_indices + p / a.P);
    const int pid = aoa ? (a.kv_indices ? __ldg(a.kv_indices + p) : p) : 0;
    if (mp < 0 || mp >= a.meta_cap || pid < 0 || (aoa && pid >= a.kv_cap)) {
      raise_dev_error(a.err, AOAKV_DEV_ERR_BAD_PAGE);
      mp = -1;
    }
    ids_s[2 * t] = mp;
    ids_s[2 * t + 1] = pid;
  }
  __syncthreads();
  auto issue = [&](int j) {  // thread 0 only
    const int s = j % kEstStages;
    const int mp = ids_s[2 * j], pid = ids_s[2 * j + 1];
    if (mp < 0) {
      mbar_arrive(&bars[s]);  // complete the phase; the page is skipped
      return;
    }
    uint8_t* st = stages + s * sb;
    const int p = p_begin + j;
    const uint32_t blk = static_cast<uint32_t>(HD * 2);
    mbar_arrive_expect_tx(&bars[s], 2 * blk + (aoa ? static_cast<uint32_t>(H * 2) : 0u));
    const __half* row = a.meta + (static_cast<size_t>(mp) * 2 * a.P + p % a.P) * HD;
    bulk_g2s(st, row, blk, &bars[s]);
    bulk_g2s(st + blk, row + static_cast<size_t>(a.P) * HD, blk, &bars[s]);
    if (aoa) bulk_g2s(st + 2 * blk, a.vlog + static_cast<size_t>(pid) * H, H * 2, &bars[s]);
  };
  if (threadIdx.x == 0) {
    fence_proxy_async_smem();
    for (int j = 0; j < R && j < kEstStages; ++j) issue(j);
  }
  // The issuing thread must rejoin its warp before anyone polls the
  // barriers: without this block barrier its head's scores came out wrong
  // inside the fused step kernel.
  __syncthreads();
  for (int j = 0; j < R; ++j) {
    const int s = j % kEstStages;
    const bool arrived = mbar_wait_bounded(&bars[s], (*phase_bits >> s) & 1u, a.err);
    *phase_bits ^= 1u << s;
    const uint8_t* st = stages + s * sb;
    const bool ok = arrived && ids_s[2 * j] >= 0;
    const size_t off = (static_cast<size_t>(h) * D + lane * 8) * 2;
    const uint4 mx = *reinterpret_cast<const uint4*>(st + off);
    const uint4 mn = *reinterpret_cast<const uint4*>(st + HD * 2 + off);
    const float vl = aoa ? __half2float(reinterpret_cast<const __half*>(st + HD * 4)[h]) : 0.f;
    uint4 sel;
    sel.x = (mx.x & msk[0]) | (mn.x & ~msk[0]);
    sel.y = (mx.y & msk[1]) | (mn.y & ~msk[1]);
    sel.z = (mx.z & msk[2]) | (mn.z & ~msk[2]);
    sel.w = (mx.w & msk[3]) | (mn.w & ~msk[3]);
    float f[8];
    u4_to_f8(sel, f);
    float s0 = qv[0] * f[0], s1 = qv[1] * f[1];
#pragma unroll
    for (int i = 2; i < 8; i += 2) {
      s0 = fmaf(qv[i], f[i], s0);
      s1 = fmaf(qv[i + 1], f[i + 1], s1);
    }
    float sc = s0 + s1;
#pragma unroll
    for (int off2 = L / 2; off2 > 0; off2 >>= 1) sc += __shfl_xor_sync(0xffffffffu, sc, off2);
    if (ok && lane == 0) {
      const float score = aoa ? a.two_rsqrt_d * sc + 2.f * vl : sc;
      const size_t o = static_cast<size_t>(h) * a.out_stride + (p_begin + j);
      if (a.out_f32)
        static_cast<float*>(a.out)[o] = score;
      else
        static_cast<__half*>(a.out)[o] = __float2half_rn(score);
    }
    __syncthreads();  // stage s is free again
    if (threadIdx.x == 0 && j + kEstStages < R) {
      fence_proxy_async_smem();
      issue(j + kEstStages);
    }
    __syncwarp();  // the issuing thread rejoins warp 0 before its next wait
  }
}

// Tensor-map variant of estimate_pages_tma: the max and min blocks of a
// page are two 3-D TMA boxes {D, H, 1} of `mmap` (the metadata viewed as
// [rows = meta_page*2*P + slot*P + entry][H][D]); v_log_norm values are
// plain loads issued before the wait. Same results, same stage layout.
// `overlap()` runs on every thread after the first boxes are issued and
// before the first wait (the fused step appends the new token there).
struct NoOverlap {
  __device__ void operator()() const {}
};

template <int D, typename Overlap = NoOverlap>
__device__ __forceinline__ void estimate_pages_tmap(const EstimateArgs& a, const CUtensorMap* mmap,
                                                    int p_begin, int p_end, uint8_t* stages,
                                                    uint64_t* bars, int* ids_s,
                                                    uint32_t* phase_bits,
                                                    Overlap overlap = Overlap()) {
  constexpr int L = D / 8;
  const int h = threadIdx.x / L, lane = threadIdx.x % L;
  const int R = p_end - p_begin;
  const bool aoa = a.mode == AOAKV_SCORE_AOAKV;
  const int H = a.H;
  const size_t HD = static_cast<size_t>(H) * D;
  const int sb = est_stage_bytes(H, D);
  for (int t = threadIdx.x; t < R; t += blockDim.x) {
    const int p = p_begin + t;
    int mp = __ldg(a.meta_indices + p / a.P);
    const int pid = aoa ? (a.kv_indices ? __ldg(a.kv_indices + p) : p) : 0;
    if (mp < 0 || mp >= a.meta_cap || pid < 0 || (aoa && pid >= a.kv_cap)) {
      raise_dev_error(a.err, AOAKV_DEV_ERR_BAD_PAGE);
      mp = -1;
    }
    ids_s[2 * t] = mp;
    ids_s[2 * t + 1] = pid;
  }
  __syncthreads();
  const uint32_t blk = static_cast<uint32_t>(HD * 2);
  if (threadIdx.x == 0) {
    fence_proxy_async();
    for (int j = 0; j < R && j < kEstStages; ++j) {
      const int mp = ids_s[2 * j];
      if (mp < 0) {
        mbar_arrive(&bars[j]);
        continue;
      }
      const int row = (mp * 2) * a.P + (p_begin + j) % a.P;
      mbar_arrive_expect_tx(&bars[j], 2 * blk);
      tma_load_3d(stages + j * sb, mmap, 0, 0, row, &bars[j]);
      tma_load_3d(stages + j * sb + blk, mmap, 0, 0, row + a.P, &bars[j]);
    }
  }
  overlap();
  __syncthreads();  // the issuing thread rejoins its warp before the waits
  float qv[8];
  uint32_t msk[4];
  u4_to_f8(__ldg(reinterpret_cast<const uint4*>(a.q + static_cast<size_t>(h) * D + lane * 8)),
           qv);
#pragma unroll
  for (int i = 0; i < 4; ++i)
    msk[i] = (qv[2 * i] > 0.f ? 0x0000ffffu : 0u) | (qv[2 * i + 1] > 0.f ? 0xffff0000u : 0u);
  for (int j = 0; j < R; ++j) {
    const int s = j % kEstStages;
    const int pid = ids_s[2 * j + 1];
    const float vl =
        (aoa && ids_s[2 * j] >= 0) ? __half2float(a.vlog[static_cast<size_t>(pid) * H + h]) : 0.f;
    const bool arrived = mbar_wait_bounded(&bars[s], (*phase_bits >> s) & 1u, a.err);
    *phase_bits ^= 1u << s;
    const uint8_t* st = stages + s * sb;
    const bool ok = arrived && ids_s[2 * j] >= 0;
    const size_t off = (static_cast<size_t>(h) * D + lane * 8) * 2;
    const uint4 mx = *reinterpret_cast<const uint4*>(st + off);
    const uint4 mn = *reinterpret_cast<const uint4*>(st + blk + off);
    uint4 sel;
    sel.x = (mx.x & msk[0]) | (mn.x & ~msk[0]);
    sel.y = (mx.y & msk[1]) | (mn.y & ~msk[1]);
    sel.z = (mx.z & msk[2]) | (mn.z & ~msk[2]);
    sel.w = (mx.w & msk[3]) | (mn.w & ~msk[3]);
    float f[8];
    u4_to_f8(sel, f);
    float s0 = qv[0] * f[0], s1 = qv[1] * f[1];
#pragma unroll
    for (int i = 2; i < 8; i += 2) {
      s0 = fmaf(qv[i], f[i], s0);
      s1 = fmaf(qv[i + 1], f[i + 1], s1);
    }
    float sc = s0 + s1;
#pragma unroll
    for (int off2 = L / 2; off2 > 0; off2 >>= 1) sc += __shfl_xor_sync(0xffffffffu, sc, off2);
    if (ok && lane == 0) {
      const float score = aoa ? a.two_rsqrt_d * sc + 2.f * vl : sc;
      const size_t o = static_cast<size_t>(h) * a.out_stride + (p_begin + j);
      if (a.out_f32)
        static_cast<float*>(a.out)[o] = score;
      else
        static_cast<__half*>(a.out)[o] = __float2half_rn(score);
    }
    __syncthreads();  // stage s is free again
    const int jn = j + kEstStages;
    if (threadIdx.x == 0 && jn < R) {
      fence_proxy_async();
      const int mp = ids_s[2 * jn];
      if (mp < 0) {
        mbar_arrive(&bars[s]);
      } else {
        const int row = (mp * 2) * a.P + (p_begin + jn) % a.P;
        mbar_arrive_expect_tx(&bars[s], 2 * blk);
        tma_load_3d(stages + s * sb, mmap, 0, 0, row, &bars[s]);
        tma_load_3d(stages + s * sb + blk, mmap, 0, 0, row + a.P, &bars[s]);
      }
    }
    __syncwarp();
  }
}

// Contiguous page range [*b, *e) of CTA `cta` out of `ctas` over n pages.
__device__ __forceinline__ void page_range(int n, int cta, int ctas, int* b, int* e) {
  const int per = (n + ctas - 1) / ctas;
  *b = min(n, cta * per);
  *e = min(n, *b + per);
}

// Stages q (fp16 [H, D]) into shared memory as fp32, 16 bytes per load so a
// CTA needs one or two round trips to L2 however many heads there are.
template <int D>
__device__ __forceinline__ void stage_q(const __half* q, float* q_s, int H) {
  const int n8 = H * D / 8;
  for (int i = threadIdx.x; i < n8; i += blockDim.x) {
    float f[8];
    u4_to_f8(__ldg(reinterpret_cast<const uint4*>(q) + i), f);
    float4* dst = reinterpret_cast<float4*>(q_s + i * 8);
    dst[0] = make_float4(f[0], f[1], f[2], f[3]);
    dst[1] = make_float4(f[4], f[5], f[6], f[7]);
  }
}

}  // namespace aoakv
