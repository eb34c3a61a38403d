// Pipelined fused per-layer step: ONE cooperative launch, two CTA roles on
// every SM, so page selection and sparse decode of the first heads overlap
// the scoring of the last ones.
//
//   scorers   CTAs [0, G/2): CTA e < H first appends head e of the new token
//             (a1, step_append.cuh). Then, for head groups g = 0, 1, ... of
//             8 heads in turn, it scores its contiguous page range for the
//             group's heads (a3, decode_attn.cuh:143-199, :263-443): each
//             page's key max/min rows of the 8 heads are two TMA boxes
//             {D, 8, 1} streamed through a 6-stage shared-memory ring that
//             runs on across groups; fp32 scores go to the workspace and the
//             CTA arrives on est_done[g] after the group.
//   units     every CTA (the other half from the start, scorers once their
//             scoring is done) claims units (head, chunk of selected page
//             slots) in head order from one counter. A unit waits (bounded)
//             for est_done[g] of its head's group, selects the head's pages
//             (a4 with decode_select_k.cuh:25-61 semantics: topk_hist.cuh,
//             bitonic / radix when many scores tie), keeps its chunk's page
//             ids and decodes them (a5, decode_attn.cuh:469-688); the last
//             unit of a head merges the partial states (ticket,
//             :937-1047).
// Units are claimed in group order and a scorer claims only after its
// scoring, so a unit waits only on scorers that never wait: no deadlock.
// Every counter is re-armed by its last user, so the workspace stays zeroed
// between calls; a wait past ~1 s records AOAKV_DEV_ERR_TIMEOUT and the CTA
// returns (the caller must then zero the workspace again).
#include <cmath>

#include "decode.cuh"
#include "estimate.cuh"
#include "fused.h"
#include "grid_sync.cuh"
#include "plan.h"
#include "step_append.cuh"
#include "topk.cuh"
#include "topk_bitonic.cuh"

#ifdef AOAKV_PHASE_PROBE
// Development builds with -DAOAKV_PHASE_PROBE record %globaltimer per CTA at
// phase boundaries (8 slots per CTA); the library build has no stamps.
namespace aoakv {
__device__ uint64_t g_pipe_ns[2048 * 8];
}  // namespace aoakv
#define PIPE_STAMP(i)                                                          \
  do {                                                                         \
    if (threadIdx.x == 0) g_pipe_ns[blockIdx.x * 8 + (i)] = aoakv::global_ns(); \
  } while (0)
#else
#define PIPE_STAMP(i) \
  do {                \
  } while (0)
#endif
#define AOAKV_TOPK_STAMP(i) PIPE_STAMP(i)
#include "topk_hist.cuh"

namespace aoakv {
namespace {

constexpr int kPThreads = kFusedThreads;  // 512
constexpr int kPWarps = kPThreads / 32;
constexpr int kPGroup = 8;       // heads per scoring group
constexpr int kPStages = 6;      // scorer ring depth
constexpr int kPMaxRange = 64;   // pages per scorer
constexpr int kPMaxWin = kDecMaxChunk;

__host__ __device__ constexpr int pipe_stage_bytes(int D) {
  // pages per stage x (max, min) x 8 heads x D fp16 = 16 KB for D = 64 or 128
  return (kPThreads / (kPGroup * (D / 8))) * 2 * kPGroup * D * 2;
}
__host__ __device__ inline int pipe_q_bytes(int H, int D) { return (H * D * 2 + 127) / 128 * 128; }
__host__ __device__ inline int pipe_keys_bytes(int n_score) {
  return hist_stage_bytes(n_score, true);
}
__host__ __device__ inline int pipe_vl_bytes(int H) { return (kPMaxRange * H * 2 + 127) / 128 * 128; }

__host__ __device__ inline int pipe_smem_bytes(int H, int D, int P, int n_score, int chunk) {
  const int scorer = pipe_q_bytes(H, D) + pipe_vl_bytes(H) + kPStages * pipe_stage_bytes(D);
  const int xb = static_cast<int>(bitonic_xbuf_bytes(kPWarps, kBitonicMaxK));
  const int hb = static_cast<int>(sizeof(HistSmem));
  const int sel = pipe_keys_bytes(n_score) + (xb > hb ? xb : hb);
  const int dec = static_cast<int>(dec_smem_bytes(D, P, chunk, kPWarps));
  int m = scorer > sel ? scorer : sel;
  if (dec > m) m = dec;
  return m + 128;  // alignment slack for the TMA tiles
}

// Scorer: a1 for head b (b < H), then the page range [pb, pe) for every
// head group, arriving on est_done[g] after each group.
template <int D>
__device__ __forceinline__ void pipe_score(const FusedArgs& f, const CUtensorMap* gmap, int e,
                                           int NE, uint8_t* smem, uint64_t* ebars, int* ids_s,
                                           uint32_t* est_done) {
  constexpr int L = D / 8;              // lanes per head row
  constexpr int TPP = kPGroup * L;      // threads per page
  constexpr int PPS = kPThreads / TPP;  // pages per stage
  constexpr int HGD2 = kPGroup * D * 2;  // bytes of one (max or min) box
  const EstimateArgs& a = f.est;
  const int tid = threadIdx.x, H = f.H, P = f.P;
  const int NG = H / kPGroup;
  const bool aoa = a.mode == AOAKV_SCORE_AOAKV;
  int pb, pe;
  page_range(a.n_score, e, NE, &pb, &pe);
  const int R = pe - pb;
  const int nc = (R + PPS - 1) / PPS;  // stages per group
  const int NI = NG * nc;
  __half* q_s = reinterpret_cast<__half*>(smem);
  __half* vl_s = reinterpret_cast<__half*>(smem + pipe_q_bytes(H, D));  // [R][H]
  uint8_t* ring = smem + pipe_q_bytes(H, D) + pipe_vl_bytes(H);
  for (int i = tid; i < H * D / 8; i += kPThreads)
    reinterpret_cast<uint4*>(q_s)[i] = __ldg(reinterpret_cast<const uint4*>(a.q) + i);
  for (int t = tid; t < R; t += kPThreads) {
    const int p = pb + t;
    int mp = __ldg(a.meta_indices + p / P);
    const int pid = aoa ? (a.kv_indices ? __ldg(a.kv_indices + p) : p) : 0;
    if (mp < 0 || mp >= a.meta_cap || pid < 0 || (aoa && pid >= a.kv_cap)) {
      raise_dev_error(a.err, AOAKV_DEV_ERR_BAD_PAGE);
      mp = -1;
    }
    ids_s[2 * t] = mp;
    ids_s[2 * t + 1] = pid;
  }
  __syncthreads();
  if (aoa)  // every page's v_log_norm row, once: no global load inside the ring loop
    for (int i = tid; i < R * H; i += kPThreads) {
      const int t = i / H;
      vl_s[i] = ids_s[2 * t] >= 0 ? a.vlog[static_cast<size_t>(ids_s[2 * t + 1]) * H + i % H]
                                  : __float2half(0.f);
    }
  auto issue = [&](int i) {  // thread 0: stage i % kPStages <- group i / nc, chunk i % nc
    const int g = i / nc, j = i % nc, s = i % kPStages;
    uint8_t* st = ring + s * pipe_stage_bytes(D);
    uint32_t nbytes = 0;
    for (int uu = 0; uu < PPS; ++uu) {
      const int t = j * PPS + uu;
      if (t < R && ids_s[2 * t] >= 0) nbytes += 2 * HGD2;
    }
    if (nbytes == 0) {
      mbar_arrive(&ebars[s]);
      return;
    }
    mbar_arrive_expect_tx(&ebars[s], nbytes);
    for (int uu = 0; uu < PPS; ++uu) {
      const int t = j * PPS + uu;
      if (t >= R || ids_s[2 * t] < 0) continue;
      const int row = ids_s[2 * t] * 2 * P + (pb + t) % P;
      tma_load_3d(st + (uu * 2) * HGD2, gmap, 0, g * kPGroup, row, &ebars[s]);
      tma_load_3d(st + (uu * 2 + 1) * HGD2, gmap, 0, g * kPGroup, row + P, &ebars[s]);
    }
  };
  if (tid == 0) {
    fence_proxy_async();
    for (int i = 0; i < NI && i < kPStages; ++i) issue(i);
  }
  // a1 while the first boxes are in flight
  if (e < H && tid < 32) append_head<D>(f, e);
  __syncthreads();  // the issuing thread rejoins its warp; q_s, ids_s ready

  const int u = tid / TPP, hl = (tid / L) % kPGroup, lane = tid % L;
  float qv[8];
  uint32_t msk[4];
  for (int i = 0; i < NI; ++i) {
    const int g = i / nc, j = i % nc, s = i % kPStages;
    const int h = g * kPGroup + hl;
    if (j == 0) {  // new group: this thread's head changes
      u4_to_f8(*reinterpret_cast<const uint4*>(q_s + h * D + lane * 8), qv);
#pragma unroll
      for (int k = 0; k < 4; ++k)
        msk[k] = (qv[2 * k] > 0.f ? 0x0000ffffu : 0u) | (qv[2 * k + 1] > 0.f ? 0xffff0000u : 0u);
    }
    const int t = j * PPS + u;
    const bool valid = t < R && ids_s[2 * t] >= 0;
    const bool arrived = mbar_wait_bounded(&ebars[s], (i / kPStages) & 1u, a.err);
    const uint8_t* st = ring + s * pipe_stage_bytes(D) + (u * 2) * HGD2 +
                        (static_cast<size_t>(hl) * D + lane * 8) * 2;
    const uint4 mx = *reinterpret_cast<const uint4*>(st);
    const uint4 mn = *reinterpret_cast<const uint4*>(st + HGD2);
    uint4 sel;
    sel.x = (mx.x & msk[0]) | (mn.x & ~msk[0]);
    sel.y = (mx.y & msk[1]) | (mn.y & ~msk[1]);
    sel.z = (mx.z & msk[2]) | (mn.z & ~msk[2]);
    sel.w = (mx.w & msk[3]) | (mn.w & ~msk[3]);
    float fv[8];
    u4_to_f8(sel, fv);
    float s0 = qv[0] * fv[0], s1 = qv[1] * fv[1];
#pragma unroll
    for (int k = 2; k < 8; k += 2) {
      s0 = fmaf(qv[k], fv[k], s0);
      s1 = fmaf(qv[k + 1], fv[k + 1], s1);
    }
    float sc = s0 + s1;
#pragma unroll
    for (int o = L / 2; o > 0; o >>= 1) sc += __shfl_xor_sync(0xffffffffu, sc, o);
    if (valid && arrived && lane == 0) {
      const float score =
          aoa ? a.two_rsqrt_d * sc + 2.f * __half2float(vl_s[t * H + h]) : sc;
      static_cast<float*>(a.out)[static_cast<size_t>(h) * a.out_stride + pb + t] = score;
    }
    __syncthreads();  // stage s consumed; this group's scores of the stage written
    if (tid == 0) {
      if (j == nc - 1) {  // group g complete in this CTA
        __threadfence();
        atomicAdd(est_done + g, 1u);
      }
      if (i + kPStages < NI) {
        fence_proxy_async();
        issue(i + kPStages);
      }
    }
    __syncwarp();  // the issuing thread rejoins warp 0 before its next wait
  }
  if (NI == 0 && tid == 0) {  // no pages here: arrive on every group
    __threadfence();
    for (int g = 0; g < NG; ++g) atomicAdd(est_done + g, 1u);
  }
}

template <int D>
__global__ void __launch_bounds__(kPThreads, 2)
    pipe_step_kernel(const __grid_constant__ CUtensorMap tmap,
                     const __grid_constant__ CUtensorMap gmap, FusedArgs f) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 127) & ~static_cast<uintptr_t>(127));
  __shared__ TopkSmem tsm;
  __shared__ int ok_s, flag_s, unit_s;
  __shared__ uint64_t bars[kDecMaxChunk];
  __shared__ int tok_s[kDecMaxChunk];
  __shared__ int win_s[kPMaxWin];
  __shared__ uint64_t ebars[kPStages];
  __shared__ int ids_s[2 * kPMaxRange];

  const int G = gridDim.x, b = blockIdx.x, H = f.H;
  const int NE = G / 2, NG = H / kPGroup;
  uint32_t* unit_ctr = f.sync;
  uint32_t* est_done = f.sync + 1;
  uint32_t* passed = f.sync + 1 + NG;

  PIPE_STAMP(0);
  if (threadIdx.x == 0) {
    for (int j = 0; j < kDecMaxChunk; ++j) mbar_init(&bars[j], 1);
    for (int j = 0; j < kPStages; ++j) mbar_init(&ebars[j], 1);
    fence_mbar_init();
    tma_prefetch_desc(&tmap);
    if (b < NE) tma_prefetch_desc(&gmap);
  }
  __syncthreads();
  if (b < NE) pipe_score<D>(f, &gmap, b, NE, smem, ebars, ids_s, est_done);
  PIPE_STAMP(1);

  // ---- units: claim (head, chunk) in head order until none is left
  const int n_chunks = f.dec.n_chunks, C = f.dec.chunk_pages;
  const int n_units = H * n_chunks;
  const uint32_t units_per_group = static_cast<uint32_t>(kPGroup * n_chunks);
  float* mrg = reinterpret_cast<float*>(smem + kDecHeader);
  __half* tiles = reinterpret_cast<__half*>(smem + dec_tile_offset(D, kPWarps));
  uint32_t* keys = reinterpret_cast<uint32_t*>(smem);
  uint32_t phase_bits = 0;
  for (;;) {
    __syncthreads();  // smem of the previous unit (or of the scorer) is free
    if (threadIdx.x == 0) unit_s = static_cast<int>(atomicAdd(unit_ctr, 1u));
    __syncthreads();
    const int u = unit_s;
    if (u >= n_units) {
      if (threadIdx.x == 0 && u == n_units + G - 1) *unit_ctr = 0u;  // the last claim
      break;
    }
    const int h = u / n_chunks, c = u % n_chunks, g = h / kPGroup;
    if (!cta_wait_geq(est_done + g, static_cast<uint32_t>(NE), &ok_s, f.err)) return;
    PIPE_STAMP(2);
    if (threadIdx.x == 0 && atomicAdd(passed + g, 1u) == units_per_group - 1) {
      est_done[g] = 0u;  // every unit of the group has passed its wait
      passed[g] = 0u;
    }
    const int win_lo = c * C;
    const int win_hi = min(f.k_sel, win_lo + C);
    TopkArgs ta;
    ta.scores = f.est.out;
    ta.s_stride = f.est.out_stride;
    ta.in_idx = f.kv_indices;
    ta.in_stride = 0;
    ta.out_vals = nullptr;
    ta.ov_stride = 0;
    const bool full_row = f.selected_out && c == 0;
    ta.out_idx = full_row ? f.selected_out : nullptr;
    ta.oi_stride = f.sel_cols;
    ta.f32 = 1;
    ta.n = f.est.n_score;
    ta.k = f.k_sel;
    ta.sink = f.sink;
    uint8_t* un = smem + pipe_keys_bytes(ta.n);
    if (!topk_row_hist<true>(ta, h, reinterpret_cast<uint8_t*>(keys), true,
                             *reinterpret_cast<HistSmem*>(un), win_s, win_lo, win_hi)) {
      // many equal scores: exact fallbacks
      if (f.k_sel <= 128)
        topk_row_small<true, 4>(ta, h, keys, reinterpret_cast<uint64_t*>(un), win_s, win_lo,
                                win_hi);
      else
        topk_row_cg(ta, h, keys, tsm, win_s, win_lo, win_hi);
    }
    if (full_row)  // the last page after the selection, -1 padding
      for (int i = f.k_sel + threadIdx.x; i < f.sel_cols; i += blockDim.x)
        f.selected_out[static_cast<size_t>(h) * f.sel_cols + i] =
            i == f.k_sel ? __ldg(f.kv_indices + f.n_pages - 1) : -1;
    __syncthreads();
    PIPE_STAMP(3);
    if (threadIdx.x == 0)  // (issues a proxy fence: appended page -> TMA reads)
      decode_issue(f.dec, &tmap, h, c, bars, tok_s, tiles, D, win_s, win_lo);
    __syncthreads();
    decode_compute_multi<D, kPWarps>(f.dec, h, c, bars, tok_s, tiles, mrg, &flag_s,
                                     phase_bits, nullptr);
    const int ns = min(f.dec.n_sel + 1, (c + 1) * C) - c * C;
    for (int j = 0; j < ns; ++j)
      if (tok_s[j] > 0) phase_bits ^= 1u << j;
    PIPE_STAMP(4);
  }
}

}  // namespace

int pipe_supported(int H, int D, int P, int n_score, int k_sel, int* grid_out,
                   size_t* smem_out, int* chunk_out, int* n_chunks_out) {
  if (H % kPGroup != 0 || H * D * 2 > 32 * 1024 || (D != 64 && D != 128)) return 0;
  const int chunk = kDecMaxChunk;
  const int smem = pipe_smem_bytes(H, D, P, n_score, chunk);
  if (smem > 200 * 1024) return 0;
  const void* fn = D == 128 ? reinterpret_cast<const void*>(pipe_step_kernel<128>)
                            : reinterpret_cast<const void*>(pipe_step_kernel<64>);
  if (cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess)
    return 0;
  int occ = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, fn, kPThreads, smem) != cudaSuccess ||
      occ < 2)
    return 0;
  const int grid = 2 * num_sms();  // one scorer and one unit CTA per SM
  const int NE = grid / 2;
  if ((n_score + NE - 1) / NE > kPMaxRange) return 0;
  *grid_out = grid;
  *smem_out = static_cast<size_t>(smem);
  *chunk_out = chunk;
  *n_chunks_out = (k_sel + 1 + chunk - 1) / chunk;
  return 1;
}

int launch_pipe(const CUtensorMap& tmap, const CUtensorMap& gmap, const FusedArgs& f, int D,
                int grid, size_t smem, cudaStream_t s) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kPThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (D == 128)
    AOAKV_CUDA_TRY(cudaLaunchKernelEx(&cfg, pipe_step_kernel<128>, tmap, gmap, f),
                   "pipelined step launch");
  else
    AOAKV_CUDA_TRY(cudaLaunchKernelEx(&cfg, pipe_step_kernel<64>, tmap, gmap, f),
                   "pipelined step launch");
  return AOAKV_OK;
}

int pipe_group_heads() { return kPGroup; }

}  // namespace aoakv

#ifdef AOAKV_PHASE_PROBE
extern "C" __attribute__((visibility("default"))) int aoakv_probe_pipe_ns(uint64_t* host, int n) {
  return cudaMemcpyFromSymbol(host, aoakv::g_pipe_ns, static_cast<size_t>(n) * 8) == cudaSuccess
             ? 0
             : 3;
}
#endif
