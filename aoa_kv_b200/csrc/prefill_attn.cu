// Paged prefill attention on the tcgen05 tensor cores: the counterpart of
// the reference's prefill_with_paged_kv_cache (quest/ops/csrc/
// batch_prefill.cu:27-116 over include/prefill/prefill.cuh:688-1119), one
// sequence of qo_len new tokens whose K/V already sit in the paged cache.
// Query i sits at position kv_len - qo_len + i and, causal, attends KV
// tokens j <= i + kv_len - qo_len (the mask tril(kv_len - qo_len) of
// quest/tests/test_prefill_attention.py:34-36); scale 1/sqrt(D) unless
// given. Query head h reads KV head h / (Hq / Hk).
//
// One CTA per (128-query tile, query head), 224 threads:
//   warps 0-3  softmax: thread r owns query row r (tensor-memory lane r)
//   warp 4     TMA: the Q tile once, then K tiles of 128 tokens (one box per
//              page and 64-channel half) through a 3-stage ring
//   warp 6     TMA: the V tiles through a 2-stage ring
//   warp 5     tensor memory allocation; one thread issues the MMAs
// Per KV tile j:  S_j = Q K_j^T   (M 128, N 128, K D) into S buffer j % 2
//                 softmax warps read S_j, write P_j (fp16) to shared memory
//                 O += P_j V_j     (M 128, N D, K 128; V read MN-major)
// S_{j+1} is issued before PV_j, so the tensor cores compute the next
// scores while the softmax warps exponentiate. A K tile is released when its
// S is done, a V tile when its PV is: the K ring runs further ahead. A row's running max is only
// raised (and its O row rescaled in tensor memory) when the tile's max
// exceeds it by more than 8 in log2 units; P then stays <= 256, well inside
// fp16, and the final O / l is unchanged by which max was used.
#include <cudaTypedefs.h>

#include <cmath>

#include "plan.h"
#include "tcgen05.cuh"

namespace aoakv {
namespace {

constexpr int kPfRows = 128;                   // query rows per CTA, KV tokens per tile
constexpr int kPfThreads = 224;
constexpr int kPfKStages = 3;                  // K tiles are freed as soon as S_j is done
constexpr int kPfVStages = 2;                  // V tiles only after PV_j
constexpr uint32_t kPfBlock = kPfRows * 128;   // 128 rows x 64 fp16: one swizzled block
constexpr uint32_t kPfTmemCols = 512;
constexpr uint32_t kPfTmemO = 256u;            // S buffers at columns 0 and 128
constexpr float kPfRescale = 8.f;              // log2 growth that forces a rescale

struct PrefillArgs {
  __half* o;                   // [qo_len, Hq, D]
  float* lse;                  // optional [qo_len, Hq], natural log
  const int32_t* kv_indices;   // [n_pages]
  int n_pages, kv_len, kv_cap;
  int qo_len, Hq, group, P;
  int causal;
  int n_qtiles;
  float scale_log2;            // sm_scale * log2(e)
  int* err;
};

template <int D>
struct PfLayout {
  static constexpr int NH = D / 64;                      // 64-channel blocks
  static constexpr uint32_t tile = NH * kPfBlock;        // one Q, K or V tile
  static constexpr uint32_t q = 0;
  static constexpr uint32_t k = tile;                    // kPfKStages tiles
  static constexpr uint32_t v = k + kPfKStages * tile;   // kPfVStages tiles
  static constexpr uint32_t p = v + kPfVStages * tile;   // 128 x 128 fp16: 2 blocks
  static constexpr uint32_t bars = p + 2 * kPfBlock;
  static constexpr uint32_t bytes = bars + 256;
};

// Bounded waits that give up for good once one of them has failed.
__device__ __forceinline__ bool pf_wait(uint64_t* bar, uint32_t parity, int* err,
                                        volatile int* abort_flag) {
  if (*abort_flag) return false;
  if (mbar_wait_bounded(bar, parity, err)) return true;
  *abort_flag = 1;
  return false;
}

// The same for a whole warp: true only if every lane's wait succeeded, so
// the warp stays converged for the .sync.aligned tensor-memory accesses.
__device__ __forceinline__ bool pf_wait_warp(uint64_t* bar, uint32_t parity, int* err,
                                             volatile int* abort_flag) {
  return __all_sync(0xffffffffu, pf_wait(bar, parity, err, abort_flag));
}

// One thread streams the K (kvsel 0) or V (kvsel 1) tiles of the CTA's KV
// range through a ring of `stages` tiles: one TMA box per page and 64-channel
// block; pages past the sequence read as zeros (page id = capacity is out
// of the tensor map). Waits at the end for its own copies still in flight.
template <int NH>
__device__ void pf_produce(const PrefillArgs& a, const CUtensorMap* map, uint8_t* ring,
                           int stages, uint64_t* full, uint64_t* empty, int kvsel, int hk,
                           int n_tiles, volatile int* abort_flag) {
  const int per_tile = kPfRows / a.P;
  int issued = 0;
  for (int j = 0; j < n_tiles; ++j) {
    const int s = j % stages;
    if (j >= stages && !pf_wait(&empty[s], ((j / stages) - 1) & 1, a.err, abort_flag)) break;
    uint8_t* buf = ring + s * NH * kPfBlock;
    mbar_arrive_expect_tx(&full[s], NH * kPfBlock);
    for (int pi = 0; pi < per_tile; ++pi) {
      const int g = j * per_tile + pi;
      int phys = a.kv_cap;
      if (g < a.n_pages) {
        phys = __ldg(a.kv_indices + g);
        if (phys < 0 || phys >= a.kv_cap) {
          raise_dev_error(a.err, AOAKV_DEV_ERR_BAD_PAGE);
          phys = a.kv_cap;
        }
      }
#pragma unroll
      for (int c = 0; c < NH; ++c)
        tma_load_3d(buf + c * kPfBlock + pi * a.P * 128, map, c * 64, hk,
                    (2 * phys + kvsel) * a.P, &full[s]);
    }
    issued = j + 1;
  }
  for (int j = max(0, issued - stages); j < issued; ++j)
    mbar_wait_bounded(&full[j % stages], (j / stages) & 1, a.err);
}

template <int D>
__global__ void __launch_bounds__(kPfThreads, 1)
    prefill_attn_kernel(const __grid_constant__ CUtensorMap qmap,
                        const __grid_constant__ CUtensorMap kvmap, const PrefillArgs a) {
  using L = PfLayout<D>;
  constexpr int NH = L::NH;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align_smem<1024>(smem_raw);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::bars);
  uint64_t* q_full = bars;
  uint64_t* k_full = q_full + 1;               // [kPfKStages]
  uint64_t* k_empty = k_full + kPfKStages;     // [kPfKStages]
  uint64_t* v_full = k_empty + kPfKStages;     // [kPfVStages]
  uint64_t* v_empty = v_full + kPfVStages;     // [kPfVStages]
  uint64_t* s_full = v_empty + kPfVStages;     // [2]
  uint64_t* p_ready = s_full + 2;
  uint64_t* o_done = p_ready + 1;
  uint64_t* mma_idle = o_done + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(mma_idle + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int qt = a.causal ? a.n_qtiles - 1 - static_cast<int>(blockIdx.x)
                          : static_cast<int>(blockIdx.x);  // causal: longest rows first
  const int h = blockIdx.y, hk = h / a.group;
  const int q0 = qt * kPfRows;
  const int off = a.kv_len - a.qo_len;
  const int last_q = min(q0 + kPfRows, a.qo_len) - 1;
  const int kv_hi = a.causal ? min(a.kv_len, last_q + off + 1) : a.kv_len;
  const int n_tiles = (kv_hi + kPfRows - 1) / kPfRows;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int s = 0; s < kPfKStages; ++s) {
      mbar_init(&k_full[s], 1);
      mbar_init(&k_empty[s], 1);
    }
    for (int s = 0; s < kPfVStages; ++s) {
      mbar_init(&v_full[s], 1);
      mbar_init(&v_empty[s], 1);
    }
    mbar_init(&s_full[0], 1);
    mbar_init(&s_full[1], 1);
    mbar_init(p_ready, 128);
    mbar_init(o_done, 1);
    mbar_init(mma_idle, 1);
    *abort_flag = 0;
    fence_mbar_init();
    tma_prefetch_desc(&qmap);
    tma_prefetch_desc(&kvmap);
  }
  if (warp == 5) tmem_alloc(tmem_slot, kPfTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 4) {
    // -------------------------------------------------- Q and K producer
    if (lane == 0) {
      mbar_arrive_expect_tx(q_full, NH * kPfBlock);
      for (int c = 0; c < NH; ++c)
        tma_load_3d(smem + L::q + c * kPfBlock, &qmap, c * 64, h, q0, q_full);
      pf_produce<NH>(a, &kvmap, smem + L::k, kPfKStages, k_full, k_empty, 0, hk, n_tiles,
                     abort_flag);
      mbar_wait_bounded(q_full, 0, a.err);
    }
  } else if (warp == 6) {
    // ------------------------------------------------------- V producer
    if (lane == 0)
      pf_produce<NH>(a, &kvmap, smem + L::v, kPfVStages, v_full, v_empty, 1, hk, n_tiles,
                     abort_flag);
  } else if (warp == 5) {
    // ---------------------------------------------------------- MMA issuer
    if (lane == 0) {
      constexpr uint32_t id_s = umma_idesc_f16_f32(128, 128, 0, 0);
      constexpr uint32_t id_o = umma_idesc_f16_f32(128, D, 0, 1);
      const uint32_t q_addr = smem_addr(smem + L::q);
      const uint32_t p_addr = smem_addr(smem + L::p);
      auto issue_s = [&](int j) -> bool {
        const int s = j % kPfKStages;
        if (!pf_wait(&k_full[s], (j / kPfKStages) & 1, a.err, abort_flag)) return false;
        tc_fence_after();
        const uint32_t k_addr = smem_addr(smem + L::k + s * L::tile);
#pragma unroll
        for (int k = 0; k < D / 16; ++k) {
          const uint32_t o = (k >> 2) * kPfBlock + (k & 3) * 32;
          umma_f16_ss(tmem + (j & 1) * 128u, umma_desc_sw128(q_addr + o, 16, 1024),
                      umma_desc_sw128(k_addr + o, 16, 1024), id_s, k > 0);
        }
        umma_commit(&s_full[j & 1]);
        umma_commit(&k_empty[s]);
        return true;
      };
      bool ok = pf_wait(q_full, 0, a.err, abort_flag) && issue_s(0);
      for (int j = 0; ok && j < n_tiles; ++j) {
        // S_{j+1} first: the tensor cores compute it while the softmax warps
        // still work on tile j
        if (j + 1 < n_tiles && !issue_s(j + 1)) break;
        const int s = j % kPfVStages;
        if (!pf_wait(p_ready, j & 1, a.err, abort_flag)) break;
        if (!pf_wait(&v_full[s], (j / kPfVStages) & 1, a.err, abort_flag)) break;
        tc_fence_after();
        const uint32_t v_addr = smem_addr(smem + L::v + s * L::tile);
#pragma unroll
        for (int k = 0; k < kPfRows / 16; ++k) {
          umma_f16_ss(tmem + kPfTmemO,
                      umma_desc_sw128(p_addr + (k >> 2) * kPfBlock + (k & 3) * 32, 16, 1024),
                      umma_desc_sw128(v_addr + k * 16 * 128, kPfBlock, 1024), id_o,
                      (j > 0 || k > 0) ? 1u : 0u);
        }
        umma_commit(o_done);
        umma_commit(&v_empty[s]);
      }
      umma_commit(mma_idle);  // every MMA issued above has finished
      mbar_wait_bounded(mma_idle, 0, a.err);
    }
  } else if (warp < 4) {
    // ------------------------------------------------------------- softmax
    // Every branch around a tensor-memory access is warp-uniform (votes):
    // tcgen05.ld / st are .sync.aligned.
    const int r = threadIdx.x;  // query row of the tile, tensor-memory lane
    const uint32_t lane_base = tmem + (static_cast<uint32_t>(warp * 32) << 16);
    const int q_row = q0 + r;
    const int row_hi = min(a.kv_len, a.causal ? q_row + off + 1 : a.kv_len);
    float m_run = -INFINITY, l_run = 0.f;
    bool ok = true;
    for (int j = 0; j < n_tiles; ++j) {
      if (!pf_wait_warp(&s_full[j & 1], (j >> 1) & 1, a.err, abort_flag)) {
        ok = false;
        break;
      }
      tc_fence_after();
      float sv[128];
      {
        uint32_t u[128];
        tmem_ld128(lane_base + (j & 1) * 128u, u);
#pragma unroll
        for (int i = 0; i < 128; ++i) sv[i] = __uint_as_float(u[i]);
      }
      const int kv0 = j * kPfRows;
      const int lim = row_hi - kv0;  // valid columns [0, lim)
      if (lim < kPfRows) {
#pragma unroll
        for (int i = 0; i < 128; ++i)
          if (i >= lim) sv[i] = -INFINITY;
      }
      float mx8[8];  // eight independent chains: one warp per scheduler has no
                     // other warps to hide a 128-long dependent chain behind
#pragma unroll
      for (int t = 0; t < 8; ++t) mx8[t] = sv[t];
#pragma unroll
      for (int i = 8; i < 128; ++i) mx8[i & 7] = fmaxf(mx8[i & 7], sv[i]);
      float mx = fmaxf(fmaxf(fmaxf(mx8[0], mx8[1]), fmaxf(mx8[2], mx8[3])),
                       fmaxf(fmaxf(mx8[4], mx8[5]), fmaxf(mx8[6], mx8[7])));
      mx *= a.scale_log2;
      const bool raise = mx > m_run + kPfRescale;
      const float f = raise ? ex2_approx(m_run - mx) : 1.f;  // 0 while m_run is -inf
      // PV_{j-1} accumulates into O and reads the P buffer: it must be done
      // before O is rescaled or P_j is written
      if (j > 0) {
        if (!pf_wait_warp(o_done, (j - 1) & 1, a.err, abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        if (__any_sync(0xffffffffu, raise)) {
#pragma unroll
          for (int c = 0; c < D / 32; ++c) {
            uint32_t u[32];
            tmem_ld32(lane_base + kPfTmemO + c * 32, u);
#pragma unroll
            for (int i = 0; i < 32; ++i) u[i] = __float_as_uint(__uint_as_float(u[i]) * f);
            tmem_st32(lane_base + kPfTmemO + c * 32, u);
          }
        }
      }
      if (raise) {
        l_run *= f;
        m_run = mx;
      }
      // the last tile may hold cache slots past kv_len (the last page's
      // unused tail): zero those V rows, since 0 * NaN would poison O
      if (kv0 + kPfRows > a.kv_len) {
        const int s = j % kPfVStages;
        if (!pf_wait_warp(&v_full[s], (j / kPfVStages) & 1, a.err, abort_flag)) {
          ok = false;
          break;
        }
        if (r >= a.kv_len - kv0) {
          uint8_t* vb = smem + L::v + s * L::tile + r * 128;
#pragma unroll
          for (int c = 0; c < NH; ++c)
#pragma unroll
            for (int u = 0; u < 8; ++u)
              *reinterpret_cast<uint4*>(vb + c * kPfBlock + u * 16) = make_uint4(0, 0, 0, 0);
        }
      }
      const float neg_m = m_run == -INFINITY ? 0.f : -m_run;
      float sum8[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
      uint8_t* prow = smem + L::p + r * 128;
#pragma unroll
      for (int cc = 0; cc < 16; ++cc) {  // 16 units of 8 columns
        uint32_t w[4];
#pragma unroll
        for (int t = 0; t < 4; ++t) {
          const float p0 = ex2_approx(fmaf(sv[cc * 8 + 2 * t], a.scale_log2, neg_m));
          const float p1 = ex2_approx(fmaf(sv[cc * 8 + 2 * t + 1], a.scale_log2, neg_m));
          sum8[t] += p0;
          sum8[t + 4] += p1;
          const __half2 hp = __floats2half2_rn(p0, p1);
          w[t] = *reinterpret_cast<const uint32_t*>(&hp);
        }
        const int unit = (cc & 7) ^ (r & 7);
        *reinterpret_cast<uint4*>(prow + (cc >> 3) * kPfBlock + unit * 16) =
            make_uint4(w[0], w[1], w[2], w[3]);
      }
      l_run += ((sum8[0] + sum8[1]) + (sum8[2] + sum8[3])) +
               ((sum8[4] + sum8[5]) + (sum8[6] + sum8[7]));
      fence_proxy_async_smem();  // P (and zeroed V rows) visible to the tensor cores
      tc_fence_before();
      mbar_arrive(p_ready);
    }
    if (ok && pf_wait_warp(o_done, (n_tiles - 1) & 1, a.err, abort_flag)) {
      tc_fence_after();
      const bool live = q_row < a.qo_len;
      const float inv = live ? 1.f / l_run : 0.f;
      __half* dst = a.o + (static_cast<size_t>(live ? q_row : 0) * a.Hq + h) * D;
#pragma unroll
      for (int c = 0; c < D / 32; ++c) {
        uint32_t u[32];
        tmem_ld32(lane_base + kPfTmemO + c * 32, u);  // whole warp, rows past qo_len too
        if (live) {
#pragma unroll
          for (int g = 0; g < 4; ++g) {
            uint32_t w[4];
#pragma unroll
            for (int t = 0; t < 4; ++t) {
              const __half2 hv = __floats2half2_rn(__uint_as_float(u[g * 8 + 2 * t]) * inv,
                                                   __uint_as_float(u[g * 8 + 2 * t + 1]) * inv);
              w[t] = *reinterpret_cast<const uint32_t*>(&hv);
            }
            *reinterpret_cast<uint4*>(dst + c * 32 + g * 8) = make_uint4(w[0], w[1], w[2], w[3]);
          }
        }
      }
      if (live && a.lse)
        a.lse[static_cast<size_t>(q_row) * a.Hq + h] =
            (m_run + log2f(l_run)) * 0.6931471805599453f;
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 5) {
    __syncwarp();
    tmem_dealloc(tmem, kPfTmemCols);
  }
}

}  // namespace

}  // namespace aoakv

using namespace aoakv;

extern "C" int aoakv_prefill_paged(const void* q, void* o, float* lse, const void* kv_data,
                                   int32_t kv_capacity_pages, const int32_t* kv_indices,
                                   int32_t num_kv_pages, int32_t kv_last_page_len,
                                   int32_t qo_len, int32_t num_qo_heads, int32_t num_kv_heads,
                                   int32_t head_dim, int32_t page_size, int32_t layout,
                                   int32_t causal, float sm_scale, void* stream) {
  AOAKV_NVTX("aoakv_prefill_paged");
  AOAKV_CHECK_ARG(q && o && kv_data && kv_indices, "prefill: NULL pointer");
  if (layout != AOAKV_LAYOUT_NHD)
    return set_error(AOAKV_ERR_UNSUPPORTED, "prefill: only the NHD layout is built");
  AOAKV_CHECK_ARG(head_dim == 64 || head_dim == 128, "prefill: head_dim must be 64 or 128");
  AOAKV_CHECK_ARG(page_size == 8 || page_size == 16 || page_size == 32 || page_size == 64 ||
                      page_size == 128,
                  "prefill: page_size must be 8, 16, 32, 64 or 128");
  AOAKV_CHECK_ARG(num_kv_heads >= 1 && num_qo_heads >= num_kv_heads &&
                      num_qo_heads % num_kv_heads == 0 && num_qo_heads <= 65535,
                  "prefill: num_qo_heads must be a multiple of num_kv_heads");
  AOAKV_CHECK_ARG(num_kv_pages >= 1 && kv_last_page_len >= 1 && kv_last_page_len <= page_size,
                  "prefill: need at least one page and 1 <= kv_last_page_len <= page_size");
  AOAKV_CHECK_ARG(kv_capacity_pages >= 1 &&
                      (static_cast<int64_t>(kv_capacity_pages) * 2 + 1) * page_size < (1LL << 31),
                  "prefill: kv_capacity_pages out of range");
  const int64_t kv_len = static_cast<int64_t>(num_kv_pages - 1) * page_size + kv_last_page_len;
  AOAKV_CHECK_ARG(qo_len >= 0, "prefill: qo_len must be >= 0");
  AOAKV_CHECK_ARG(!causal || qo_len <= kv_len,
                  "prefill: causal attention needs qo_len <= kv_len");
  AOAKV_CHECK_ARG(reinterpret_cast<uintptr_t>(q) % 16 == 0 &&
                      reinterpret_cast<uintptr_t>(o) % 16 == 0,
                  "prefill: q and o must be 16-byte aligned");
  if (qo_len == 0) return AOAKV_OK;
  CUtensorMap qmap, kvmap;
  int st = make_q_tmap_sw128(&qmap, q, num_qo_heads, head_dim, qo_len);
  if (st != AOAKV_OK) return st;
  st = make_kv_tmap_sw128(&kvmap, kv_data, num_kv_heads, head_dim, page_size, kv_capacity_pages);
  if (st != AOAKV_OK) return st;

  PrefillArgs a;
  a.o = static_cast<__half*>(o);
  a.lse = lse;
  a.kv_indices = kv_indices;
  a.n_pages = num_kv_pages;
  a.kv_len = static_cast<int>(kv_len);
  a.kv_cap = kv_capacity_pages;
  a.qo_len = qo_len;
  a.Hq = num_qo_heads;
  a.group = num_qo_heads / num_kv_heads;
  a.P = page_size;
  a.causal = causal != 0;
  a.n_qtiles = (qo_len + kPfRows - 1) / kPfRows;
  const float scale = sm_scale > 0.f ? sm_scale : 1.f / std::sqrt(static_cast<float>(head_dim));
  a.scale_log2 = scale * 1.4426950408889634f;
  a.err = dev_error_ptr();

  const size_t smem = (head_dim == 128 ? PfLayout<128>::bytes : PfLayout<64>::bytes) + 1024;
  const void* fn = head_dim == 128 ? reinterpret_cast<const void*>(prefill_attn_kernel<128>)
                                   : reinterpret_cast<const void*>(prefill_attn_kernel<64>);
  AOAKV_CUDA_TRY(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      static_cast<int>(smem)),
                 "prefill smem attribute");
  const dim3 grid(a.n_qtiles, num_qo_heads);
  auto s = static_cast<cudaStream_t>(stream);
  if (head_dim == 128)
    prefill_attn_kernel<128><<<grid, kPfThreads, smem, s>>>(qmap, kvmap, a);
  else
    prefill_attn_kernel<64><<<grid, kPfThreads, smem, s>>>(qmap, kvmap, a);
  return cuda_status(cudaGetLastError(), "prefill launch");
}
