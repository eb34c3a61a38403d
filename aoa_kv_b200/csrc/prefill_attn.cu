// Paged prefill attention on the tcgen05 tensor cores: the counterpart of
// the reference's prefill_with_paged_kv_cache (quest/ops/csrc/
// batch_prefill.cu:27-116 over include/prefill/prefill.cuh:688-1119), one
// sequence of qo_len new tokens whose K/V already sit in the paged cache.
// Query i sits at position kv_len - qo_len + i and, causal, attends KV
// tokens j <= i + kv_len - qo_len (the mask tril(kv_len - qo_len) of
// quest/tests/test_prefill_attention.py:34-36); scale 1/sqrt(D) unless
// given. Query head h reads KV head h / (Hq / Hk).
//
// One CTA per (256-query block, query head): two query tiles A and B of 128
// rows share every K/V tile. 352 threads:
//   warps 0-3  softmax of tile A: thread r owns row r (tensor-memory lane r)
//   warps 4-7  softmax of tile B, same lanes, its own tensor-memory columns
//   warp 8     TMA: the Q tiles once, then K tiles of 128 tokens (one box per
//              page and 64-channel block) through a 3-stage ring
//   warp 10    TMA: the V tiles through a 2-stage ring
//   warp 9     tensor memory allocation; one thread issues the MMAs
// Tensor memory (512 columns): S_A / P_A, S_B / P_B (128 each), O_A, O_B.
// Per KV tile j the MMA thread issues, in this order,
//   PV_A(j)    O_A += P_A(j) V_j   (P_A read from tensor memory)
//   S_A(j+1)   S_A = Q_A K_{j+1}^T (over P_A: after PV_A(j) in issue order)
//   PV_B(j), S_B(j+1)
// so the tensor cores work on one tile while the softmax warps of the other
// exponentiate. Each softmax warp reads its S row, writes P (fp16) over the
// first 64 columns of S, and signals; the completion of S(j+1) also means
// PV(j) is done, so O can be rescaled right then. A row's running max is
// only raised (and its O row rescaled) when the tile's max exceeds it by
// more than 8 in log2 units; P then stays <= 256, well inside fp16, and the
// final O / l does not depend on which max was used.
#include <cudaTypedefs.h>

#include <cmath>

#include "plan.h"
#include "tcgen05.cuh"

namespace aoakv {
namespace {

constexpr int kPfRows = 128;                   // rows per query tile, KV tokens per tile
constexpr int kPfThreads = 352;
constexpr int kPfKStages = 3;                  // K tiles are freed as soon as both S are done
constexpr int kPfVStages = 2;                  // V tiles after both PV
constexpr uint32_t kPfBlock = kPfRows * 128;   // 128 rows x 64 fp16: one swizzled block
constexpr uint32_t kPfTmemCols = 512;
constexpr float kPfRescale = 8.f;              // log2 growth that forces a rescale

struct PrefillArgs {
  __half* o;                   // [qo_len, Hq, D]
  float* lse;                  // optional [qo_len, Hq], natural log
  const int32_t* kv_indices;   // [n_pages]
  int n_pages, kv_len, kv_cap;
  int qo_len, Hq, group, P;
  int causal;
  int n_blocks;                // 256-row query blocks
  float scale_log2;            // sm_scale * log2(e)
  int* err;
};

template <int D>
struct PfLayout {
  static constexpr int NH = D / 64;                      // 64-channel blocks
  static constexpr uint32_t tile = NH * kPfBlock;        // one Q, K or V tile
  static constexpr uint32_t q = 0;                       // Q_A, Q_B
  static constexpr uint32_t k = 2 * tile;                // kPfKStages tiles
  static constexpr uint32_t v = k + kPfKStages * tile;   // kPfVStages tiles
  static constexpr uint32_t bars = v + kPfVStages * tile;
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

// KV tiles a query tile needs: causal rows stop at their diagonal.
__device__ __forceinline__ int pf_tiles(const PrefillArgs& a, int row0) {
  if (row0 >= a.qo_len) return 0;
  const int last = min(row0 + kPfRows, a.qo_len) - 1;
  const int hi = a.causal ? min(a.kv_len, last + a.kv_len - a.qo_len + 1) : a.kv_len;
  return (hi + kPfRows - 1) / kPfRows;
}

// The softmax warpgroup of one query tile (rows row0 ..): n_tiles KV tiles,
// S / P at tensor-memory column s_col, O at o_col.
template <int D>
__device__ void pf_softmax(const PrefillArgs& a, uint8_t* smem, uint32_t tmem, int row0,
                           int n_tiles, int zero_from, uint32_t s_col, uint32_t o_col,
                           uint64_t* s_full, uint64_t* p_ready, uint64_t* o_final,
                           uint64_t* v_full, int h, volatile int* abort_flag) {
  using L = PfLayout<D>;
  const int warp = (threadIdx.x >> 5) & 3;
  const int r = (threadIdx.x & 127);  // row of the tile, tensor-memory lane
  const uint32_t lane_base = tmem + (static_cast<uint32_t>(warp * 32) << 16);
  const int q_row = row0 + r;
  const int row_hi = min(a.kv_len, a.causal ? q_row + a.kv_len - a.qo_len + 1 : a.kv_len);
  float m_run = -INFINITY, l_run = 0.f;
  for (int j = 0; j < n_tiles; ++j) {
    if (!pf_wait_warp(&s_full[0], j & 1, a.err, abort_flag)) return;
    tc_fence_after();
    const int lim = row_hi - j * kPfRows;  // valid columns [0, lim)
    // pass 1: the tile's row max
    float mx8[8];
#pragma unroll
    for (int t = 0; t < 8; ++t) mx8[t] = -INFINITY;
#pragma unroll
    for (int half = 0; half < 2; ++half) {
      uint32_t u[64];
      tmem_ld64(lane_base + s_col + half * 64, u);
      const int lh = lim - half * 64;
      if (lh < 64) {
#pragma unroll
        for (int i = 0; i < 64; ++i)
          if (i >= lh) u[i] = 0xff800000u;  // -inf
      }
#pragma unroll
      for (int i = 0; i < 64; ++i) mx8[i & 7] = fmaxf(mx8[i & 7], __uint_as_float(u[i]));
    }
    float mx = fmaxf(fmaxf(fmaxf(mx8[0], mx8[1]), fmaxf(mx8[2], mx8[3])),
                     fmaxf(fmaxf(mx8[4], mx8[5]), fmaxf(mx8[6], mx8[7])));
    mx *= a.scale_log2;
    const bool raise = mx > m_run + kPfRescale;
    const float f = raise ? ex2_approx(m_run - mx) : 1.f;  // 0 while m_run is -inf
    // S(j) complete means PV(j-1) is too: O holds tiles < j
    if (j > 0 && __any_sync(0xffffffffu, raise)) {
#pragma unroll
      for (int c = 0; c < D / 32; ++c) {
        uint32_t u[32];
        tmem_ld32(lane_base + o_col + c * 32, u);
#pragma unroll
        for (int i = 0; i < 32; ++i) u[i] = __float_as_uint(__uint_as_float(u[i]) * f);
        tmem_st32(lane_base + o_col + c * 32, u);
      }
    }
    if (raise) {
      l_run *= f;
      m_run = mx;
    }
    // the tile holding kv_len may hold cache slots past it (the last page's
    // unused tail): zero those V rows, since 0 * NaN would poison O. The
    // first warpgroup to attend the tile does it, before its PV.
    const int kv0 = j * kPfRows;
    if (kv0 + kPfRows > a.kv_len && j >= zero_from) {
      const int s = j % kPfVStages;
      if (!pf_wait_warp(&v_full[s], (j / kPfVStages) & 1, a.err, abort_flag)) return;
      if (r >= a.kv_len - kv0) {
        uint8_t* vb = smem + L::v + s * L::tile + r * 128;
#pragma unroll
        for (int c = 0; c < L::NH; ++c)
#pragma unroll
          for (int u = 0; u < 8; ++u)
            *reinterpret_cast<uint4*>(vb + c * kPfBlock + u * 16) = make_uint4(0, 0, 0, 0);
      }
      fence_proxy_async_smem();
    }
    // pass 2: P = 2^(s * scale_log2 - m), fp16, over the first 64 columns
    const float neg_m = m_run == -INFINITY ? 0.f : -m_run;
    float sum8[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int half = 0; half < 2; ++half) {
      uint32_t u[64];
      tmem_ld64(lane_base + s_col + half * 64, u);
      const int lh = lim - half * 64;
      if (lh < 64) {
#pragma unroll
        for (int i = 0; i < 64; ++i)
          if (i >= lh) u[i] = 0xff800000u;
      }
      uint32_t pk[32];
#pragma unroll
      for (int t = 0; t < 32; ++t) {
        const float p0 = ex2_approx(fmaf(__uint_as_float(u[2 * t]), a.scale_log2, neg_m));
        const float p1 = ex2_approx(fmaf(__uint_as_float(u[2 * t + 1]), a.scale_log2, neg_m));
        sum8[t & 7] += p0 + p1;
        const __half2 hp = __floats2half2_rn(p0, p1);
        pk[t] = *reinterpret_cast<const uint32_t*>(&hp);
      }
      tmem_st32(lane_base + s_col + half * 32, pk);
    }
    l_run += ((sum8[0] + sum8[1]) + (sum8[2] + sum8[3])) +
             ((sum8[4] + sum8[5]) + (sum8[6] + sum8[7]));
    tc_fence_before();
    mbar_arrive(p_ready);
  }
  if (n_tiles == 0 || !pf_wait_warp(o_final, 0, a.err, abort_flag)) return;
  tc_fence_after();
  const bool live = q_row < a.qo_len;
  const float inv = live ? 1.f / l_run : 0.f;
  __half* dst = a.o + (static_cast<size_t>(live ? q_row : 0) * a.Hq + h) * D;
#pragma unroll
  for (int c = 0; c < D / 32; ++c) {
    uint32_t u[32];
    tmem_ld32(lane_base + o_col + c * 32, u);  // whole warp, rows past qo_len too
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
    a.lse[static_cast<size_t>(q_row) * a.Hq + h] = (m_run + log2f(l_run)) * 0.6931471805599453f;
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
  uint64_t* s_full = v_empty + kPfVStages;     // [2]: tiles A, B
  uint64_t* p_ready = s_full + 2;              // [2]
  uint64_t* o_final = p_ready + 2;
  uint64_t* mma_idle = o_final + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(mma_idle + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int qb = a.causal ? a.n_blocks - 1 - static_cast<int>(blockIdx.x)
                          : static_cast<int>(blockIdx.x);  // causal: longest rows first
  const int h = blockIdx.y, hk = h / a.group;
  const int q0 = qb * 2 * kPfRows;
  const int n_a = pf_tiles(a, q0), n_b = pf_tiles(a, q0 + kPfRows);
  const int n_tiles = max(n_a, n_b);  // n_b is n_a or n_a + 1, or 0 past qo_len
  // tensor-memory columns of tile t: S / P at 128 t, O at 256 + 128 t

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
    for (int t = 0; t < 2; ++t) {
      mbar_init(&s_full[t], 1);
      mbar_init(&p_ready[t], 128);
    }
    mbar_init(o_final, 1);
    mbar_init(mma_idle, 1);
    *abort_flag = 0;
    fence_mbar_init();
    tma_prefetch_desc(&qmap);
    tma_prefetch_desc(&kvmap);
  }
  if (warp == 9) tmem_alloc(tmem_slot, kPfTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 8) {
    // ---------------------------------------------- Q and K producer
    if (lane == 0) {
      const int nq = n_b > 0 ? 2 : 1;
      mbar_arrive_expect_tx(q_full, nq * NH * kPfBlock);
      for (int t = 0; t < nq; ++t)
        for (int c = 0; c < NH; ++c)
          tma_load_3d(smem + L::q + t * L::tile + c * kPfBlock, &qmap, c * 64, h,
                      q0 + t * kPfRows, q_full);
      pf_produce<NH>(a, &kvmap, smem + L::k, kPfKStages, k_full, k_empty, 0, hk, n_tiles,
                     abort_flag);
      mbar_wait_bounded(q_full, 0, a.err);
    }
  } else if (warp == 10) {
    // ---------------------------------------------------- V producer
    if (lane == 0)
      pf_produce<NH>(a, &kvmap, smem + L::v, kPfVStages, v_full, v_empty, 1, hk, n_tiles,
                     abort_flag);
  } else if (warp == 9) {
    // ------------------------------------------------------- MMA issuer
    if (lane == 0) {
      constexpr uint32_t id_s = umma_idesc_f16_f32(128, 128, 0, 0);
      constexpr uint32_t id_o = umma_idesc_f16_f32(128, D, 0, 1);
      const uint32_t q_addr = smem_addr(smem + L::q);
      auto issue_s = [&](int t, int j) {  // S_t(j) = Q_t K_j^T
        const uint32_t qa = q_addr + t * L::tile;
        const uint32_t ka = smem_addr(smem + L::k + (j % kPfKStages) * L::tile);
#pragma unroll
        for (int k = 0; k < D / 16; ++k) {
          const uint32_t o = (k >> 2) * kPfBlock + (k & 3) * 32;
          umma_f16_ss(tmem + t * 128u, umma_desc_sw128(qa + o, 16, 1024),
                      umma_desc_sw128(ka + o, 16, 1024), id_s, k > 0);
        }
        umma_commit(&s_full[t]);
      };
      auto issue_pv = [&](int t, int j) {  // O_t += P_t(j) V_j
        const uint32_t va = smem_addr(smem + L::v + (j % kPfVStages) * L::tile);
#pragma unroll
        for (int k = 0; k < kPfRows / 16; ++k)
          umma_f16_ts(tmem + 256u + t * 128u, tmem + t * 128u + k * 8,
                      umma_desc_sw128(va + k * 16 * 128, kPfBlock, 1024), id_o,
                      (j > 0 || k > 0) ? 1u : 0u);
      };
      bool ok = pf_wait(q_full, 0, a.err, abort_flag) &&
                pf_wait(&k_full[0], 0, a.err, abort_flag);
      if (ok) {
        tc_fence_after();
        for (int t = 0; t < 2; ++t)
          if ((t == 0 ? n_a : n_b) > 0) issue_s(t, 0);
        umma_commit(&k_empty[0]);
      }
      for (int j = 0; ok && j < n_tiles; ++j) {
        const int vs = j % kPfVStages;
        if (!pf_wait(&v_full[vs], (j / kPfVStages) & 1, a.err, abort_flag)) break;
        const bool next = j + 1 < n_tiles;
        bool k_ready = false;
        for (int t = 0; t < 2; ++t) {
          const int n_t = t == 0 ? n_a : n_b;
          if (j < n_t) {
            if (!pf_wait(&p_ready[t], j & 1, a.err, abort_flag)) {
              ok = false;
              break;
            }
            tc_fence_after();
            issue_pv(t, j);
          }
          if (next && j + 1 < n_t) {
            if (!k_ready) {
              if (!pf_wait(&k_full[(j + 1) % kPfKStages], ((j + 1) / kPfKStages) & 1, a.err,
                           abort_flag)) {
                ok = false;
                break;
              }
              tc_fence_after();
              k_ready = true;
            }
            issue_s(t, j + 1);
          }
        }
        if (!ok) break;
        if (next) umma_commit(&k_empty[(j + 1) % kPfKStages]);
        umma_commit(&v_empty[vs]);
      }
      umma_commit(o_final);  // every MMA issued above has finished
      umma_commit(mma_idle);
      mbar_wait_bounded(mma_idle, 0, a.err);
    }
  } else {
    // ------------------------------------------- softmax, tiles A and B
    const int t = warp >> 2;
    pf_softmax<D>(a, smem, tmem, q0 + t * kPfRows, t == 0 ? n_a : n_b, t == 0 ? 0 : n_a,
                  t * 128u, 256u + t * 128u, &s_full[t], &p_ready[t], o_final, v_full, h,
                  abort_flag);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 9) {
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
  a.n_blocks = (qo_len + 2 * kPfRows - 1) / (2 * kPfRows);
  const float scale = sm_scale > 0.f ? sm_scale : 1.f / std::sqrt(static_cast<float>(head_dim));
  a.scale_log2 = scale * 1.4426950408889634f;
  a.err = dev_error_ptr();

  const size_t smem = (head_dim == 128 ? PfLayout<128>::bytes : PfLayout<64>::bytes) + 1024;
  const void* fn = head_dim == 128 ? reinterpret_cast<const void*>(prefill_attn_kernel<128>)
                                   : reinterpret_cast<const void*>(prefill_attn_kernel<64>);
  AOAKV_CUDA_TRY(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                      static_cast<int>(smem)),
                 "prefill smem attribute");
  const dim3 grid(a.n_blocks, num_qo_heads);
  auto s = static_cast<cudaStream_t>(stream);
  if (head_dim == 128)
    prefill_attn_kernel<128><<<grid, kPfThreads, smem, s>>>(qmap, kvmap, a);
  else
    prefill_attn_kernel<64><<<grid, kPfThreads, smem, s>>>(qmap, kvmap, a);
  return cuda_status(cudaGetLastError(), "prefill launch");
}
