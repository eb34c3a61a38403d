// Shared device helpers and host plumbing for libaoakv (sm_100a only).
#pragma once

#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <nvtx3/nvToolsExt.h>

#include <string>

#include "../../include/aoakv.h"

namespace aoakv {

// ---------------------------------------------------------------- host side
// Records `msg` as the calling thread's last error and returns `code`.
int set_error(int code, const std::string& msg);
// Converts a CUDA status into AOAKV_ERR_CUDA with context, or AOAKV_OK.
int cuda_status(cudaError_t st, const char* what);
// Device pointer of the library's device-side error word on the current
// device (looked up once per device).
int* dev_error_ptr();
// Number of SMs of the current device (cached per device).
int num_sms();

#define AOAKV_CHECK_ARG(cond, msg)                                   \
  do {                                                               \
    if (!(cond)) return ::aoakv::set_error(AOAKV_ERR_INVALID_ARG, msg); \
  } while (0)

// NVTX range around a C-ABI call, so a profiler's timeline names every
// library call (the reference wraps each stage in NVTX ranges,
// QuestAttention.py:87-176); with no tool attached the calls do nothing.
struct NvtxRange {
  explicit NvtxRange(const char* name) { nvtxRangePushA(name); }
  ~NvtxRange() { nvtxRangePop(); }
  NvtxRange(const NvtxRange&) = delete;
  NvtxRange& operator=(const NvtxRange&) = delete;
};
#define AOAKV_NVTX(name) ::aoakv::NvtxRange aoakv_nvtx_range_(name)

#define AOAKV_CUDA_TRY(expr, what)                                   \
  do {                                                               \
    cudaError_t _st = (expr);                                        \
    if (_st != cudaSuccess) return ::aoakv::cuda_status(_st, what);  \
  } while (0)

// --------------------------------------------------------------- device side
// First device error wins; later ones are dropped.
__device__ __forceinline__ void raise_dev_error(int* err, int code) {
  if (err) atomicCAS(err, 0, code);
}

// 16-byte streaming load that bypasses L1 (data read exactly once).
__device__ __forceinline__ uint4 ld_stream_u4(const void* p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}

__device__ __forceinline__ void u4_to_f8(const uint4& u, float f[8]) {
  const __half2* h = reinterpret_cast<const __half2*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    float2 t = __half22float2(h[i]);
    f[2 * i] = t.x;
    f[2 * i + 1] = t.y;
  }
}

// Monotone map float -> uint32: a > b  <=>  key(a) > key(b) and -0 == +0
// (IEEE equality, as torch.topk compares); NaN -> 0, which ranks below
// -inf (key 0x007fffff).
__device__ __forceinline__ uint32_t float_to_key(float x) {
  uint32_t u = __float_as_uint(x);
  if ((u & 0x7f800000u) == 0x7f800000u && (u & 0x007fffffu)) return 0u;
  if (u == 0x80000000u) u = 0u;
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

__device__ __forceinline__ float key_to_float(uint32_t k) {
  uint32_t u = (k & 0x80000000u) ? (k & 0x7fffffffu) : ~k;
  return __uint_as_float(u);
}

// ------------------------------------------------- mbarrier + TMA (sm_90+)
__device__ __forceinline__ uint32_t smem_addr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// The dynamic shared memory base advanced to the next multiple of Align
// bytes. Offsetting the __shared__ array itself (instead of rounding the
// address as an integer) keeps the pointer's state space visible to the
// compiler, so accesses through it stay shared-memory instructions rather
// than generic ones.
template <uint32_t Align>
__device__ __forceinline__ uint8_t* align_smem(uint8_t* base) {
  const uint32_t a = smem_addr(base);
  return base + (((a + Align - 1u) & ~(Align - 1u)) - a);
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)),
               "r"(count));
}

__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar,
                                                      uint32_t bytes) {
  asm volatile(
      "mbarrier.arrive.expect_tx.release.cta.shared::cta.b64 _, [%0], %1;" ::"r"(
          smem_addr(bar)),
      "r"(bytes)
      : "memory");
}

// Plain arrival (no transaction bytes): completes a phase expected by 1 arrival.
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.release.cta.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar))
               : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cta.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_addr(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait on an mbarrier phase. Returns false (and records
// AOAKV_DEV_ERR_TIMEOUT) if the phase did not complete within ~2^26 polls.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar,
                                                  uint32_t parity, int* err) {
  for (uint32_t i = 0; i < (1u << 26); ++i) {
    if (mbar_try_wait(bar, parity)) return true;
    if (i > 64) __nanosleep(32);
  }
  raise_dev_error(err, AOAKV_DEV_ERR_TIMEOUT);
  return false;
}

// Rotate-half RoPE of one channel pair: x0 is channel j < D/2, x1 channel
// j + D/2, at position pos; angle pos * rcp_scale * 2^(log2_rcp_theta *
// 2j/D) in fp32, accurate sincosf, each product and sum rounded once (no
// fused multiply-add), results rounded to fp16. The stand-alone RoPE kernel
// and the fused step share it, so both give the same bits.
__device__ __forceinline__ void rope_pair(float x0, float x1, int j, int D, float pos,
                                          float rcp_scale, float log2_rcp_theta, __half* o0,
                                          __half* o1) {
  const float f = __fmul_rn(rcp_scale, exp2f(__fmul_rn(log2_rcp_theta,
                                                        __fdiv_rn(2.f * j, static_cast<float>(D)))));
  float s, c;
  sincosf(__fmul_rn(pos, f), &s, &c);
  *o0 = __float2half_rn(__fadd_rn(__fmul_rn(x0, c), -__fmul_rn(x1, s)));
  *o1 = __float2half_rn(__fadd_rn(__fmul_rn(x1, c), __fmul_rn(x0, s)));
}

// Words exchanged with other GPUs through their memory (peer pointers over
// NVLink) carry their own epoch: a 64-bit {value, epoch} store is single-copy
// atomic, so a reader that sees the expected epoch also sees the value, and
// no fence or flag is needed. Relaxed at system scope; the wait gives up
// (AOAKV_DEV_ERR_TIMEOUT, returns the stale word) after about 0.1 s.
__device__ __forceinline__ void tagged_store_sys(uint64_t* p, uint32_t value, uint32_t epoch) {
  const uint64_t w = static_cast<uint64_t>(value) | (static_cast<uint64_t>(epoch) << 32);
  asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(w) : "memory");
}
// A pair of tagged words in one 16-byte access (each 8-byte half is still
// single-copy atomic on its own; volatile global accesses are relaxed at
// system scope). p is 16-byte aligned.
__device__ __forceinline__ void tagged_store2_sys(uint64_t* p, uint32_t v0, uint32_t v1,
                                                  uint32_t epoch) {
  const uint64_t e = static_cast<uint64_t>(epoch) << 32;
  asm volatile("st.volatile.global.v2.u64 [%0], {%1, %2};" ::"l"(p), "l"(e | v0), "l"(e | v1)
               : "memory");
}
__device__ __forceinline__ uint2 tagged_wait2_sys(const uint64_t* p, uint32_t epoch, int* err) {
  uint64_t w0 = 0, w1 = 0;
  for (uint32_t i = 0; i < (1u << 20); ++i) {
    asm volatile("ld.volatile.global.v2.u64 {%0, %1}, [%2];" : "=l"(w0), "=l"(w1) : "l"(p)
                 : "memory");
    if (static_cast<uint32_t>(w0 >> 32) == epoch && static_cast<uint32_t>(w1 >> 32) == epoch)
      return make_uint2(static_cast<uint32_t>(w0), static_cast<uint32_t>(w1));
    if (i > 32) __nanosleep(100);
  }
  raise_dev_error(err, AOAKV_DEV_ERR_TIMEOUT);
  return make_uint2(static_cast<uint32_t>(w0), static_cast<uint32_t>(w1));
}
__device__ __forceinline__ uint32_t tagged_wait_sys(const uint64_t* p, uint32_t epoch, int* err) {
  uint64_t w = 0;
  for (uint32_t i = 0; i < (1u << 20); ++i) {
    asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(w) : "l"(p) : "memory");
    if (static_cast<uint32_t>(w >> 32) == epoch) return static_cast<uint32_t>(w);
    if (i > 32) __nanosleep(100);
  }
  raise_dev_error(err, AOAKV_DEV_ERR_TIMEOUT);
  return static_cast<uint32_t>(w);
}

// 3-D tiled TMA load global -> shared, completion counted on `bar`.
// Coordinates are element indices (c0 innermost).
__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map,
                                            int c0, int c1, int c2,
                                            uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::"
      "bytes [%0], [%1, {%2, %3, %4}], [%5];" ::"r"(smem_addr(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2),
      "r"(smem_addr(bar))
      : "memory");
}

// 1-D bulk copy global -> shared (both 16-byte aligned, bytes % 16 == 0),
// completion counted on `bar`.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes,
                                         uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::
          "r"(smem_addr(dst)),
      "l"(reinterpret_cast<uint64_t>(src)), "r"(bytes), "r"(smem_addr(bar))
      : "memory");
}

// Orders this thread's earlier generic shared-memory accesses before its
// later async-proxy (TMA / bulk copy) writes to shared memory.
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// Same ordering for every state space (global data written by this grid
// before a TMA load reads it, shared tiles reused by the next TMA).
__device__ __forceinline__ void fence_proxy_async() {
  asm volatile("fence.proxy.async;" ::: "memory");
}

__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map))
               : "memory");
}

// Programmatic dependent launch: wait for the previous kernel in the stream
// (no-op when launched without the PDL attribute) / allow the next to start.
__device__ __forceinline__ void pdl_wait() {
  asm volatile("griddepcontrol.wait;" ::: "memory");
}
__device__ __forceinline__ void pdl_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

}  // namespace aoakv
