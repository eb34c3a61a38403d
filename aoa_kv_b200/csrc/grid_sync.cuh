// Bounded grid-level waits shared by the fused step kernels (all CTAs of
// those kernels are co-resident: cooperative launch).
#pragma once

#include "common.cuh"

namespace aoakv {

constexpr uint64_t kGridWaitNs = 1000000000ull;  // 1 s

__device__ __forceinline__ uint32_t ld_acquire(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Thread 0 spins until *p >= target or limit_ns (~1 s by default) has
// passed; the result is broadcast through *ok_s. Returns false on timeout
// (AOAKV_DEV_ERR_TIMEOUT recorded). Every thread of the CTA calls it.
__device__ __forceinline__ bool cta_wait_geq(const uint32_t* p, uint32_t target, int* ok_s,
                                             int* err, uint64_t limit_ns = kGridWaitNs) {
  if (threadIdx.x == 0) {
    int ok = 1;
    if (ld_acquire(p) < target) {
      const uint64_t t0 = global_ns();
      uint32_t it = 0;
      while (ld_acquire(p) < target) {
        if (++it > 2048) __nanosleep(it < 8192 ? 64 : 256);  // each poll is a round trip
        if ((it & 255u) == 0 && global_ns() - t0 > limit_ns) {
          raise_dev_error(err, AOAKV_DEV_ERR_TIMEOUT);
          ok = 0;
          break;
        }
      }
    }
    __threadfence();
    *ok_s = ok;
  }
  __syncthreads();
  return *ok_s != 0;
}

}  // namespace aoakv
