// Fifth-generation tensor core (tcgen05) building blocks for sm_100a:
// tensor-memory allocation, shared-memory operand descriptors, the f16 MMA
// with fp32 accumulation in tensor memory, its completion signal, and
// tensor-memory loads and stores of one warp's 32 lanes.
#pragma once

#include <stdint.h>

#include "common.cuh"

namespace aoakv {

// Operand descriptor of a shared-memory tile in the 128-byte-swizzle
// canonical layout: rows of 128 bytes, 8-row groups of 1024 bytes, 16-byte
// unit u of row r stored at unit u ^ (r % 8). Fields: start address >> 4
// (bits 0-13), leading byte offset >> 4 (16-29), stride byte offset >> 4
// (32-45), descriptor version 1 (46-47), layout 2 = 128-byte swizzle (61-63).
//   K-major operand (rows = M or N, 64 K-elements per 128-byte row): sbo =
//   1024 (next 8 rows); lbo is not used while one MMA's K (16 elements, 32
//   bytes) stays inside the row; a K step advances the start by 32 bytes.
//   MN-major operand (rows = K, 64 M/N-elements per row): sbo = 1024 (next 8
//   K rows), lbo = byte distance to the next 64 M/N elements.
__device__ __forceinline__ uint64_t umma_desc_sw128(uint32_t saddr, uint32_t lbo,
                                                    uint32_t sbo) {
  return static_cast<uint64_t>((saddr >> 4) & 0x3fffu) |
         (static_cast<uint64_t>((lbo >> 4) & 0x3fffu) << 16) |
         (static_cast<uint64_t>((sbo >> 4) & 0x3fffu) << 32) | (1ull << 46) | (2ull << 61);
}

// Instruction descriptor of tcgen05.mma kind::f16: fp16 A and B, fp32
// accumulator (bits 4-5 = 1), A / B major (bits 15 / 16: 0 = K-major, 1 =
// MN-major), N >> 3 (bits 17-22), M >> 4 (bits 24-28).
__host__ __device__ constexpr uint32_t umma_idesc_f16_f32(int M, int N, int a_mn, int b_mn) {
  return (1u << 4) | (static_cast<uint32_t>(a_mn) << 15) |
         (static_cast<uint32_t>(b_mn) << 16) | (static_cast<uint32_t>(N >> 3) << 17) |
         (static_cast<uint32_t>(M >> 4) << 24);
}

// D[tmem] (+)= A[smem] * B[smem]^T, issued by one thread.
__device__ __forceinline__ void umma_f16_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                            uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// D[tmem] (+)= A[tmem] * B[smem]^T: A (M x K, K-major) sits in tensor
// memory, row i in lane i, two 16-bit elements per 32-bit column (element k
// in column k / 2, the even element in the low half).
__device__ __forceinline__ void umma_f16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc,
                                            uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrives once on `bar` when every tcgen05 operation this thread issued so
// far has completed.
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
          smem_addr(bar))
      : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// Whole-warp tensor-memory allocation of `cols` columns (a power of two >=
// 32); the base address lands in shared memory at `slot`.
__device__ __forceinline__ void tmem_alloc(uint32_t* slot, uint32_t cols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   smem_addr(slot)),
               "r"(cols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t base, uint32_t cols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(base), "r"(cols)
               : "memory");
}

#define AOAKV_R8(i) "=r"(v[i]), "=r"(v[i + 1]), "=r"(v[i + 2]), "=r"(v[i + 3]), \
                    "=r"(v[i + 4]), "=r"(v[i + 5]), "=r"(v[i + 6]), "=r"(v[i + 7])
#define AOAKV_W8(i) "r"(v[i]), "r"(v[i + 1]), "r"(v[i + 2]), "r"(v[i + 3]), \
                    "r"(v[i + 4]), "r"(v[i + 5]), "r"(v[i + 6]), "r"(v[i + 7])

// 32 consecutive fp32 columns of this thread's lane (warp w reads lanes
// 32 (w % 4) ..; taddr carries the lane in bits 16-31). The load and its
// wait sit in one statement, so no use of v can be scheduled before the
// data has arrived.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&v)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, "
      "[%32];\n\t"
      "tcgen05.wait::ld.sync.aligned;"
      : AOAKV_R8(0), AOAKV_R8(8), AOAKV_R8(16), AOAKV_R8(24)
      : "r"(taddr)
      : "memory");
}

// 64 consecutive fp32 columns of this thread's lane in one load.
__device__ __forceinline__ void tmem_ld64(uint32_t taddr, uint32_t (&v)[64]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x64.b32 {"
      "%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, "
      "%32, %33, %34, %35, %36, %37, %38, %39, %40, %41, %42, %43, %44, %45, %46, %47, "
      "%48, %49, %50, %51, %52, %53, %54, %55, %56, %57, %58, %59, %60, %61, %62, %63"
      "}, [%64];\n\t"
      "tcgen05.wait::ld.sync.aligned;"
      : AOAKV_R8(0), AOAKV_R8(8), AOAKV_R8(16), AOAKV_R8(24), AOAKV_R8(32), AOAKV_R8(40), AOAKV_R8(48), AOAKV_R8(56)
      : "r"(taddr)
      : "memory");
}

// 128 consecutive fp32 columns of this thread's lane in one load.
__device__ __forceinline__ void tmem_ld128(uint32_t taddr, uint32_t (&v)[128]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x128.b32 {"
      "%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, "
      "%32, %33, %34, %35, %36, %37, %38, %39, %40, %41, %42, %43, %44, %45, %46, %47, "
      "%48, %49, %50, %51, %52, %53, %54, %55, %56, %57, %58, %59, %60, %61, %62, %63, "
      "%64, %65, %66, %67, %68, %69, %70, %71, %72, %73, %74, %75, %76, %77, %78, %79, "
      "%80, %81, %82, %83, %84, %85, %86, %87, %88, %89, %90, %91, %92, %93, %94, %95, "
      "%96, %97, %98, %99, %100, %101, %102, %103, %104, %105, %106, %107, %108, %109, %110, %111, "
      "%112, %113, %114, %115, %116, %117, %118, %119, %120, %121, %122, %123, %124, %125, %126, %127"
      "}, [%128];\n\t"
      "tcgen05.wait::ld.sync.aligned;"
      : AOAKV_R8(0), AOAKV_R8(8), AOAKV_R8(16), AOAKV_R8(24), AOAKV_R8(32), AOAKV_R8(40), AOAKV_R8(48), AOAKV_R8(56), AOAKV_R8(64), AOAKV_R8(72), AOAKV_R8(80), AOAKV_R8(88), AOAKV_R8(96), AOAKV_R8(104), AOAKV_R8(112), AOAKV_R8(120)
      : "r"(taddr)
      : "memory");
}

// Stores 32 columns of this thread's lane; completes before it returns.
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&v)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16, "
      "%17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};\n\t"
      "tcgen05.wait::st.sync.aligned;" ::"r"(taddr),
      AOAKV_W8(0), AOAKV_W8(8), AOAKV_W8(16), AOAKV_W8(24)
      : "memory");
}

#undef AOAKV_R8
#undef AOAKV_W8

// 2^x on the special-function unit (flush-to-zero; 2^-inf = 0).
__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

}  // namespace aoakv
