// RMSNorm: aoakv_rms_norm.
//
// Reference: quest._kernels.rms_norm_forward (ops/csrc/rms_norm.cu, bound
// in bsk_ops.cu; py utils/__init__.py:54-67). Per row of n fp16 values:
//   r = 1 / sqrt(sum_i x_i^2 / n + eps)   (fp32)
//   out_i = fp16(x_i * r * w_i)
// n must be a multiple of 8 (16-byte vectors), as in the reference.
#include <cmath>

#include "common.cuh"

namespace aoakv {
namespace {

constexpr int kNormThreads = 256;

__global__ void __launch_bounds__(kNormThreads) rms_norm_kernel(const __half* in,
                                                                const __half* w, __half* out,
                                                                int n, float eps) {
  __shared__ float warp_sum[kNormThreads / 32];
  const uint4* x = reinterpret_cast<const uint4*>(in + static_cast<size_t>(blockIdx.x) * n);
  uint4* y = reinterpret_cast<uint4*>(out + static_cast<size_t>(blockIdx.x) * n);
  const uint4* g = reinterpret_cast<const uint4*>(w);
  const int n8 = n / 8;
  float acc = 0.f;
  for (int i = threadIdx.x; i < n8; i += blockDim.x) {
    float f[8];
    u4_to_f8(x[i], f);
#pragma unroll
    for (int j = 0; j < 8; ++j) acc = fmaf(f[j], f[j], acc);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
  if ((threadIdx.x & 31) == 0) warp_sum[threadIdx.x >> 5] = acc;
  __syncthreads();
  float tot = 0.f;
#pragma unroll
  for (int k = 0; k < kNormThreads / 32; ++k) tot += warp_sum[k];
  const float r = rsqrtf(tot / n + eps);
  for (int i = threadIdx.x; i < n8; i += blockDim.x) {
    float f[8], gw[8];
    u4_to_f8(x[i], f);
    u4_to_f8(g[i], gw);
    __half2 h[4];
#pragma unroll
    for (int j = 0; j < 4; ++j)
      h[j] = __floats2half2_rn(f[2 * j] * r * gw[2 * j], f[2 * j + 1] * r * gw[2 * j + 1]);
    y[i] = *reinterpret_cast<const uint4*>(h);
  }
}

}  // namespace
}  // namespace aoakv

using namespace aoakv;

extern "C" int aoakv_rms_norm(const void* input, const void* weight, void* out, int32_t rows,
                              int32_t columns, float epsilon, void* stream) {
  AOAKV_NVTX("aoakv_rms_norm");
  AOAKV_CHECK_ARG(input && weight && out, "rms_norm: NULL pointer argument");
  AOAKV_CHECK_ARG(rows >= 0 && columns >= 8 && columns % 8 == 0,
                  "rms_norm: columns must be a positive multiple of 8");
  AOAKV_CHECK_ARG(epsilon >= 0.f, "rms_norm: epsilon must be >= 0");
  AOAKV_CHECK_ARG((reinterpret_cast<uintptr_t>(input) | reinterpret_cast<uintptr_t>(weight) |
                   reinterpret_cast<uintptr_t>(out)) % 16 == 0,
                  "rms_norm: buffers must be 16-byte aligned");
  if (rows == 0) return AOAKV_OK;
  rms_norm_kernel<<<rows, kNormThreads, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const __half*>(input), static_cast<const __half*>(weight),
      static_cast<__half*>(out), columns, epsilon);
  AOAKV_CUDA_TRY(cudaGetLastError(), "rms_norm launch");
  return AOAKV_OK;
}
