// RoPE in place on q and k (NHD [seq, heads, head_dim], fp16):
// aoakv_apply_rope_in_place.
//
// Reference: quest._kernels.apply_rope_in_place (page.cu:224-264 ->
// QKApplyRotaryInPlace, decode_page.cuh:786-869, with FlashInfer's
// vec_apply_llama_rope). For token t (position p = past_kv_len + t) and
// channel i of a head of dimension D, with j = i mod D/2:
//   f_i = (1 / rope_scale) * (1 / rope_theta)^(2j / D),   a = p * f_i
//   out_i = x_i cos a - x_{i+D/2} sin a   (i <  D/2)
//   out_i = x_i cos a + x_{i-D/2} sin a   (i >= D/2)
// the rotate-half ("llama") convention, computed in fp32 with the
// accurate sincosf (the reference's fast intrinsics lose accuracy at large
// angles) and stored back to fp16.
#include <cmath>

#include "common.cuh"

namespace aoakv {
namespace {

// One warp per (token, head) row of q or k; lane l owns channel pairs
// (j, j + D/2) for j = l, l + 32, ... < D/2.
__global__ void rope_kernel(__half* q, __half* k, int seq_len, int past_kv_len, int H, int D,
                            float rcp_scale, float log2_rcp_theta) {
  const int lane = threadIdx.x & 31;
  const int64_t row = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int64_t rows = static_cast<int64_t>(seq_len) * H;
  if (row >= 2 * rows) return;
  __half* x = (row < rows ? q : k) + (row % rows) * D;
  const int t = static_cast<int>((row % rows) / H);
  const float pos = static_cast<float>(past_kv_len + t);
  const int half = D / 2;
  for (int j = lane; j < half; j += 32)
    rope_pair(__half2float(x[j]), __half2float(x[j + half]), j, D, pos, rcp_scale,
              log2_rcp_theta, &x[j], &x[j + half]);
}

}  // namespace
}  // namespace aoakv

using namespace aoakv;

extern "C" int aoakv_apply_rope_in_place(void* q, void* k, int32_t seq_len, int32_t past_kv_len,
                                         int32_t num_heads, int32_t head_dim, float rope_scale,
                                         float rope_theta, void* stream) {
  AOAKV_NVTX("aoakv_apply_rope_in_place");
  AOAKV_CHECK_ARG(q && k, "rope: NULL pointer argument");
  AOAKV_CHECK_ARG(seq_len >= 0 && past_kv_len >= 0 && num_heads >= 1, "rope: bad sizes");
  AOAKV_CHECK_ARG(head_dim >= 2 && head_dim % 2 == 0 && head_dim <= 1024,
                  "rope: head_dim must be even and <= 1024");
  AOAKV_CHECK_ARG(rope_scale > 0.f && rope_theta > 0.f, "rope: scale and theta must be > 0");
  if (seq_len == 0) return AOAKV_OK;
  const int64_t rows = 2LL * seq_len * num_heads;
  const int warps = 8;
  const int64_t blocks = (rows + warps - 1) / warps;
  AOAKV_CHECK_ARG(blocks <= 0x7fffffffLL, "rope: too many rows");
  rope_kernel<<<static_cast<unsigned>(blocks), warps * 32, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<__half*>(q), static_cast<__half*>(k), seq_len, past_kv_len, num_heads, head_dim,
      1.f / rope_scale, std::log2(1.f / rope_theta));
  AOAKV_CUDA_TRY(cudaGetLastError(), "rope launch");
  return AOAKV_OK;
}
