// Log-sum-exp merge of partial decode states: aoakv_merge_states.
//
// Reference: the split-KV merge FlashInfer's VariableLengthMergeStates runs
// after BatchDecodeWithPagedKVCacheKernel (call site decode_attn.cuh:1035-1043),
// restated from its definition. For head h over parts g with partial output
// o_g (already normalised by its own softmax denominator) and
// lse_g = ln(sum of exp(scores)) of that part:
//   m = max_g lse_g,  w_g = exp(lse_g - m),
//   o = sum_g w_g o_g / sum_g w_g,  lse = m + ln(sum_g w_g).
// A part with lse = -inf (no tokens) contributes nothing; a head with no
// tokens in any part gets o = 0 and lse = -inf. Used by the page-range
// sharded step, where each GPU decodes the selected pages it owns; that
// step's global -> local page-id map (aoakv_map_pages) lives here too.
#include <cmath>

#include "common.cuh"
#include "step_cluster.h"

namespace aoakv {
namespace {

__global__ void merge_states_kernel(const float* o_parts, const float* lse_parts, int G, int H,
                                    int D, __half* o, float* lse_out) {
  const int h = blockIdx.x;
  float m = -INFINITY;
  for (int g = 0; g < G; ++g) m = fmaxf(m, lse_parts[static_cast<size_t>(g) * H + h]);
  for (int d = threadIdx.x; d < D; d += blockDim.x) {
    float acc = 0.f, sum = 0.f;
    if (m != -INFINITY) {
      for (int g = 0; g < G; ++g) {
        const float l = lse_parts[static_cast<size_t>(g) * H + h];
        if (l == -INFINITY) continue;
        const float w = expf(l - m);
        sum += w;
        acc += w * o_parts[(static_cast<size_t>(g) * H + h) * D + d];
      }
    }
    o[static_cast<size_t>(h) * D + d] = __float2half_rn(sum > 0.f ? acc / sum : 0.f);
    if (lse_out && d == 0) lse_out[h] = sum > 0.f ? m + logf(sum) : -INFINITY;
  }
}

// The same merge over states packed as the sharded step exchanges them:
// states[g, h] = {o[D], lse}.
__global__ void merge_packed_kernel(const float* states, int G, int H, int D, __half* o) {
  const int h = blockIdx.x;
  const size_t row = static_cast<size_t>(D) + 1;
  float m = -INFINITY;
  for (int g = 0; g < G; ++g) m = fmaxf(m, states[(static_cast<size_t>(g) * H + h) * row + D]);
  for (int d = threadIdx.x; d < D; d += blockDim.x) {
    float acc = 0.f, sum = 0.f;
    if (m != -INFINITY) {
      for (int g = 0; g < G; ++g) {
        const float* st = states + (static_cast<size_t>(g) * H + h) * row;
        const float l = st[D];
        if (l == -INFINITY) continue;
        const float w = expf(l - m);
        sum += w;
        acc += w * st[d];
      }
    }
    o[static_cast<size_t>(h) * D + d] = __float2half_rn(sum > 0.f ? acc / sum : 0.f);
  }
}

// The merge of a sharded step whose states arrive in this GPU's mailbox
// (tagged words stored by every GPU's finish pass): head blockIdx.x waits for
// this exchange's epoch on every word it reads, merges, and the last head to
// finish closes the exchange (ep).
__global__ void merge_mailbox_kernel(ShardMail m, int world, int rank, int H, int D,
                                     int proposals, __half* o, int* err) {
  const int h = blockIdx.x;
  uint32_t* ep = reinterpret_cast<uint32_t*>(m.base[rank] + m.ep_off);
  const uint32_t epoch = __ldcg(ep + 1) + 1u;
  const uint64_t* box = reinterpret_cast<const uint64_t*>(m.base[rank] + m.state_off);
  const size_t row = static_cast<size_t>(D) + 1;
  __shared__ float lse_s[8];
  if (threadIdx.x < world)
    lse_s[threadIdx.x] = __uint_as_float(
        tagged_wait_sys(box + (static_cast<size_t>(threadIdx.x) * H + h) * row + D, epoch, err));
  __syncthreads();
  float mx = -INFINITY;
  for (int g = 0; g < world; ++g) mx = fmaxf(mx, lse_s[g]);
  for (int d = threadIdx.x; d < D; d += blockDim.x) {
    float acc = 0.f, sum = 0.f;
    if (mx != -INFINITY) {
      for (int g = 0; g < world; ++g) {
        const float l = lse_s[g];
        if (l == -INFINITY) continue;
        const float w = expf(l - mx);
        sum += w;
        acc += w * __uint_as_float(
                       tagged_wait_sys(box + (static_cast<size_t>(g) * H + h) * row + d, epoch, err));
      }
    }
    o[static_cast<size_t>(h) * D + d] = __float2half_rn(sum > 0.f ? acc / sum : 0.f);
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    if (atomicAdd(ep + 2, 1u) == static_cast<uint32_t>(H) - 1u) {  // every head read ep
      ep[2] = 0u;
      if (proposals) ep[0] += 1u;
      ep[1] += 1u;
      __threadfence();
    }
  }
}

__global__ void map_pages_kernel(const int32_t* ids, int64_t count, int32_t lo, int32_t n_local,
                                 const int32_t* local, int32_t* out) {
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < count;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int32_t r = ids[i] - lo;
    out[i] = (r >= 0 && r < n_local) ? __ldg(local + r) : -1;
  }
}

}  // namespace
}  // namespace aoakv

using namespace aoakv;

extern "C" int aoakv_map_pages(const int32_t* global_ids, int64_t count, int32_t page_lo,
                               int32_t n_local, const int32_t* local_kv_indices, int32_t* out,
                               void* stream) {
  AOAKV_NVTX("aoakv_map_pages");
  AOAKV_CHECK_ARG(global_ids && local_kv_indices && out, "map_pages: NULL pointer argument");
  AOAKV_CHECK_ARG(count >= 0 && n_local >= 0, "map_pages: bad sizes");
  if (count == 0) return AOAKV_OK;
  const int threads = 256;
  const int64_t blocks = (count + threads - 1) / threads;
  map_pages_kernel<<<static_cast<int>(blocks < 1024 ? blocks : 1024), threads, 0,
                     static_cast<cudaStream_t>(stream)>>>(global_ids, count, page_lo, n_local,
                                                          local_kv_indices, out);
  AOAKV_CUDA_TRY(cudaGetLastError(), "map_pages launch");
  return AOAKV_OK;
}

extern "C" int aoakv_merge_states(const float* o_parts, const float* lse_parts,
                                  int32_t num_parts, int32_t num_heads, int32_t head_dim,
                                  void* o, float* lse_out, void* stream) {
  AOAKV_NVTX("aoakv_merge_states");
  AOAKV_CHECK_ARG(o_parts && lse_parts && o, "merge_states: NULL pointer argument");
  AOAKV_CHECK_ARG(num_parts >= 1 && num_heads >= 1 && head_dim >= 1 && head_dim <= 1024,
                  "merge_states: bad sizes");
  const int threads = head_dim < 128 ? ((head_dim + 31) / 32) * 32 : 128;
  merge_states_kernel<<<num_heads, threads, 0, static_cast<cudaStream_t>(stream)>>>(
      o_parts, lse_parts, num_parts, num_heads, head_dim, static_cast<__half*>(o), lse_out);
  AOAKV_CUDA_TRY(cudaGetLastError(), "merge_states launch");
  return AOAKV_OK;
}

extern "C" int aoakv_merge_packed_states(const float* states, int32_t num_parts,
                                         int32_t num_heads, int32_t head_dim, void* o,
                                         void* stream) {
  AOAKV_NVTX("aoakv_merge_packed_states");
  AOAKV_CHECK_ARG(states && o, "merge_packed_states: NULL pointer argument");
  AOAKV_CHECK_ARG(num_parts >= 1 && num_heads >= 1 && head_dim >= 1 && head_dim <= 1024,
                  "merge_packed_states: bad sizes");
  const int threads = head_dim < 128 ? ((head_dim + 31) / 32) * 32 : 128;
  merge_packed_kernel<<<num_heads, threads, 0, static_cast<cudaStream_t>(stream)>>>(
      states, num_parts, num_heads, head_dim, static_cast<__half*>(o));
  AOAKV_CUDA_TRY(cudaGetLastError(), "merge_packed_states launch");
  return AOAKV_OK;
}

namespace aoakv {
int launch_merge_mailbox(const ShardMail& m, int world, int rank, int H, int D, int proposals,
                         void* o, cudaStream_t s) {
  const int threads = D < 128 ? ((D + 31) / 32) * 32 : 128;
  merge_mailbox_kernel<<<H, threads, 0, s>>>(m, world, rank, H, D, proposals,
                                             static_cast<__half*>(o), dev_error_ptr());
  AOAKV_CUDA_TRY(cudaGetLastError(), "merge (mailbox) launch");
  return AOAKV_OK;
}
}  // namespace aoakv
