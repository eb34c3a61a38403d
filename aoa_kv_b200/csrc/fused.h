// Arguments and host helpers of the fused per-layer step kernel.
#pragma once

#include "decode.cuh"
#include "estimate.cuh"

namespace aoakv {

constexpr int kFusedThreads = 512;  // threads per CTA of the fused step kernel

struct FusedArgs {
  const __half* k_new;          // [H, D] new token
  const __half* v_new;
  __half* kv;                   // [kv_cap, 2, P, H, D]
  const int32_t* kv_indices;    // [n_pages] physical ids, last page last
  int n_pages, last_len, kv_cap;
  __half* meta;                 // [meta_cap, 2, P, H, D]
  const int32_t* meta_indices;
  int meta_cap;
  __half* vlog;                 // [kv_cap, H]
  int H, P;
  int k_sel;                    // pages chosen by top-k per head
  int sink;
  int32_t* sel;                 // [H, k_sel] workspace
  uint32_t* sync;               // zeroed sync words, see step_fused.cu
  int32_t* selected_out;        // optional [H, sel_cols]
  int sel_cols;
  int est_tma;                  // 1: TMA-pipelined scorer (estimate_pages_tmap)
  int* err;
  EstimateArgs est;             // out = fp32 scores [H, out_stride]
  DecodeArgs dec;               // indices = sel
};

// Returns 1 and the launch shape if the fused kernel can run this problem
// with every CTA co-resident; max_grid > 0 caps the grid.
int fused_supported(int H, int D, int P, int n_score, int k_sel, int* grid, size_t* smem,
                    int* chunk, int* n_chunks, int max_grid = 0);
size_t fused_sync_bytes(int H);
// The pipelined step kernel (step_pipe.cu): same arguments; its sync words
// (1 + 2 * H / 8) fit in fused_sync_bytes(H).
int pipe_supported(int H, int D, int P, int n_score, int k_sel, int* grid, size_t* smem,
                   int* chunk, int* n_chunks);
int pipe_group_heads();
int launch_pipe(const CUtensorMap& tmap, const CUtensorMap& gmap, const FusedArgs& f, int D,
                int grid, size_t smem, cudaStream_t s);
int launch_fused(const CUtensorMap& tmap, const CUtensorMap& mtmap, const FusedArgs& f, int D,
                 int grid, size_t smem, cudaStream_t s);

}  // namespace aoakv
