// Arguments and host helpers of the cluster step kernel (step_cluster.cu):
// the whole per-layer decode step, one thread-block cluster per head.
#pragma once

#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

namespace aoakv {

constexpr int kShardMaxWorld = 8;

// The exchange buffers of a page-range sharded sequence when the GPUs write
// into each other's memory (aoakv_shard_mailbox_*): every rank's mailbox,
// peers' mapped over NVLink, all with the same layout. Per mailbox:
//   cand  [world, H, n_prop, 2] 64-bit words {key | epoch}, {page | epoch}:
//         proposals, sender-major
//   state [world, H, D + 1] 64-bit words {fp32 bits | epoch}: partial states
//   stage [H, n_prop] {key, page}: this GPU's own proposals before they are
//         sent (local)
//   ep[3]: proposal exchanges done, state exchanges done, heads merged in
//          the current exchange (written by this GPU's merge only); the n-th
//          exchange of each kind tags its words with epoch n
struct ShardMail {
  uint8_t* base[kShardMaxWorld];
  uint32_t cand_off, state_off, stage_off, ep_off;
};

struct ClusterStepArgs {
  const __half* q;              // [H, D]
  const __half* k_new;          // [H, D] the new token
  const __half* v_new;
  __half* o;                    // [H, D]
  __half* kv;                   // [kv_cap, 2, P, H, D]
  const int32_t* kv_indices;    // [n_pages] physical ids, last page last
  int n_pages, last_len, kv_cap;
  __half* meta;                 // [meta_cap, 2, P, H, D]
  const int32_t* meta_indices;  // [ceil(n_pages / P)]
  int meta_cap;
  __half* vlog;                 // [kv_cap, H]
  int H, P;
  int k_slots;                  // attended pages, last page included: min(budget, N)
  int sink;                     // page 0 always attended (simulation's `fixed`)
  int mode;                     // AOAKV_SCORE_*
  float two_rsqrt_d;            // 2 / sqrt(D)
  float scale_log2;             // sm_scale * log2(e)
  int32_t* selected_out;        // optional [H, sel_cols]
  int sel_cols;
  int* err;
  // Batched steps (kv_indptr != NULL): request blockIdx.z owns pages
  // kv_indices[kv_indptr[r] .. kv_indptr[r+1]) and metadata pages from
  // meta_indptr[r]; its last page holds last_lens[r] tokens; q, k_new, v_new,
  // o and selected_out advance by one request; k_slots follows from budget.
  const int32_t* kv_indptr;
  const int32_t* meta_indptr;
  const int32_t* last_lens;
  const int32_t* kv_ends;       // optional: request r's pages end at kv_ends[r] (not
                                // kv_indptr[r+1]); then an empty request is skipped silently
  int budget;
  int max_pages;                // a request with more pages (or none) is skipped
  // One sequence split over GPUs by page range (shard != kShardNone). The
  // local pages are global pages page_lo, page_lo + 1, ...; k_slots is the
  // whole sequence's k and n_prop = k - 1 entries travel per (rank, head).
  //   propose: score the local pages (all n_pages - 1 of them; n_pages
  //            counts one page past the local ones when another GPU owns the
  //            last page), keep the local top-n_prop and write them to
  //            cand_out[h, 0..n_prop) as {order key, global page id}, best
  //            first, unused entries {0, 0xffffffff}. No append, no decode.
  //   finish:  rank this GPU's list in cand_in[world, H, n_prop] against
  //            the others, decode the winners it holds (plus the last page,
  //            appending the new token, when owns_last) and write the
  //            partial state state_out[h] = {o[D] normalised, lse (natural
  //            log)}; n_prop == 0: every local page (dense) or only the last.
  int shard;
  int page_lo;
  int n_prop;
  uint2* cand_out;
  const uint2* cand_in;
  int world, rank;
  int owns_last, dense;
  float* state_out;
  // p2p != 0: the exchanges go through `mail` instead of the caller:
  // propose writes each head's list, tagged with the exchange's epoch, into
  // every GPU's mailbox; finish reads the lists from its own mailbox (waiting
  // for the epoch) and writes its tagged state into every mailbox.
  int p2p;
  ShardMail mail;
  // RoPE fused into the step (rope != 0): q and k_new arrive unrotated and
  // are rotated at position rope_pos (< 0: the request's own new-token
  // position, (n_pages - 1) * P + last_len - 1) before use; the rotated q
  // and k_new are written back in place (not by a propose pass).
  int rope, rope_pos;
  float rope_rcp_scale, rope_log2_rcp_theta;
};

enum { kShardNone = 0, kShardPropose = 1, kShardFinish = 2 };

// Sizes the kernel's shared memory is carved for.
struct CsShape {
  int max_local;    // scored pages per CTA
  int max_slots;    // attended pages per head, last page included
};

// Launch shape of the cluster step for one problem size.
struct ClusterPlan {
  int cluster;      // CTAs per head (1, 2, 4 or 8)
  CsShape shape;
  size_t smem;      // dynamic shared memory per CTA
  int waves;        // clusters resident at once vs heads: 1 = one wave
};

// Returns 1 and the plan when the cluster step can run (H heads of head_dim
// D, page size P, up to max_pages pages of which up to max_slots are
// attended, at most max_ctas CTAs when max_ctas > 0); 0 otherwise (the
// caller uses the multi-kernel chain).
// slots_beyond_pages keeps max_slots above max_pages (a page-range shard
// attends up to the whole sequence's k pages, some held by other GPUs).
int cluster_step_plan(int H, int D, int P, int max_pages, int max_slots, int max_ctas,
                      ClusterPlan* plan, bool slots_beyond_pages = false);
// Launches num_requests x H clusters (num_requests > 1 needs a.kv_indptr).
int launch_cluster_step(const ClusterStepArgs& a, const CUtensorMap& kv_map,
                        const CUtensorMap& meta_map, int D, const ClusterPlan& plan,
                        cudaStream_t s, int num_requests = 1);

}  // namespace aoakv
