// Host-side launch helpers shared between the stand-alone entry points and
// the per-layer step.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

namespace aoakv {

struct DecodeArgs;
struct EstimateArgs;
struct TopkArgs;

// Chunking of a split-KV decode: slots per CTA and CTAs per head, chosen so
// the grid covers ~4 CTAs per SM with at most kDecMaxChunk slots each.
struct DecodePlan {
  int chunk_pages;
  int n_chunks;
  size_t smem;
};

DecodePlan plan_decode(int H, int n_slots, int D, int P);
size_t decode_ws_bytes(int H, int D, int max_slots);
void carve_decode_ws(void* ws, int H, int D, int max_slots, DecodeArgs& a);
int check_decode_shape(int H, int D, int P, int kv_cap, int layout);
// 3-D tensor map over one layer's KV pages: dims {D, H, cap*2*P}, box {D,1,P}.
int make_kv_tmap(CUtensorMap* map, const void* kv, int H, int D, int P, int cap);
// The same view with box {64, 1, P} and the 128-byte swizzle: a page's K (or
// V) rows arrive as D/64 tiles of P rows x 128 bytes, 16-byte units of row r
// permuted by r mod 8 (bank-conflict-free 8x8 matrix loads).
int make_kv_tmap_sw128(CUtensorMap* map, const void* kv, int H, int D, int P, int cap);
// 3-D tensor map over rows [rows, H, D] fp16 (q of a prefill): box {64, 1,
// 128} with the 128-byte swizzle, one 64-channel block of 128 rows.
int make_q_tmap_sw128(CUtensorMap* map, const void* q, int H, int D, int rows);
// 3-D tensor map over one layer's metadata pages: dims {D, H, meta_cap*2*P},
// box {D, box_heads, 1} (one page's max or min block for box_heads heads).
int make_meta_tmap(CUtensorMap* map, const void* meta, int H, int D, int P, int meta_cap,
                   int box_heads);

int launch_decode(const DecodeArgs& a, const CUtensorMap& tmap, int D,
                  const DecodePlan& pl, cudaStream_t s, bool pdl);
int launch_estimate(const EstimateArgs& a, int D, cudaStream_t s);
// GQA: a.H = KV heads, a.q holds a.H * group query heads (gqa.cu).
int launch_gqa_estimate(const EstimateArgs& a, int D, int group, cudaStream_t s);
int launch_topk(const TopkArgs& a, int rows, cudaStream_t s, bool pdl);

}  // namespace aoakv
