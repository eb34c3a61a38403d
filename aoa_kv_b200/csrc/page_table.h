// Device-resident page table: the page lists, counts and free lists of a
// set of sequences in one caller-provided device buffer (page_table.cu).
#pragma once

#include <stddef.h>
#include <stdint.h>

namespace aoakv {

// Offsets (in int32 words) of the regions of a page-table buffer.
struct PageTableLayout {
  int R, M, Mm, P, cap, mcap;   // sequences, KV pages / metadata pages per sequence, page
                                // size, pool capacities
  size_t kv_top, meta_top;      // free-stack heights
  size_t kv_start, kv_end, last_len, seq_len, meta_start, meta_count;  // [R] each
  size_t kv_indices, meta_indices;  // [R * M], [R * Mm]
  size_t kv_free, meta_free;        // [cap], [mcap]
  size_t words;
};

PageTableLayout page_table_layout(int R, int M, int cap, int mcap, int P);

struct PageTable {
  int32_t* buf;
  PageTableLayout L;
};

}  // namespace aoakv
