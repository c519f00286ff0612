// pages.cuh — block-table updates of a paged KV arena.
//
// A paged arena maps each sequence's logical pages to physical pages of a
// per-layer pool through a device block table (one row per sequence, shared
// by all layers). The host allocator decides the mapping; this kernel writes
// the new entries in stream order, so a decode launched after it (which
// waits for it in griddepcontrol.wait) sees them, and a decode launched
// before it still sees the old ones. The updates travel as kernel
// parameters: no host buffer has to outlive the call.
#pragma once

namespace qx {

constexpr int kPageUpdates = 480;  // keeps the parameter block under 4 KB

struct PageUpdates {
  int* table;
  int n;
  int index[kPageUpdates];  // entry of the table (sequence * stride + logical page)
  int page[kPageUpdates];   // physical page
};

__global__ void __launch_bounds__(128) qx_page_table_kernel(const __grid_constant__ PageUpdates u) {
  for (int i = threadIdx.x; i < u.n; i += 128) u.table[u.index[i]] = u.page[i];
}

}  // namespace qx
