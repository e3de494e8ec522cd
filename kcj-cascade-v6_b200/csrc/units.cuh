// Work units of the batched copy / pack kernels: descriptor i owns units
// [unit_start[i], unit_start[i+1]) of kCopyUnit bytes; each CTA takes one
// contiguous range of units.
#pragma once

#include "common.cuh"

namespace cb {

// Largest i with unit_start[i] <= u (requests with no units are skipped).
CB_D int find_req(const uint32_t *unit_start, int n, uint32_t u) {
  int lo = 0, hi = n - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (unit_start[mid] <= u)
      lo = mid;
    else
      hi = mid - 1;
  }
  return lo;
}

CB_D void cta_unit_range(uint32_t total_units, uint32_t &u0, uint32_t &u1) {
  const uint32_t per = (total_units + gridDim.x - 1) / gridDim.x;
  u0 = blockIdx.x * per;
  u1 = min(total_units, u0 + per);
}

}  // namespace cb
