// Slot validity of the fp16 KV caches (shared by the attention kernels).
#pragma once

#include "common.cuh"

namespace e4b {

// Which cache slots a query at position qp attends (kernels/attsplit.wgsl):
// cachemode 0: linear cache of len slots, the last `window` when window > 0;
// 1: ring of `ring` slots holding the last `window` positions;
// 2: linear cache of len slots, all valid.
struct SlotRule {
  int cachemode, ring, window;
  uint32_t qp, len;
  E4B_DEV uint32_t nslots() const {
    if (cachemode == 1) return min(qp + 1, (uint32_t)ring);
    return len;
  }
  E4B_DEV bool valid(uint32_t t) const {
    if (cachemode == 1) {
      const uint32_t ps = qp - ((qp + (uint32_t)ring - t) % (uint32_t)ring);  // slot t's true position
      return ps <= qp && ps + (uint32_t)window > qp;
    }
    if (t >= len) return false;
    if (cachemode == 0 && window > 0 && len > (uint32_t)window) return t >= len - (uint32_t)window;
    return true;
  }
};

}  // namespace e4b
