// cp.async helpers shared by the map and grouped kernels.
#pragma once

#include <cstdint>

namespace t0b {

// Asynchronous global -> shared copy of one element (no register round trip).
// The copies are ordered against shared-memory reads by the wait on their
// cp.async group and the CTA barrier that follows it.
template <int Bytes>
__device__ __forceinline__ void CopyAsync(uint32_t smem, const void* gmem) {
  if constexpr (Bytes == 16) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;\n" ::"r"(smem), "l"(gmem));
  } else {
    asm volatile("cp.async.ca.shared.global [%0], [%1], %2;\n" ::"r"(smem), "l"(gmem), "n"(Bytes));
  }
}

}  // namespace t0b
