// Checkpoint upload: the parameter arrays of a record stream
// (xfold/params.py:39-95: per record a '<5i' header, scope, name, dtype, shape,
// then the raw little-endian array bytes) are copied to the device as one blob
// and scattered by this kernel into an arena where every array starts on a
// 256-byte boundary, so each becomes a typed tensor view without a host-side
// repack.  Record payloads start at arbitrary byte offsets in the blob.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace xfb {

// spans[r] = {source byte offset, destination byte offset (4-byte aligned), bytes}
__global__ void __launch_bounds__(256) gather_bytes_kernel(const uint8_t* src, uint8_t* dst,
                                                           const int64_t* spans, int64_t count) {
  for (int64_t r = blockIdx.x; r < count; r += gridDim.x) {
    const int64_t so = spans[3 * r], dof = spans[3 * r + 1], nb = spans[3 * r + 2];
    const uint8_t* s = src + so;
    uint8_t* d = dst + dof;
    const int64_t words = nb / 4;
    // four source bytes per thread, one aligned 32-bit store
    for (int64_t w = threadIdx.x; w < words; w += blockDim.x) {
      const uint8_t* p = s + 4 * w;
      const uint32_t v = static_cast<uint32_t>(p[0]) | (static_cast<uint32_t>(p[1]) << 8) |
                         (static_cast<uint32_t>(p[2]) << 16) | (static_cast<uint32_t>(p[3]) << 24);
      reinterpret_cast<uint32_t*>(d)[w] = v;
    }
    for (int64_t b = 4 * words + threadIdx.x; b < nb; b += blockDim.x) d[b] = s[b];
  }
}

}  // namespace xfb
