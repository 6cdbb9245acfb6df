// Strided block copy for the row-sharded pair's exchanges between GPUs.
//
// Each box copies a [d0][d1][d2] array of 16-byte vectors from a local source
// to a destination that may be another GPU's memory (a CUDA IPC mapping of its
// receive buffer): plain 16-byte loads here, plain 16-byte stores over NVLink
// there.  Strides are free on both sides, so the same kernel scatters row blocks
// into channel shards, gathers rows of a bias, and transposes pair blocks on the
// way.  No TMA, no multicast: only ordinary loads and stores.  The threads end
// with a system-scope fence so the peer's next stream operation after the
// exchange barrier sees every store.
#pragma once

#include "common.cuh"

namespace xfb {

constexpr int kMaxCopyBoxes = 16;

struct CopyBox {
  const uint4* src;
  uint4* dst;
  uint32_t d0, d1, d2;        // extents; d2 = contiguous 16-byte vectors per run
  int64_t s0, s1;             // source strides (vectors) of dims 0 and 1
  int64_t t0, t1;             // destination strides (vectors) of dims 0 and 1
};

struct CopyBoxes {
  CopyBox box[kMaxCopyBoxes];
  int count;
};

// blockIdx.y selects the box; blocks along x stride over its vectors.
__global__ void __launch_bounds__(256) exchange_copy_kernel(const __grid_constant__ CopyBoxes boxes) {
  const CopyBox& b = boxes.box[blockIdx.y];
  const uint64_t run = b.d2;
  const uint64_t plane = run * b.d1;
  const uint64_t total = plane * b.d0;
  for (uint64_t v = static_cast<uint64_t>(blockIdx.x) * blockDim.x + threadIdx.x; v < total;
       v += static_cast<uint64_t>(gridDim.x) * blockDim.x) {
    const uint64_t i0 = v / plane;
    const uint64_t r = v - i0 * plane;
    const uint64_t i1 = r / run;
    const uint64_t i2 = r - i1 * run;
    const uint4 x = b.src[i0 * b.s0 + i1 * b.s1 + i2];
    b.dst[i0 * b.t0 + i1 * b.t1 + i2] = x;
  }
  __threadfence_system();
}

}  // namespace xfb
