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

// blockIdx.y selects the box; blocks along x stride over its vectors, four
// independent vectors per thread per step so several loads are in flight
// before the (remote) stores.  Boxes hold fewer than 2^32 vectors.
__global__ void __launch_bounds__(256) exchange_copy_kernel(const __grid_constant__ CopyBoxes boxes) {
  const CopyBox& b = boxes.box[blockIdx.y];
  const uint32_t run = b.d2;
  const uint32_t plane = run * b.d1;
  const uint32_t total = plane * b.d0;
  const uint32_t nthreads = gridDim.x * blockDim.x;
  for (uint32_t v0 = blockIdx.x * blockDim.x + threadIdx.x; v0 < total; v0 += 4 * nthreads) {
    uint4 x[4];
    int64_t dst[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const uint32_t v = v0 + k * nthreads;
      dst[k] = -1;
      if (v < total) {
        const uint32_t i0 = v / plane;
        const uint32_t r = v - i0 * plane;
        const uint32_t i1 = r / run;
        const uint32_t i2 = r - i1 * run;
        x[k] = b.src[i0 * b.s0 + i1 * b.s1 + i2];
        dst[k] = i0 * b.t0 + i1 * b.t1 + i2;
      }
    }
#pragma unroll
    for (int k = 0; k < 4; ++k)
      if (dst[k] >= 0) b.dst[dst[k]] = x[k];
  }
  __threadfence_system();
}

// Barrier of an exchange between GPUs, lighter than a collective call.  After
// this GPU's copy kernel (same stream, so its stores are complete and fenced),
// exchange_signal_kernel writes `epoch` into slot `rank` of every GPU's flag
// array with system-scope release stores; exchange_wait_kernel then spins,
// with acquire loads, until every slot of this GPU's own array holds at least
// `epoch`.  The spin gives up after XFB_WAIT_NS of global time, records
// kErrWaitPeer and returns, so a peer that never signals cannot hang this GPU.
constexpr int kMaxPeers = 16;

//
// With a counter (a uint32 in this GPU's memory, zero at the start) the epoch
// is not a launch argument: the signal kernel advances the counter and uses
// its new value, the wait kernel reads it.  Every rank passes the same barriers
// in the same order, so the counters agree, and a stream segment holding such
// barriers can be captured into a CUDA graph and replayed.
struct PeerFlags {
  uint32_t* flags[kMaxPeers];  // each GPU's flag array, as mapped in this process
  int world;
  int rank;
  uint32_t epoch;
  uint32_t* counter;  // or null: use epoch
};

__global__ void exchange_signal_kernel(const __grid_constant__ PeerFlags p) {
  __shared__ uint32_t epoch;
  if (threadIdx.x == 0) {
    uint32_t e = p.epoch;
    if (p.counter != nullptr) {
      e = *p.counter + 1;
      *p.counter = e;
    }
    epoch = e;
  }
  __syncthreads();
  const int s = threadIdx.x;
  if (s < p.world) {
    __threadfence_system();
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p.flags[s] + p.rank), "r"(epoch)
                 : "memory");
  }
}

__global__ void exchange_wait_kernel(const uint32_t* flags, int world, uint32_t epoch,
                                     const uint32_t* counter) {
  const int s = threadIdx.x;
  if (s >= world) return;
  if (counter != nullptr) epoch = *counter;
  const uint64_t start = global_ns();
  while (true) {
    uint32_t v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(flags + s) : "memory");
    if (static_cast<int32_t>(v - epoch) >= 0) break;
    if (global_ns() - start > XFB_WAIT_NS) {
      record_error(kErrWaitPeer);
      break;
    }
    __nanosleep(200);
  }
}

}  // namespace xfb
