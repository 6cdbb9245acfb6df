// GLU transition fused into one kernel for c = 128 (the pair Transition,
// xfold/nn/primitives.py:33-37 with gated_linear_unit_torch,
// xfold/fastnn/gated_linear_unit.py:103-107):
//
//   h   = silu(x W1_gate^T) * (x W1_value^T)      [rows][hid]
//   out (=|+=) bf16(h W2^T)                        [rows][128] f32
//
// The two-GEMM form writes h (rows x hid bf16, 1 GiB for the N = 1024 pair at
// hid = 512) to HBM and reads it back.  Here each CTA keeps a 128-row tile of h
// on chip, 64 hidden columns ("chunk") at a time:
//   GEMM1(j)  acc1[j % 2] = x W1[chunk j]^T       M = 128, N = 128 (64 gate | 64
//                                                 value rows of the packed W1), K = 128
//   epilogue  h(j) = silu(gate) * value -> bf16, 128-byte-swizzled K-major tile
//   GEMM2(j)  acc2 (+)= h(j) W2[:, chunk j]^T      M = 128, N = 128, K = 64
// and only the final acc2 tile leaves the SM (TMA reduce-add into the f32
// residual, or a store).  GEMM1 and GEMM2 have their own issuing threads, so
// GEMM1(j + 1) never waits behind GEMM2(j), whose h(j) the epilogue is still
// writing (with one issuer a clock64 trace showed the MMAs of a chunk issued one
// after another with the tensor pipe idle in between).
//
// TMEM (512 columns): acc1 x 2 at columns 0 / 128, acc2 x 2 at 256 / 384.
// Warps 0-7: epilogue (warp w: TMEM lane quarter w % 4, column half w / 4);
// warp 8: TMA producer of x and W1; warp 9: TMEM owner and GEMM1 issuer; warp
// 10: TMA producer of W2; warp 11: GEMM2 issuer.  The two weight rings have their own producers: W2(q)
// waits for GEMM2(q - 2), and a single producer would hold W1(q + 1) behind that
// wait (a clock64 trace showed GEMM1 issued ~1000 cycles late on every chunk).
#pragma once

#include "common.cuh"
#include "gemm.cuh"  // sw128_chunk, stage32_bf16_sw128

namespace xfb {

constexpr int kFtThreads = 384;
constexpr int kFtEpiThreads = 256;

struct FtSmem {
  static constexpr int kXBytes = 128 * 128 * 2;   // x tile: two 64-column swizzle atoms
  static constexpr int kW1Bytes = 128 * 128 * 2;  // W1 chunk: 64 gate + 64 value rows, K = 128
  static constexpr int kW2Bytes = 128 * 64 * 2;   // W2 chunk: 128 output rows, K = 64
  static constexpr int kHBytes = 128 * 64 * 2;    // h chunk: 128 rows, K = 64
  static constexpr int kOutBytes = 2 * 128 * 128; // two [128 rows][32 f32] boxes
  static constexpr int kXOff = 0;
  static constexpr int kW1Off = kXOff + 2 * kXBytes;
  static constexpr int kW2Off = kW1Off + 2 * kW1Bytes;
  static constexpr int kHOff = kW2Off + 2 * kW2Bytes;
  static constexpr int kOutOff = kHOff + 2 * kHBytes;
  static constexpr int kBarOff = kOutOff + kOutBytes;
  // x_full/empty, w1_full/empty, w2_full/empty, a1_full/empty, h_full/empty,
  // a2_full/empty: two of each
  static constexpr int kNumBars = 24;
  static constexpr int kTotal = kBarOff + kNumBars * 8 + 16;
  static constexpr int kLaunchBytes = kTotal + 1024;
  static_assert(kLaunchBytes <= 232448, "fused transition shared memory exceeds 227 KB");
};

// K-major operand in two (x, W1) or one (h, W2) 128-byte swizzle atoms of 64
// columns; k16 selects 16 columns.
__device__ __forceinline__ uint64_t ft_desc(uint32_t base, int k16) {
  return sw128_desc(base + (k16 >> 2) * 16384 + (k16 & 3) * 32, 16, 1024);
}

__global__ void __launch_bounds__(kFtThreads, 1)
    fused_transition_kernel(const __grid_constant__ CUtensorMap tmX,
                            const __grid_constant__ CUtensorMap tmW1,
                            const __grid_constant__ CUtensorMap tmW2,
                            const __grid_constant__ CUtensorMap tmOut, int rows, int chunks,
                            int accumulate) {
  using L = FtSmem;
  constexpr uint32_t kIdesc = idesc_bf16(128, 128, false, false);
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::kBarOff);
  uint64_t* x_full = bars;
  uint64_t* x_empty = bars + 2;
  uint64_t* w1_full = bars + 4;
  uint64_t* w1_empty = bars + 6;
  uint64_t* w2_full = bars + 8;
  uint64_t* w2_empty = bars + 10;
  uint64_t* a1_full = bars + 12;
  uint64_t* a1_empty = bars + 14;
  uint64_t* h_full = bars + 16;
  uint64_t* h_empty = bars + 18;
  uint64_t* a2_full = bars + 20;
  uint64_t* a2_empty = bars + 22;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + L::kNumBars);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int m_tiles = (rows + 127) / 128;

  if (threadIdx.x == 0) {
    for (int i = 0; i < 2; ++i) {
      mbar_init(&x_full[i], 1);
      mbar_init(&x_empty[i], 1);
      mbar_init(&w1_full[i], 1);
      mbar_init(&w1_empty[i], 1);
      mbar_init(&w2_full[i], 1);
      mbar_init(&w2_empty[i], 1);
      mbar_init(&a1_full[i], 1);
      mbar_init(&a1_empty[i], kFtEpiThreads);
      mbar_init(&h_full[i], kFtEpiThreads);
      mbar_init(&h_empty[i], 1);
      mbar_init(&a2_full[i], 1);
      mbar_init(&a2_empty[i], kFtEpiThreads);
    }
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 9) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  if (warp == 8 && lane == 0) {
    tma_prefetch(&tmX);
    tma_prefetch(&tmW1);
    tma_prefetch(&tmW2);
    tma_prefetch(&tmOut);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 8) {
    // ------------------------------------------------ TMA producer
    if (lane == 0) {
      int t_it = 0, q = 0;
      bool ok = true;
      for (int tile = blockIdx.x; ok && tile < m_tiles; tile += gridDim.x, ++t_it) {
        const int xb = t_it & 1;
        if (!mbar_wait(&x_empty[xb], ((t_it >> 1) & 1) ^ 1, kErrWaitProducer, abort_flag)) break;
        mbar_arrive_expect_tx(&x_full[xb], L::kXBytes);
        uint8_t* sx = smem + L::kXOff + xb * L::kXBytes;
        tma_load_3d(sx, &tmX, &x_full[xb], 0, tile * 128, 0);
        tma_load_3d(sx + 16384, &tmX, &x_full[xb], 64, tile * 128, 0);
        for (int j = 0; j < chunks; ++j, ++q) {
          const int s = q & 1;
          if (!mbar_wait(&w1_empty[s], ((q >> 1) & 1) ^ 1, kErrWaitProducer, abort_flag)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&w1_full[s], L::kW1Bytes);
          uint8_t* sw1 = smem + L::kW1Off + s * L::kW1Bytes;
          tma_load_3d(sw1, &tmW1, &w1_full[s], 0, 128 * j, 0);
          tma_load_3d(sw1 + 16384, &tmW1, &w1_full[s], 64, 128 * j, 0);
        }
      }
    }
  } else if (warp == 10) {
    // ------------------------------------------------ TMA producer of W2
    if (lane == 0) {
      int q = 0;
      bool ok = true;
      for (int tile = blockIdx.x; ok && tile < m_tiles; tile += gridDim.x) {
        for (int j = 0; j < chunks; ++j, ++q) {
          const int s = q & 1;
          if (!mbar_wait(&w2_empty[s], ((q >> 1) & 1) ^ 1, kErrWaitProducer, abort_flag)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&w2_full[s], L::kW2Bytes);
          tma_load_3d(smem + L::kW2Off + s * L::kW2Bytes, &tmW2, &w2_full[s], 64 * j, 0, 0);
        }
      }
    }
  } else if (warp == 9) {
    // ------------------------------------------------ MMA issuer
    if (lane == 0) {
      // GEMM1 issuer: runs ahead of the epilogue as far as the two acc1 buffers allow
      bool ok = true;
      int t_it = 0, q = 0;
      for (int tile = blockIdx.x; ok && tile < m_tiles; tile += gridDim.x, ++t_it) {
        const int xb = t_it & 1;
        if (!mbar_wait(&x_full[xb], (t_it >> 1) & 1, kErrWaitMma, abort_flag)) break;
        const uint32_t x_addr = smem_u32(smem + L::kXOff + xb * L::kXBytes);
        for (int j = 0; j < chunks; ++j, ++q) {
          const int s = q & 1;
          if (!mbar_wait(&w1_full[s], (q >> 1) & 1, kErrWaitMma, abort_flag) ||
              !mbar_wait(&a1_empty[s], ((q >> 1) & 1) ^ 1, kErrWaitMma, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t w1_addr = smem_u32(smem + L::kW1Off + s * L::kW1Bytes);
#pragma unroll
          for (int k = 0; k < 8; ++k)
            umma_bf16(tmem_base + s * 128, ft_desc(x_addr, k), ft_desc(w1_addr, k), kIdesc,
                      k > 0 ? 1u : 0u);
          umma_commit(&a1_full[s]);
          umma_commit(&w1_empty[s]);
          if (j == chunks - 1) umma_commit(&x_empty[xb]);
        }
      }
    }
  } else if (warp == 11) {
    // ------------------------------------------------ GEMM2 issuer
    // acc2[t % 2] (+)= h(q) W2[:, chunk q]^T as soon as the epilogue wrote h(q)
    if (lane == 0) {
      bool ok = true;
      int t_it = 0, q = 0;
      for (int tile = blockIdx.x; ok && tile < m_tiles; tile += gridDim.x, ++t_it) {
        const int ab = t_it & 1;
        for (int j = 0; j < chunks; ++j, ++q) {
          const int s = q & 1;
          if ((j == 0 &&
               !mbar_wait(&a2_empty[ab], ((t_it >> 1) & 1) ^ 1, kErrWaitMma, abort_flag)) ||
              !mbar_wait(&h_full[s], (q >> 1) & 1, kErrWaitMma, abort_flag) ||
              !mbar_wait(&w2_full[s], (q >> 1) & 1, kErrWaitMma, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t h_addr = smem_u32(smem + L::kHOff + s * L::kHBytes);
          const uint32_t w2_addr = smem_u32(smem + L::kW2Off + s * L::kW2Bytes);
          const uint32_t d = tmem_base + 256 + ab * 128;
#pragma unroll
          for (int k = 0; k < 4; ++k)
            umma_bf16(d, ft_desc(h_addr, k), ft_desc(w2_addr, k), kIdesc,
                      (j > 0 || k > 0) ? 1u : 0u);
          umma_commit(&h_empty[s]);
          umma_commit(&w2_empty[s]);
          if (j == chunks - 1) umma_commit(&a2_full[ab]);
        }
      }
    }
  } else if (warp < 8) {
    // ------------------------------------------------ epilogue warps 0-7
    const int row = (warp & 3) * 32 + lane;
    const int half = warp >> 2;
    const uint32_t t_row = tmem_base + (static_cast<uint32_t>((warp & 3) * 32) << 16);
    bool ok = true;
    int t_it = 0, q = 0;
    for (int tile = blockIdx.x; tile < m_tiles; tile += gridDim.x, ++t_it) {
      for (int j = 0; j < chunks; ++j, ++q) {
        const int s = q & 1;
        ok = mbar_wait(&a1_full[s], (q >> 1) & 1, kErrWaitEpilogue, abort_flag) && ok;
        tc_fence_after();
        float gv[32], vv[32];
        tmem_ld32(t_row + s * 128 + half * 32, gv);
        tmem_ld32(t_row + s * 128 + 64 + half * 32, vv);
        tc_fence_before();
        mbar_arrive(&a1_empty[s]);  // the accumulator may take GEMM1(q + 2)
#pragma unroll
        for (int i = 0; i < 32; ++i) gv[i] = gv[i] * sigmoid_fast(gv[i]) * vv[i];
        // GEMM2(q - 2) must be done reading this h buffer
        ok = mbar_wait(&h_empty[s], ((q >> 1) & 1) ^ 1, kErrWaitEpilogue, abort_flag) && ok;
        stage32_bf16_sw128(smem + L::kHOff + s * L::kHBytes, row, half * 4, gv);
        fence_async_smem();
        mbar_arrive(&h_full[s]);
      }
      // ---- the tile's output: acc2 -> bf16-rounded f32 -> TMA store / reduce-add,
      //      64 columns per round through the two staging boxes
      const int ab = t_it & 1;
      ok = mbar_wait(&a2_full[ab], (t_it >> 1) & 1, kErrWaitEpilogue, abort_flag) && ok;
      tc_fence_after();
#pragma unroll 1
      for (int r = 0; r < 2; ++r) {
        float o[32];
        tmem_ld32(t_row + 256 + ab * 128 + 64 * r + 32 * half, o);
        if (r == 1) {
          tc_fence_before();
          mbar_arrive(&a2_empty[ab]);
        }
        // the previous round's stores must have read the staging boxes
        if (threadIdx.x == 0) bulk_wait_read<0>();
        named_barrier(1, kFtEpiThreads);
        uint8_t* box = smem + L::kOutOff + half * 16384;
#pragma unroll
        for (int c = 0; c < 8; ++c)
          *reinterpret_cast<float4*>(sw128_chunk(box, row, c)) =
              make_float4(bf16r(o[4 * c]), bf16r(o[4 * c + 1]), bf16r(o[4 * c + 2]),
                          bf16r(o[4 * c + 3]));
        fence_async_smem();
        named_barrier(1, kFtEpiThreads);
        if (threadIdx.x == 0 && ok && !*abort_flag) {
#pragma unroll
          for (int b = 0; b < 2; ++b) {
            const uint8_t* src = smem + L::kOutOff + b * 16384;
            if (accumulate) {
              tma_reduce_add_3d(&tmOut, src, 64 * r + 32 * b, tile * 128, 0);
            } else {
              tma_store_3d(&tmOut, src, 64 * r + 32 * b, tile * 128, 0);
            }
          }
        }
        if (threadIdx.x == 0) bulk_commit();
      }
    }
    if (threadIdx.x == 0) bulk_wait<0>();
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 9) {
    tc_fence_after();
    tmem_dealloc(tmem_base, 512);
  }
}

}  // namespace xfb
