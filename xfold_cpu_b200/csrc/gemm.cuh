// Persistent, warp-specialised bf16 GEMM on tcgen05 for sm_100a.
//
//   D[bat][m][n] = sum_k A[bat](m, k) * B[bat or 0](n, k)     (f32 accumulate in TMEM)
//
// A and B are read by TMA into 128-byte-swizzled shared-memory stages.  Each
// operand is K-major (K contiguous: activations [rows][K], nn.Linear weights
// [out][in]) or MN-major (M/N contiguous: the incoming triangle contraction).
// With `b_shared` the B operand is the same for every batch index — used to
// run the K = c projections "batched over pair rows" so that no output tile
// straddles two rows of the pair.
//
// Warp roles (320 threads, one CTA per SM):
//   warps 0-7  epilogue: warp w reads TMEM lane quarter w%4 and column half w/4
//   warp 8     TMA producer (one elected lane): A/B stages + the epilogue's
//              auxiliary input tile (e.g. the output gate), double-buffered
//   warp 9     TMEM allocator + MMA issuer (one elected lane)
// The accumulator is double-buffered in TMEM (2 x BN columns), so the epilogue
// of tile i overlaps the main loop of tile i+1.  Epilogues stage their output
// tile in shared memory and one thread writes it with TMA bulk stores (or a
// TMA reduce-add into an f32 residual stream), so global traffic is in full
// lines regardless of the output layout.
//
// Epilogue protocol (all 256 epilogue threads, one call per tile):
//   Epi::compute(ctx)  TMEM -> registers -> math -> staging buffer
//   Epi::store(ctx)    (one thread) bulk stores from the staging buffer
#pragma once

#include <type_traits>

#include "common.cuh"

namespace xfb {

constexpr int kGemmBM = 128;
constexpr int kGemmBK = 64;  // one 128-byte swizzle atom of bf16
constexpr int kGemmEpiThreads = 256;  // one epilogue group: 8 warps

// Epilogues that declare kGroups = 2 (and have two staging buffers) run two
// epilogue groups of 8 warps: group g takes the tiles that use TMEM accumulator
// g and staging buffer g, so two tiles' epilogues are in flight at once.  It
// pays where the epilogue is long per tile (the triangle projection), and costs
// elsewhere (registers drop to 96 with 19 warps).
template <class E, class = void>
struct EpiGroupsOf {
  static constexpr int value = 1;
};
template <class E>
struct EpiGroupsOf<E, std::void_t<decltype(E::kGroups)>> {
  static constexpr int value = E::kGroups;
};

// Epilogues with `route` (an int member) may store into other GPUs' receive
// buffers: the kernel then ends with a system-scope fence in every thread, so
// the exchange barrier that follows on the stream publishes those stores.
template <class E, class = void>
struct EpiRoutedOf {
  static constexpr bool value = false;
};
template <class E>
struct EpiRoutedOf<E, std::void_t<decltype(E::route)>> {
  static constexpr bool value = true;
};

// Epilogues with kGroupCopy = true get Epi::group_copy(ctx, t) called by every
// thread t (0..255) of the epilogue group after the tile is staged, between two
// group barriers: plain 16-byte stores of the staged tile by all 256 threads,
// for destinations no tensor map describes (another GPU's receive buffer).
// Both barriers are reached by every thread whatever its waits returned, so an
// aborting CTA cannot strand a barrier.
template <class E, class = void>
struct EpiGroupCopyOf {
  static constexpr bool value = false;
};
template <class E>
struct EpiGroupCopyOf<E, std::void_t<decltype(E::kGroupCopy)>> {
  static constexpr bool value = E::kGroupCopy;
};

// Destinations of a routed store: one receive buffer per rank of the exchange
// (this GPU's own buffer among them), as mapped in this process.
constexpr int kMaxRoute = 16;

// Warp layout of the GEMM kernel for epilogue Epi: the epilogue group(s), then
// the TMA producer, the MMA issuer and the bulk-store issuer.
template <class Epi>
struct GemmWarps {
  static constexpr int kGroups =
      (Epi::kStagingBytes > 0 && Epi::kStagingBufs == 2 && EpiGroupsOf<Epi>::value == 2) ? 2 : 1;
  static constexpr int kProducer = 8 * kGroups;
  static constexpr int kMma = kProducer + 1;
  static constexpr int kStore = kProducer + 2;
  static constexpr int kThreads = kGemmEpiThreads * kGroups + 96;
};

struct GemmShape {
  int M, N, K, batch;
  int m_tiles, n_tiles, k_blocks;
  int b_shared;  // 1: B has no batch dimension
};

// What an epilogue sees for its share of one tile.
struct EpiCtx {
  int bat;            // batch index
  int m0, n0;         // tile origin
  int row;            // row inside the tile (0..127) = TMEM lane
  int half;           // column half (0/1) handled by this thread
  uint32_t tmem;      // TMEM address of tile column 0 in this thread's lane quarter
  uint8_t* staging;   // staging buffer of this tile
  const uint8_t* aux; // auxiliary input tile (nullptr when the epilogue has none)
  float2 pre;         // Epi::prefetch(ctx), read before the accumulator was ready
};

// Epilogues with a `float2 prefetch(const EpiCtx&) const` method get it called
// for each tile before the epilogue waits for the tile's accumulator, so a
// global load it issues overlaps the main loop; compute() reads it as ctx.pre.
template <class E, class = void>
struct EpiPrefetchOf {
  static constexpr bool value = false;
};
template <class E>
struct EpiPrefetchOf<E, std::void_t<decltype(&E::prefetch)>> {
  static constexpr bool value = true;
};

template <int BN, int STAGES, class Epi>
struct GemmSmem {
  static constexpr int kABytes = kGemmBM * kGemmBK * 2;
  static constexpr int kBBytes = BN * kGemmBK * 2;
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kAuxStride = ((Epi::kAuxBytes + 1023) / 1024) * 1024;
  static constexpr int kStagingStride = ((Epi::kStagingBytes + 1023) / 1024) * 1024;
  static constexpr int kAuxOff = STAGES * kStageBytes;
  static constexpr int kStagingOff = kAuxOff + 2 * kAuxStride;
  static constexpr int kBarOff = kStagingOff + Epi::kStagingBufs * kStagingStride;
  // full[S], empty[S], tfull[2], tempty[2], aux_full[2], aux_empty[2],
  // staging_full[2], staging_free[2]
  static constexpr int kNumBars = 2 * STAGES + 12;
  static constexpr int kTotal = kBarOff + kNumBars * 8 + 16;
  static constexpr int kLaunchBytes = kTotal + 1024;  // slack for 1024-byte alignment
  static_assert(kLaunchBytes <= 232448, "GEMM shared memory exceeds 227 KB");
};

template <int BN, int STAGES, bool A_MN, bool B_MN, class Epi>
__global__ void __launch_bounds__(GemmWarps<Epi>::kThreads, 1)
    gemm_bf16_kernel(const __grid_constant__ CUtensorMap tmA,
                     const __grid_constant__ CUtensorMap tmB, GemmShape shape,
                     const __grid_constant__ Epi epi) {
  static_assert(BN % 64 == 0 && BN >= 64 && BN <= 256, "BN must be 64, 128, 192 or 256");
  using L = GemmSmem<BN, STAGES, Epi>;
  using W = GemmWarps<Epi>;
  constexpr int kGemmProducerWarp = W::kProducer;
  constexpr int kGemmMmaWarp = W::kMma;
  constexpr int kGemmStoreWarp = W::kStore;
  constexpr uint32_t kTmemCols = (2 * BN <= 256) ? 256 : 512;
  constexpr uint32_t kIdesc = idesc_bf16(kGemmBM, BN, A_MN, B_MN);
  constexpr bool kAux = Epi::kAuxBytes > 0;

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L::kBarOff);
  uint64_t* empty = full + STAGES;
  uint64_t* tfull = empty + STAGES;
  uint64_t* tempty = tfull + 2;
  uint64_t* aux_full = tempty + 2;
  uint64_t* aux_empty = aux_full + 2;
  uint64_t* staging_full = aux_empty + 2;
  uint64_t* staging_free = staging_full + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(staging_free + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], kGemmEpiThreads);
      mbar_init(&aux_full[b], 1);
      mbar_init(&aux_empty[b], kGemmEpiThreads);
      mbar_init(&staging_full[b], kGemmEpiThreads);
      mbar_init(&staging_free[b], 1);
    }
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == kGemmMmaWarp) {
    tmem_alloc(tmem_slot, kTmemCols);
    tmem_relinquish();
  }
  if (warp == kGemmProducerWarp && lane == 0) {
    tma_prefetch(&tmA);
    tma_prefetch(&tmB);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  const int tiles_per_batch = shape.m_tiles * shape.n_tiles;
  const int total_tiles = tiles_per_batch * shape.batch;

  if (warp == kGemmProducerWarp) {
    // ------------------------------------------------ TMA producer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      for (int tile = blockIdx.x; tile < total_tiles && !*abort_flag; tile += gridDim.x) {
        const int bat = tile / tiles_per_batch;
        const int rem = tile - bat * tiles_per_batch;
        const int m0 = (rem / shape.n_tiles) * kGemmBM;
        const int n0 = (rem % shape.n_tiles) * BN;
        const int bb = shape.b_shared ? 0 : bat;
        if constexpr (kAux) {
          if (!mbar_wait(&aux_empty[acc], acc_phase ^ 1, kErrWaitProducer, abort_flag)) break;
          mbar_arrive_expect_tx(&aux_full[acc], Epi::kAuxBytes);
          epi.load_aux(smem + L::kAuxOff + acc * L::kAuxStride, &aux_full[acc], bat, m0, n0);
        }
        for (int kb = 0; kb < shape.k_blocks; ++kb) {
          if (!mbar_wait(&empty[stage], phase ^ 1, kErrWaitProducer, abort_flag)) break;
          uint8_t* sA = smem + stage * L::kStageBytes;
          uint8_t* sB = sA + L::kABytes;
          mbar_arrive_expect_tx(&full[stage], L::kStageBytes);
          const int k0 = kb * kGemmBK;
          if constexpr (A_MN) {
            tma_load_3d(sA, &tmA, &full[stage], m0, k0, bat);
            tma_load_3d(sA + 8192, &tmA, &full[stage], m0 + 64, k0, bat);
          } else {
            tma_load_3d(sA, &tmA, &full[stage], k0, m0, bat);
          }
          if constexpr (B_MN) {
#pragma unroll
            for (int c = 0; c < BN / 64; ++c)
              tma_load_3d(sB + c * 8192, &tmB, &full[stage], n0 + 64 * c, k0, bb);
          } else {
            tma_load_3d(sB, &tmB, &full[stage], k0, n0, bb);
          }
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (++acc == 2) {
          acc = 0;
          acc_phase ^= 1;
        }
      }
    }
  } else if (warp == kGemmMmaWarp) {
    // ------------------------------------------------ MMA issuer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      for (int tile = blockIdx.x; tile < total_tiles && !*abort_flag; tile += gridDim.x) {
        if (!mbar_wait(&tempty[acc], acc_phase ^ 1, kErrWaitMma, abort_flag)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * BN;
        bool ok = true;
        for (int kb = 0; kb < shape.k_blocks; ++kb) {
          if (!mbar_wait(&full[stage], phase, kErrWaitMma, abort_flag)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_addr = smem_u32(smem + stage * L::kStageBytes);
          const uint32_t b_addr = a_addr + L::kABytes;
#pragma unroll
          for (int k = 0; k < kGemmBK / 16; ++k) {
            const uint64_t adesc = A_MN ? sw128_desc(a_addr + k * 2048, 8192, 1024)
                                        : sw128_desc(a_addr + k * 32, 16, 1024);
            const uint64_t bdesc = B_MN ? sw128_desc(b_addr + k * 2048, 8192, 1024)
                                        : sw128_desc(b_addr + k * 32, 16, 1024);
            umma_bf16(d_tmem, adesc, bdesc, kIdesc, (kb > 0 || k > 0) ? 1u : 0u);
          }
          umma_commit(&empty[stage]);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) break;
        umma_commit(&tfull[acc]);
        if (++acc == 2) {
          acc = 0;
          acc_phase ^= 1;
        }
      }
    }
  } else if (warp == kGemmStoreWarp) {
    // ------------------------------------------------ bulk-store issuer
    // Takes each staged tile once every epilogue thread has written it, issues
    // the epilogue's TMA store, and frees the staging buffer as soon as that
    // store has read it.  The epilogue warps never wait for one another.
    if constexpr (Epi::kStagingBytes > 0) {
      if (lane == 0) {
        constexpr int NB = Epi::kStagingBufs;
        int iter = 0;
        EpiCtx ctx;
        ctx.row = 0;
        ctx.half = 0;
        ctx.tmem = 0;
        ctx.aux = nullptr;
        for (int tile = blockIdx.x; tile < total_tiles; tile += gridDim.x, ++iter) {
          const int b = iter % NB;
          const uint32_t ph = (iter / NB) & 1;
          const bool ok = mbar_wait(&staging_full[b], ph, kErrWaitEpilogue, abort_flag);
          const int bat = tile / tiles_per_batch;
          const int rem = tile - bat * tiles_per_batch;
          ctx.bat = bat;
          ctx.m0 = (rem / shape.n_tiles) * kGemmBM;
          ctx.n0 = (rem % shape.n_tiles) * BN;
          ctx.staging = smem + L::kStagingOff + b * L::kStagingStride;
          if (ok && !*abort_flag) epi.store(ctx);
          bulk_commit();
          // free the buffer as soon as this store has read it: the epilogue
          // warps are then never waiting on the next tile's handoff
          bulk_wait_read<0>();
          mbar_arrive(&staging_free[b]);
        }
        bulk_wait<0>();
      }
    }
  } else {
    // ------------------------------------------------ epilogue warps (1 or 2 groups of 8)
    constexpr int NB = Epi::kStagingBufs;
    constexpr int G = W::kGroups;
    const int group = warp >> 3;
    // with two groups, group g always uses accumulator g (tile iterations g, g+2, ...)
    int acc = group;
    uint32_t acc_phase = 0;
    int iter = group;
    EpiCtx ctx;
    ctx.row = (warp & 3) * 32 + lane;
    ctx.half = (warp & 7) >> 2;
    for (int tile = blockIdx.x + group * gridDim.x; tile < total_tiles;
         tile += G * gridDim.x, iter += G) {
      const int bat = tile / tiles_per_batch;
      const int rem = tile - bat * tiles_per_batch;
      ctx.bat = bat;
      ctx.m0 = (rem / shape.n_tiles) * kGemmBM;
      ctx.n0 = (rem % shape.n_tiles) * BN;
      if constexpr (EpiPrefetchOf<Epi>::value) ctx.pre = epi.prefetch(ctx);
      // Every epilogue thread runs every tile and arrives on every barrier: a
      // wait that gave up (the CTA is aborting) skips the work, not the arrivals.
      bool ok = mbar_wait(&tfull[acc], acc_phase, kErrWaitEpilogue, abort_flag);
      if constexpr (kAux) {
        ok = mbar_wait(&aux_full[acc], acc_phase, kErrWaitEpilogue, abort_flag) && ok;
      }
      tc_fence_after();
      ctx.tmem = tmem_base + (static_cast<uint32_t>((warp & 3) * 32) << 16) + acc * BN;
      ctx.staging = smem + L::kStagingOff + (iter % NB) * L::kStagingStride;
      ctx.aux = kAux ? smem + L::kAuxOff + acc * L::kAuxStride : nullptr;
      if constexpr (Epi::kStagingBytes > 0) {
        // the store that last read this staging buffer must be done reading it
        if (iter >= NB)
          ok = mbar_wait(&staging_free[iter % NB], ((iter / NB) - 1) & 1, kErrWaitEpilogue,
                         abort_flag) && ok;
      }
      if (ok) epi.compute(ctx);
      fence_async_smem();
      tc_fence_before();
      mbar_arrive(&tempty[acc]);
      if constexpr (kAux) mbar_arrive(&aux_empty[acc]);
      if constexpr (EpiGroupCopyOf<Epi>::value) {
        // the accumulator is free again; now the group stores the staged tile
        named_barrier(1 + group, kGemmEpiThreads);  // the whole tile is staged
        if (ok && !*abort_flag) epi.group_copy(ctx, threadIdx.x & (kGemmEpiThreads - 1));
        named_barrier(1 + group, kGemmEpiThreads);  // and read before it is reused
      }
      if constexpr (Epi::kStagingBytes > 0) mbar_arrive(&staging_full[iter % NB]);
      if constexpr (G == 2) {
        acc_phase ^= 1;
      } else if (++acc == 2) {
        acc = 0;
        acc_phase ^= 1;
      }
    }
  }

  if constexpr (EpiRoutedOf<Epi>::value) {
    if (epi.route) __threadfence_system();
  }
  tc_fence_before();
  __syncthreads();
  if (warp == kGemmMmaWarp) {
    tc_fence_after();
    tmem_dealloc(tmem_base, kTmemCols);
  }
}

// ====================================================================== epilogue helpers

__device__ __forceinline__ void store16_bf16(__nv_bfloat16* dst, const float (&v)[16]) {
  uint4 a, b;
  a.x = pack_bf16x2(v[0], v[1]);
  a.y = pack_bf16x2(v[2], v[3]);
  a.z = pack_bf16x2(v[4], v[5]);
  a.w = pack_bf16x2(v[6], v[7]);
  b.x = pack_bf16x2(v[8], v[9]);
  b.y = pack_bf16x2(v[10], v[11]);
  b.z = pack_bf16x2(v[12], v[13]);
  b.w = pack_bf16x2(v[14], v[15]);
  reinterpret_cast<uint4*>(dst)[0] = a;
  reinterpret_cast<uint4*>(dst)[1] = b;
}

// Address of 16-byte chunk `chunk` (0..7) of row `row` in a [rows][128 B] tile
// written / read by TMA with the 128-byte swizzle (base 1024-byte aligned).
__device__ __forceinline__ uint8_t* sw128_chunk(uint8_t* base, int row, int chunk) {
  return base + row * 128 + ((chunk ^ (row & 7)) << 4);
}
__device__ __forceinline__ const uint8_t* sw128_chunk(const uint8_t* base, int row, int chunk) {
  return base + row * 128 + ((chunk ^ (row & 7)) << 4);
}

// Same for [rows][64 B] tiles with the 64-byte swizzle (base 512-byte aligned).
__device__ __forceinline__ uint8_t* sw64_chunk(uint8_t* base, int row, int chunk) {
  return base + row * 64 + ((chunk ^ ((row >> 1) & 3)) << 4);
}

// Stores 32 floats as bf16 into four consecutive swizzled 16-byte chunks.
__device__ __forceinline__ void stage32_bf16_sw128(uint8_t* base, int row, int chunk0,
                                                   const float* v) {
#pragma unroll
  for (int c = 0; c < 4; ++c) {
    uint4 w;
    w.x = pack_bf16x2(v[8 * c + 0], v[8 * c + 1]);
    w.y = pack_bf16x2(v[8 * c + 2], v[8 * c + 3]);
    w.z = pack_bf16x2(v[8 * c + 4], v[8 * c + 5]);
    w.w = pack_bf16x2(v[8 * c + 6], v[8 * c + 7]);
    *reinterpret_cast<uint4*>(sw128_chunk(base, row, chunk0 + c)) = w;
  }
}

// ====================================================================== epilogues

// Plain output through TMA: out (f32 or bf16) [bat][m][n] = bf16(acc + bias),
// stored, or added into an f32 tensor with a TMA reduce-add (the residual
// update x += op(x)).  The output map is 3-D {N, M, batch} with a box of
// {32 f32 | 64 bf16, 128, 1} and the 128-byte swizzle.
template <int BN, bool OUT_F32>
struct EpiOut {
  static constexpr int kColsPerBox = OUT_F32 ? 32 : 64;
  static constexpr int kStagingBytes = 128 * BN * (OUT_F32 ? 4 : 2);
  static constexpr int kStagingBufs = 1;
  static constexpr int kAuxBytes = 0;
  CUtensorMap out_map;
  const float* bias;   // [N] or null
  int accumulate;      // TMA reduce-add instead of store (f32 only)

  __device__ void load_aux(void*, uint64_t*, int, int, int) const {}

  __device__ void compute(const EpiCtx& c) const {
    constexpr int kHalf = BN / 2;
#pragma unroll 1
    for (int c0 = 0; c0 < kHalf; c0 += 16) {
      const int col = c.half * kHalf + c0;
      float v[16];
      tmem_ld16(c.tmem + col, v);
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        const float b = bias ? bias[c.n0 + col + i] : 0.f;
        v[i] = bf16r(v[i] + b);
      }
      write(c, col, v);
    }
  }

  __device__ __forceinline__ void write(const EpiCtx& c, int col, const float (&v)[16]) const {
    uint8_t* box = c.staging + (col / kColsPerBox) * (128 * 128);
    const int inbox = col % kColsPerBox;
    if constexpr (OUT_F32) {
#pragma unroll
      for (int q = 0; q < 4; ++q)
        *reinterpret_cast<float4*>(sw128_chunk(box, c.row, inbox / 4 + q)) =
            make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
    } else {
#pragma unroll
      for (int q = 0; q < 2; ++q) {
        uint4 w;
        w.x = pack_bf16x2(v[8 * q + 0], v[8 * q + 1]);
        w.y = pack_bf16x2(v[8 * q + 2], v[8 * q + 3]);
        w.z = pack_bf16x2(v[8 * q + 4], v[8 * q + 5]);
        w.w = pack_bf16x2(v[8 * q + 6], v[8 * q + 7]);
        *reinterpret_cast<uint4*>(sw128_chunk(box, c.row, inbox / 8 + q)) = w;
      }
    }
  }

  __device__ void store(const EpiCtx& c) const {
#pragma unroll
    for (int b = 0; b < BN / kColsPerBox; ++b) {
      const uint8_t* src = c.staging + b * (128 * 128);
      if (OUT_F32 && accumulate) {
        tma_reduce_add_3d(&out_map, src, c.n0 + b * kColsPerBox, c.m0, c.bat);
      } else {
        tma_store_3d(&out_map, src, c.n0 + b * kColsPerBox, c.m0, c.bat);
      }
    }
  }
};

// EpiOut with an output gate [M][N] bf16 (already squashed) read through the
// auxiliary TMA ring: out = bf16(bf16(acc + bias) * gate).  Gate map 3-D
// {N, M, 1}, box {64, 128, 1}, 128-byte swizzle.
template <int BN, bool OUT_F32>
struct EpiOutGated : EpiOut<BN, OUT_F32> {
  static constexpr int kAuxBytes = 128 * BN * 2;
  CUtensorMap gate_map;

  __device__ void load_aux(void* dst, uint64_t* bar, int bat, int m0, int n0) const {
#pragma unroll
    for (int b = 0; b < BN / 64; ++b)
      tma_load_3d(static_cast<uint8_t*>(dst) + b * 16384, &gate_map, bar, n0 + 64 * b, m0, bat);
  }

  __device__ void compute(const EpiCtx& c) const {
    constexpr int kHalf = BN / 2;
#pragma unroll 1
    for (int c0 = 0; c0 < kHalf; c0 += 16) {
      const int col = c.half * kHalf + c0;
      float v[16], g[16];
      tmem_ld16(c.tmem + col, v);
      const uint8_t* gbox = c.aux + (col / 64) * 16384;
      unpack8_bf16(*reinterpret_cast<const uint4*>(sw128_chunk(gbox, c.row, (col % 64) / 8)), g);
      unpack8_bf16(*reinterpret_cast<const uint4*>(sw128_chunk(gbox, c.row, (col % 64) / 8 + 1)),
                   g + 8);
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        const float b = this->bias ? this->bias[c.n0 + col + i] : 0.f;
        v[i] = bf16r(bf16r(v[i] + b) * g[i]);
      }
      this->write(c, col, v);
    }
  }
};

// EpiOutGated whose A operand is the un-normalised input of a LayerNorm over
// the K dimension, folded into the GEMM: with per-row stats (mean, rstd) and a
// weight W'[n][k] = gamma[k] W[n][k],
//   LN(x) W^T = rstd (x W'^T - mean colsum) + colbias,
//   colsum[n] = sum_k W'[n][k],  colbias[n] = sum_k beta[k] W[n][k],
// then out = bf16(bf16(that) * gate).  The centring happens on the f32
// accumulator, so no rounding of the normalised activations is involved.
template <int BN, bool OUT_F32>
struct EpiOutLnGated : EpiOutGated<BN, OUT_F32> {
  const float2* stats;   // [rows] (mean, rstd)
  const float* colsum;   // [N]
  const float* colbias;  // [N]
  int rows;

  // the row's statistics, loaded while the tile's MMAs run
  __device__ float2 prefetch(const EpiCtx& c) const { return stats[min(c.m0 + c.row, rows - 1)]; }

  __device__ void compute(const EpiCtx& c) const {
    constexpr int kHalf = BN / 2;
    const float2 st = c.pre;
#pragma unroll 1
    for (int c0 = 0; c0 < kHalf; c0 += 16) {
      const int col = c.half * kHalf + c0;
      float v[16], g[16];
      tmem_ld16(c.tmem + col, v);
      const uint8_t* gbox = c.aux + (col / 64) * 16384;
      unpack8_bf16(*reinterpret_cast<const uint4*>(sw128_chunk(gbox, c.row, (col % 64) / 8)), g);
      unpack8_bf16(*reinterpret_cast<const uint4*>(sw128_chunk(gbox, c.row, (col % 64) / 8 + 1)),
                   g + 8);
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        const int n = c.n0 + col + i;
        const float y = fmaf(st.y, fmaf(-st.x, colsum[n], v[i]), colbias[n]);
        v[i] = bf16r(bf16r(y) * g[i]);
      }
      this->write(c, col, v);
    }
  }
};

// Direct per-thread stores (no staging): out [bat][m][ld] bf16 or f32.  Used by
// the batched contraction (whose rows are 512-byte contiguous runs) and by odd
// shapes the TMA layouts do not cover.
//
// With route != 0 each output row goes to the receive buffer of the rank that
// owns it (dst[s], s = that rank; this rank is `rank`) instead of `out`:
//   route 1, channels -> rows: row i of channel `bat` (a contraction over this
//     rank's route_batch channels) is row i % route_rows of channel
//     rank * route_batch + bat on rank s = i / route_rows
//     (receive buffer [G * route_batch][route_rows][ld_out]);
//   route 2, transpose: row jj * route_n + i (this rank's column block jj, pair
//     row i) is row (i % route_rows) * route_n + rank * route_rows + jj on rank
//     s = i / route_rows (receive buffer [route_rows][route_n][ld_out]).
template <int BN>
struct EpiDirect {
  static constexpr int kStagingBytes = 0;
  static constexpr int kStagingBufs = 1;
  static constexpr int kAuxBytes = 0;
  void* out;
  int64_t ld_out;
  int64_t bstride_out;
  int out_f32;
  int accumulate;
  const float* bias;
  const __nv_bfloat16* gate;
  int64_t ld_gate;
  int M, N;
  int route = 0;
  int rank, route_rows, route_batch, route_n;
  void* dst[kMaxRoute];

  __device__ void load_aux(void*, uint64_t*, int, int, int) const {}
  __device__ void store(const EpiCtx&) const {}

  __device__ void compute(const EpiCtx& c) const {
    constexpr int kHalf = BN / 2;
    const int row = c.m0 + c.row;
    const bool row_ok = row < M;
    int64_t row_off = c.bat * bstride_out + static_cast<int64_t>(row) * ld_out;
    void* obase = out;
    if (route != 0 && row_ok) {
      if (route == 1) {
        const int s = row / route_rows;
        obase = dst[s];
        row_off = (static_cast<int64_t>(rank * route_batch + c.bat) * route_rows +
                   (row - s * route_rows)) * ld_out;
      } else {
        const int jj = row / route_n;
        const int i = row - jj * route_n;
        const int s = i / route_rows;
        obase = dst[s];
        row_off = (static_cast<int64_t>(i - s * route_rows) * route_n + rank * route_rows + jj) *
                  ld_out;
      }
    }
    const __nv_bfloat16* grow = gate ? gate + static_cast<int64_t>(row) * ld_gate : nullptr;
#pragma unroll 1
    for (int c0 = 0; c0 < kHalf; c0 += 16) {
      float v[16];
      tmem_ld16(c.tmem + c.half * kHalf + c0, v);
      const int col = c.n0 + c.half * kHalf + c0;
      if (!row_ok || col >= N) continue;
      const bool full = col + 16 <= N;
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        float x = v[i];
        if (bias != nullptr && (full || col + i < N)) x += bias[col + i];
        v[i] = bf16r(x);
      }
      if (grow != nullptr) {
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const float g = (full || col + i < N) ? __bfloat162float(grow[col + i]) : 0.f;
          v[i] = bf16r(v[i] * g);
        }
      }
      if (out_f32) {
        float* orow = reinterpret_cast<float*>(obase) + row_off;
        if (full) {
          float4* dst = reinterpret_cast<float4*>(orow + col);
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            float4 o = make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
            if (accumulate) {
              const float4 p = dst[q];
              o.x += p.x;
              o.y += p.y;
              o.z += p.z;
              o.w += p.w;
            }
            dst[q] = o;
          }
        } else {
#pragma unroll
          for (int i = 0; i < 16; ++i)
            if (col + i < N) orow[col + i] = accumulate ? orow[col + i] + v[i] : v[i];
        }
      } else {
        __nv_bfloat16* orow = reinterpret_cast<__nv_bfloat16*>(obase) + row_off;
        if (full) {
          store16_bf16(orow + col, v);
        } else {
#pragma unroll
          for (int i = 0; i < 16; ++i)
            if (col + i < N) orow[col + i] = __float2bfloat16_rn(v[i]);
        }
      }
    }
  }
};

// bf16 output rows routed to the ranks that own them (the channels -> rows and
// transpose exchanges of a row-sharded pair, done by the producer), through a
// staged tile: the epilogue threads write their row's BN values into a
// swizzled [128][BN] bf16 staging tile, then copy it out together 16 bytes per
// thread, consecutive threads on consecutive bytes of a row, so every store
// instruction writes whole rows (BN * 2 contiguous bytes) over NVLink.
// Destinations as EpiDirect's route 1 / route 2; N % 8 == 0.
template <int BN>
struct EpiRowsRouted {
  static constexpr int kStagingBytes = 128 * BN * 2;
  static constexpr int kStagingBufs = 2;
  static constexpr int kAuxBytes = 0;
  static constexpr bool kGroupCopy = true;
  static constexpr int kChunks = BN / 8;  // 16-byte chunks per staged row
  int64_t ld_out;
  int M, N;
  int route;  // 1: channels -> rows, 2: transpose
  int rank, route_rows, route_batch, route_n;
  void* dst[kMaxRoute];

  __device__ void load_aux(void*, uint64_t*, int, int, int) const {}
  __device__ void store(const EpiCtx&) const {}

  __device__ __forceinline__ uint4* chunk(uint8_t* base, int row, int q) const {
    return reinterpret_cast<uint4*>(base + row * (BN * 2) + ((q ^ (row % kChunks)) << 4));
  }

  __device__ void compute(const EpiCtx& c) const {
    constexpr int kHalf = BN / 2;
#pragma unroll 1
    for (int c0 = 0; c0 < kHalf; c0 += 16) {
      float v[16];
      tmem_ld16(c.tmem + c.half * kHalf + c0, v);
      const int q = (c.half * kHalf + c0) / 8;
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        uint4 w;
        w.x = pack_bf16x2(v[8 * h + 0], v[8 * h + 1]);
        w.y = pack_bf16x2(v[8 * h + 2], v[8 * h + 3]);
        w.z = pack_bf16x2(v[8 * h + 4], v[8 * h + 5]);
        w.w = pack_bf16x2(v[8 * h + 6], v[8 * h + 7]);
        *chunk(c.staging, c.row, q + h) = w;
      }
    }
  }

  __device__ void group_copy(const EpiCtx& c, int t) const {
    constexpr int kRowsPerStep = kGemmEpiThreads / kChunks;
    const int q = t % kChunks;
    const int col = c.n0 + q * 8;
    if (col >= N) return;
#pragma unroll 4
    for (int r = t / kChunks; r < 128; r += kRowsPerStep) {
      const int row = c.m0 + r;
      if (row >= M) break;
      int64_t off;
      int s;
      if (route == 1) {
        s = row / route_rows;
        off = (static_cast<int64_t>(rank * route_batch + c.bat) * route_rows +
               (row - s * route_rows)) * ld_out;
      } else {
        const int jj = row / route_n;
        const int i = row - jj * route_n;
        s = i / route_rows;
        off = (static_cast<int64_t>(i - s * route_rows) * route_n + rank * route_rows + jj) *
              ld_out;
      }
      *reinterpret_cast<uint4*>(static_cast<__nv_bfloat16*>(dst[s]) + off + col) =
          *chunk(c.staging, r, q);
    }
  }
};

// Gated linear unit.  The packed weight places, in every 128-wide tile, 64 gate
// units followed by the 64 value units of the same output columns.
//   h[row][n0/2 + j] = bf16( silu(gate_j) * value_j )
// Output map 3-D {hidden, M, 1}, box {64, 128, 1}, 128-byte swizzle.
struct EpiGLU {
  static constexpr int kStagingBytes = 128 * 64 * 2;
  static constexpr int kStagingBufs = 2;
  static constexpr int kAuxBytes = 0;
  CUtensorMap out_map;

  __device__ void load_aux(void*, uint64_t*, int, int, int) const {}

  __device__ void compute(const EpiCtx& c) const {
    float a[32], b[32];
    tmem_ld32(c.tmem + c.half * 32, a);
    tmem_ld32(c.tmem + 64 + c.half * 32, b);
#pragma unroll
    for (int i = 0; i < 32; ++i) a[i] = a[i] * sigmoid_fast(a[i]) * b[i];
    stage32_bf16_sw128(c.staging, c.row, c.half * 4, a);
  }

  __device__ void store(const EpiCtx& c) const {
    tma_store_3d(&out_map, c.staging, c.n0 / 2, c.m0, c.bat);
  }
};

// Triangle-multiplication input projection, batched over pair rows i (bat) with
// tiles of 128 columns j.  Packed weight rows per 128-wide tile t < n_proj_tiles:
// 64 projection channels [64t, 64t+64) then the 64 gate channels of the same
// indices; the last tile holds the c output-gate rows.
//   p_ch = proj_ch * mask[i][j] * sigmoid(gate_ch)
//   channel 2c' -> a[c'][i][j], channel 2c'+1 -> b[c'][i][j]   (a, b: [c][n][pitch])
//   g[i][j][c'] = sigmoid(x . w_gating[c'])
// a / b maps: 3-D {n (j), n (i), c}, box {128, 1, 32}, no swizzle;
// g map: 3-D {c, n (j), n (i)}, box {64, 128, 1}, 128-byte swizzle.
// With route = 1 (a row block of a row-sharded pair: pair row i = rank *
// route_rows + bat) a and b skip their maps: the store warp's lanes write
// channel ch straight into rank s = ch / route_cs's receive buffer
// a_dst[s] / b_dst[s] [route_cs][n][n] at [ch % route_cs][i][j] -- the rows ->
// channels exchange done by the producer.
struct EpiTriProj {
  static constexpr int kStagingBytes = 32768;
  static constexpr int kStagingBufs = 2;
  static constexpr int kGroups = 2;
  static constexpr int kAuxBytes = 0;
  static constexpr bool kGroupCopy = true;
  CUtensorMap a_map, b_map, g_map;
  const float* mask;  // [n][n] or null
  int n, n_proj_tiles, c;
  int route = 0;
  int rank, route_rows, route_cs;
  void* a_dst[kMaxRoute];
  void* b_dst[kMaxRoute];

  __device__ void load_aux(void*, uint64_t*, int, int, int) const {}

  // mask value of a row (1 when there is no mask or the row is past the end)
  __device__ __forceinline__ float row_mask(int bat, int j) const {
    return (mask != nullptr && j < n) ? __ldg(mask + static_cast<int64_t>(bat) * n + j) : 1.f;
  }

  // the tile row's mask value, loaded while the tile's MMAs run
  __device__ float2 prefetch(const EpiCtx& c) const {
    return make_float2(c.n0 / 128 < n_proj_tiles ? row_mask(c.bat, c.m0 + c.row) : 1.f, 0.f);
  }

  __device__ void compute(const EpiCtx& c) const {
    const int tile = c.n0 / 128;
    if (tile < n_proj_tiles) {
      const float mval = c.pre.x;
      __nv_bfloat16* sa = reinterpret_cast<__nv_bfloat16*>(c.staging);
      __nv_bfloat16* sb = sa + 32 * 128;
      // projection and gate columns with one TMEM round trip
      float pv[32], gv[32];
      tmem_ld32_nowait(c.tmem + c.half * 32, pv);
      tmem_ld32_nowait(c.tmem + 64 + c.half * 32, gv);
      tmem_ld_wait();
#pragma unroll
      for (int q = 0; q < 32; q += 2) {
        const int ch = c.half * 16 + q / 2;  // local a / b channel
        sa[ch * 128 + c.row] = __float2bfloat16_rn(pv[q] * mval * sigmoid_fast(gv[q]));
        sb[ch * 128 + c.row] = __float2bfloat16_rn(pv[q + 1] * mval * sigmoid_fast(gv[q + 1]));
      }
    } else {
      float v[64];
      tmem_ld32_nowait(c.tmem + c.half * 64, v);
      tmem_ld32_nowait(c.tmem + c.half * 64 + 32, v + 32);
      tmem_ld_wait();
#pragma unroll
      for (int i = 0; i < 64; ++i) v[i] = sigmoid_fast(v[i]);
      stage32_bf16_sw128(c.staging + c.half * 16384, c.row, 0, v);
      stage32_bf16_sw128(c.staging + c.half * 16384, c.row, 4, v + 32);
    }
  }

  __device__ void store(const EpiCtx& c) const {
    const int tile = c.n0 / 128;
    if (tile < n_proj_tiles) {
      if (route) return;  // group_copy wrote them
      tma_store_3d(&a_map, c.staging, c.m0, c.bat, tile * 32);
      tma_store_3d(&b_map, c.staging + 8192, c.m0, c.bat, tile * 32);
    } else {
      tma_store_3d(&g_map, c.staging, 0, c.m0, c.bat);
      if (this->c > 64) tma_store_3d(&g_map, c.staging + 16384, 64, c.m0, c.bat);
    }
  }

  // a / b tile [32 channels][128 j] bf16 each: 16-byte pieces, channel by
  // channel, into the owners' receive buffers (n % 8 == 0, so a piece never
  // straddles the end of a row); 16 threads write one channel's 256 bytes
  __device__ void group_copy(const EpiCtx& c, int t) const {
    const int tile = c.n0 / 128;
    if (!route || tile >= n_proj_tiles) return;
    const int64_t i = static_cast<int64_t>(rank) * route_rows + c.bat;
#pragma unroll
    for (int idx = t; idx < 2 * 32 * 16; idx += kGemmEpiThreads) {
      const int which = idx >> 9;  // 0: a, 1: b
      const int ch = (idx >> 4) & 31;
      const int piece = idx & 15;
      const int j = c.m0 + piece * 8;
      if (j >= n) continue;
      const int gch = tile * 32 + ch;
      const int s = gch / route_cs;
      const uint4 v =
          *reinterpret_cast<const uint4*>(c.staging + which * 8192 + (ch * 128 + piece * 8) * 2);
      __nv_bfloat16* base = static_cast<__nv_bfloat16*>(which ? b_dst[s] : a_dst[s]);
      *reinterpret_cast<uint4*>(base + (static_cast<int64_t>(gch - s * route_cs) * n + i) * n + j) =
          v;
    }
  }
};

// Triangle-attention input projection for c = 128, 4 heads of 32, batched over
// pair rows i with tiles of 128 columns j.  Packed weight rows: q, k, v, gate
// (128 each).  Position (i, j) is batch row r = i, token t = j (starting node)
// or r = j, t = i (ending node).
//   q/k/v[r][h][t][0..31]  (q = bf16(acc) * q_scale before its own rounding)
//   g[i][j][col] = sigmoid(x . w_gate[col])
// q/k/v maps: starting 3-D {32, n (t), n*4 (r*4+h)}, box {32, 128, 1};
// ending 4-D {32, n (t), 4 (h), n (r)}, box {32, 1, 1, 128}; 64-byte swizzle.
struct EpiAttProjTma {
  static constexpr int kStagingBytes = 32768;
  static constexpr int kStagingBufs = 2;
  static constexpr int kAuxBytes = 0;
  CUtensorMap qkv_map[3];
  CUtensorMap g_map;
  float q_scale;
  int transpose;

  __device__ void load_aux(void*, uint64_t*, int, int, int) const {}

  __device__ void compute(const EpiCtx& c) const {
    const int which = c.n0 / 128;  // 0 q, 1 k, 2 v, 3 gate
    float v[32];
#pragma unroll
    for (int h2 = 0; h2 < 2; ++h2) {
      tmem_ld32(c.tmem + c.half * 64 + h2 * 32, v);
      if (which == 3) {
#pragma unroll
        for (int i = 0; i < 32; ++i) v[i] = sigmoid_fast(v[i]);
        stage32_bf16_sw128(c.staging + c.half * 16384, c.row, h2 * 4, v);
      } else {
        if (which == 0) {
#pragma unroll
          for (int i = 0; i < 32; ++i) v[i] = bf16r(v[i]) * q_scale;
        }
        uint8_t* head = c.staging + (c.half * 2 + h2) * 8192;  // [128 t][64 B]
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          uint4 w;
          w.x = pack_bf16x2(v[8 * q + 0], v[8 * q + 1]);
          w.y = pack_bf16x2(v[8 * q + 2], v[8 * q + 3]);
          w.z = pack_bf16x2(v[8 * q + 4], v[8 * q + 5]);
          w.w = pack_bf16x2(v[8 * q + 6], v[8 * q + 7]);
          *reinterpret_cast<uint4*>(sw64_chunk(head, c.row, q)) = w;
        }
      }
    }
  }

  __device__ void store(const EpiCtx& c) const {
    const int which = c.n0 / 128;
    if (which == 3) {
      tma_store_3d(&g_map, c.staging, 0, c.m0, c.bat);
      tma_store_3d(&g_map, c.staging + 16384, 64, c.m0, c.bat);
      return;
    }
#pragma unroll
    for (int h = 0; h < 4; ++h) {
      const uint8_t* src = c.staging + h * 8192;
      if (!transpose) {
        tma_store_3d(&qkv_map[which], src, 0, c.m0, c.bat * 4 + h);
      } else {
        tma_store_4d(&qkv_map[which], src, 0, c.bat, h, c.m0);
      }
    }
  }
};

// Attention input projection with direct stores, any c / head layout: the
// single-track and diffusion SelfAttention (one batch row) and the c = 64
// triangle attention.  Flat rows: position pos = i*n + j with batch row
// i (starting) or j (ending); q/k/v[r][h][t][dd] with head pitch dp >= d
// (padding left as is), q = bf16(bf16(acc + q_bias) * q_scale).
struct EpiAttProjDirect {
  static constexpr int kStagingBytes = 0;
  static constexpr int kStagingBufs = 1;
  static constexpr int kAuxBytes = 0;
  __nv_bfloat16* q;
  __nv_bfloat16* k;
  __nv_bfloat16* v;
  __nv_bfloat16* g;
  int n, c, heads, d, dp;
  int transpose;
  int M;
  float q_scale;
  const float* q_bias;

  __device__ void load_aux(void*, uint64_t*, int, int, int) const {}
  __device__ void store(const EpiCtx&) const {}

  __device__ void compute(const EpiCtx& cx) const {
    const int row = cx.m0 + cx.row;
    const bool row_ok = row < M;
    const int pos = row_ok ? row : 0;
    const int i = pos / n;
    const int j = pos - i * n;
    const int bidx = transpose ? j : i;
    const int tok = transpose ? i : j;
#pragma unroll 1
    for (int c0 = 0; c0 < 64; c0 += 16) {
      float x[16];
      tmem_ld16(cx.tmem + cx.half * 64 + c0, x);
      const int colg = cx.n0 + cx.half * 64 + c0;
      const int which = colg / c;
      const int cc = colg - which * c;
      if (!row_ok || which > 3) continue;
      if (which == 3) {
#pragma unroll
        for (int e = 0; e < 16; ++e) x[e] = sigmoid_fast(x[e]);
        store16_bf16(g + static_cast<int64_t>(pos) * c + cc, x);
        continue;
      }
      __nv_bfloat16* base = which == 0 ? q : (which == 1 ? k : v);
#pragma unroll
      for (int e = 0; e < 16; ++e) {
        if (which == 0) {
          const float qb = q_bias ? q_bias[cc + e] : 0.f;
          x[e] = bf16r(x[e] + qb) * q_scale;
        }
      }
#pragma unroll
      for (int e = 0; e < 16; ++e) {
        const int col = cc + e;
        const int h = col / d;
        const int dd = col - h * d;
        base[((static_cast<int64_t>(bidx) * heads + h) * n + tok) * dp + dd] =
            __float2bfloat16_rn(x[e]);
      }
    }
  }
};

// Conditioning projections of a diffusion step (AdaLN scale / shift and the
// AdaLNZero gates of every block at once): out = act(x W^T + b), bf16.  The N
// output columns are cut into chunks of `chunk` columns stored one after
// another, [N / chunk][M][chunk], so each block's tensor is contiguous; act is
// the logistic function on every chunk (sig_mode 2), on the even chunks
// (sig_mode 1: [scale, shift] pairs) or nowhere (0).  The tile is staged like
// EpiOut's (64-column 128B-swizzled boxes) and each box goes out with one TMA
// store at (column within its chunk, m0, chunk): `chunk` is a multiple of 64 so
// no box straddles two chunks, and out_map is the 3-D view {chunk, M, N/chunk}.
template <int BN>
struct EpiCondTma : EpiOut<BN, false> {
  static constexpr int kStagingBufs = 2;
  int chunk, sig_mode;

  __device__ void compute(const EpiCtx& c) const {
    constexpr int kHalf = BN / 2;
#pragma unroll 1
    for (int c0 = 0; c0 < kHalf; c0 += 16) {
      const int col = c.half * kHalf + c0;
      float v[16];
      tmem_ld16(c.tmem + col, v);
      const int q = (c.n0 + col) / chunk;
      const bool sig = sig_mode == 2 || (sig_mode == 1 && (q & 1) == 0);
      float bb[16];
      if (this->bias != nullptr) {  // 16-byte aligned (checked by the launcher)
        const float4* b4 = reinterpret_cast<const float4*>(this->bias + c.n0 + col);
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const float4 w = __ldg(b4 + k);
          bb[4 * k] = w.x;
          bb[4 * k + 1] = w.y;
          bb[4 * k + 2] = w.z;
          bb[4 * k + 3] = w.w;
        }
      } else {
#pragma unroll
        for (int i = 0; i < 16; ++i) bb[i] = 0.f;
      }
      if (sig) {
#pragma unroll
        for (int i = 0; i < 16; ++i) v[i] = sigmoid_ex2(bf16r(v[i] + bb[i]));
      } else {
#pragma unroll
        for (int i = 0; i < 16; ++i) v[i] = bf16r(v[i] + bb[i]);
      }
      this->write(c, col, v);
    }
  }

  __device__ void store(const EpiCtx& c) const {
#pragma unroll
    for (int b = 0; b < BN / 64; ++b) {
      const int n = c.n0 + b * 64;
      tma_store_3d(&this->out_map, c.staging + b * (128 * 128), n % chunk, c.m0, n / chunk);
    }
  }
};

}  // namespace xfb
