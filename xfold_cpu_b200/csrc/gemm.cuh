// Persistent, warp-specialised bf16 GEMM on tcgen05 for sm_100a.
//
//   D[bat][m][n] = sum_k A[bat](m, k) * B[bat](n, k)        (f32 accumulate in TMEM)
//
// A and B are read by TMA into 128-byte-swizzled shared-memory stages.  Each
// operand is either K-major (K contiguous in global memory, e.g. activations
// [rows][K] and nn.Linear weights [out][in]) or MN-major (M/N contiguous, the
// layout the incoming triangle contraction reads its operands in).
//
// Warp roles (192 threads, one CTA per SM):
//   warps 0-3  epilogue: TMEM lane quarter w, one accumulator row per thread
//   warp 4     TMA producer (one elected lane)
//   warp 5     TMEM allocator + MMA issuer (one elected lane)
// The accumulator is double-buffered in TMEM (2 x BN columns), so the epilogue
// of tile i overlaps the main loop of tile i+1.
#pragma once

#include "common.cuh"

namespace xfb {

constexpr int kGemmBM = 128;
constexpr int kGemmBK = 64;  // one 128-byte swizzle atom of bf16
constexpr int kGemmThreads = 192;

struct GemmShape {
  int M, N, K, batch;
  int m_tiles, n_tiles, k_blocks;
};

// What an epilogue functor sees for one accumulator row of one tile.
struct EpiRow {
  int bat;         // batch index
  int m0, n0;      // tile origin
  int row;         // global row index (m0 + lane row); may be >= M for tail tiles
  uint32_t tmem;   // TMEM address of column 0 of this thread's accumulator row
};

template <int BN, int STAGES>
struct GemmSmem {
  static constexpr int kABytes = kGemmBM * kGemmBK * 2;
  static constexpr int kBBytes = BN * kGemmBK * 2;
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kBarrierOffset = STAGES * kStageBytes;
  // full[S], empty[S], tfull[2], tempty[2], tmem slot, abort flag
  static constexpr int kTotal = kBarrierOffset + (2 * STAGES + 4) * 8 + 16;
  static constexpr int kLaunchBytes = kTotal + 1024;  // slack for 1024-byte alignment
};

template <int BN, int STAGES, bool A_MN, bool B_MN, class Epi>
__global__ void __launch_bounds__(kGemmThreads, 1)
    gemm_bf16_kernel(const __grid_constant__ CUtensorMap tmA,
                     const __grid_constant__ CUtensorMap tmB, GemmShape shape, Epi epi) {
  static_assert(BN % 64 == 0 && BN >= 64 && BN <= 256, "BN must be 64, 128, 192 or 256");
  using L = GemmSmem<BN, STAGES>;
  constexpr uint32_t kTmemCols = (2 * BN <= 256) ? 256 : 512;
  constexpr uint32_t kIdesc = idesc_bf16(kGemmBM, BN, A_MN, B_MN);

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L::kBarrierOffset);
  uint64_t* empty = full + STAGES;
  uint64_t* tfull = empty + STAGES;
  uint64_t* tempty = tfull + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty + 2);
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
      mbar_init(&tempty[b], 128);
    }
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 5) {
    tmem_alloc(tmem_slot, kTmemCols);
    tmem_relinquish();
  }
  if (warp == 4 && lane == 0) {
    tma_prefetch(&tmA);
    tma_prefetch(&tmB);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  const int tiles_per_batch = shape.m_tiles * shape.n_tiles;
  const int total_tiles = tiles_per_batch * shape.batch;

  if (warp == 4) {
    // ------------------------------------------------ TMA producer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      for (int tile = blockIdx.x; tile < total_tiles && !*abort_flag; tile += gridDim.x) {
        const int bat = tile / tiles_per_batch;
        const int rem = tile - bat * tiles_per_batch;
        const int m0 = (rem / shape.n_tiles) * kGemmBM;
        const int n0 = (rem % shape.n_tiles) * BN;
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
              tma_load_3d(sB + c * 8192, &tmB, &full[stage], n0 + 64 * c, k0, bat);
          } else {
            tma_load_3d(sB, &tmB, &full[stage], k0, n0, bat);
          }
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
    }
  } else if (warp == 5) {
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
  } else {
    // ------------------------------------------------ epilogue warps 0-3
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int tile = blockIdx.x; tile < total_tiles; tile += gridDim.x) {
      const int bat = tile / tiles_per_batch;
      const int rem = tile - bat * tiles_per_batch;
      const int m0 = (rem / shape.n_tiles) * kGemmBM;
      const int n0 = (rem % shape.n_tiles) * BN;
      if (!mbar_wait(&tfull[acc], acc_phase, kErrWaitEpilogue, abort_flag)) break;
      tc_fence_after();
      EpiRow r;
      r.bat = bat;
      r.m0 = m0;
      r.n0 = n0;
      r.row = m0 + warp * 32 + lane;
      r.tmem = tmem_base + (static_cast<uint32_t>(warp * 32) << 16) + acc * BN;
      epi(r);
      tc_fence_before();
      mbar_arrive(&tempty[acc]);
      if (++acc == 2) {
        acc = 0;
        acc_phase ^= 1;
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 5) {
    tc_fence_after();
    tmem_dealloc(tmem_base, kTmemCols);
  }
}

// ====================================================================== epilogues
//
// Each functor is called once per accumulator row by all 128 epilogue threads.
// TMEM loads are warp-collective, so every thread loads even when its row is
// past M; only the global stores are guarded.

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

__device__ __forceinline__ void load16_bf16(const __nv_bfloat16* src, float (&v)[16]) {
  const uint4 a = reinterpret_cast<const uint4*>(src)[0];
  const uint4 b = reinterpret_cast<const uint4*>(src)[1];
  const uint32_t w[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    v[2 * i] = __uint_as_float(w[i] << 16);
    v[2 * i + 1] = __uint_as_float(w[i] & 0xFFFF0000u);
  }
}

// out[bat][row][col] (=|+=) bf16(acc + bias) [* gate, rounded to bf16]
// The projection result is a bf16 tensor in the autocast reference, hence the
// rounding before the gate product and before the f32 residual add.
template <int BN>
struct EpiLinear {
  void* out;
  int64_t ld_out;
  int64_t bstride_out;
  int out_f32;       // 1: f32 output, 0: bf16 output
  int accumulate;    // 1: out (f32) += value
  const float* bias;          // [N] or null
  const __nv_bfloat16* gate;  // [M][ld_gate] (already squashed) or null
  int64_t ld_gate;
  int M, N;

  __device__ void operator()(const EpiRow& r) const {
    const bool row_ok = r.row < M;
    const int64_t row_off = r.bat * bstride_out + static_cast<int64_t>(r.row) * ld_out;
    const __nv_bfloat16* grow = gate ? gate + static_cast<int64_t>(r.row) * ld_gate : nullptr;
#pragma unroll 1
    for (int c0 = 0; c0 < BN; c0 += 16) {
      float v[16];
      tmem_ld16(r.tmem + c0, v);
      const int col = r.n0 + c0;
      if (!row_ok || col >= N) continue;
      const bool full = col + 16 <= N;
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        float x = v[i];
        if (bias != nullptr && (full || col + i < N)) x += bias[col + i];
        v[i] = bf16r(x);
      }
      if (grow != nullptr) {
        float g[16];
        if (full) {
          load16_bf16(grow + col, g);
        } else {
#pragma unroll
          for (int i = 0; i < 16; ++i)
            g[i] = (col + i < N) ? __bfloat162float(grow[col + i]) : 0.f;
        }
#pragma unroll
        for (int i = 0; i < 16; ++i) v[i] = bf16r(v[i] * g[i]);
      }
      if (out_f32) {
        float* orow = reinterpret_cast<float*>(out) + row_off;
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
        __nv_bfloat16* orow = reinterpret_cast<__nv_bfloat16*>(out) + row_off;
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

// Gated linear unit: the packed weight places, in every BN-wide tile, BN/2 gate
// units followed by the BN/2 value units of the same output columns.
//   out[row][n0/2 + j] = bf16( bf16(silu(bf16(gate_j))) * bf16(value_j) )
template <int BN>
struct EpiGLU {
  __nv_bfloat16* out;
  int64_t ld_out;
  int M, N_out;  // N_out = hidden width (half the packed weight rows)

  __device__ void operator()(const EpiRow& r) const {
    const bool row_ok = r.row < M;
    __nv_bfloat16* orow = out + static_cast<int64_t>(r.row) * ld_out;
    const int ocol0 = r.n0 / 2;
#pragma unroll 1
    for (int c0 = 0; c0 < BN / 2; c0 += 16) {
      float a[16], b[16];
      tmem_ld16(r.tmem + c0, a);
      tmem_ld16(r.tmem + BN / 2 + c0, b);
      const int col = ocol0 + c0;
      if (!row_ok || col >= N_out) continue;
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        const float g = bf16r(a[i]);
        const float act = bf16r(g * sigmoidf_stable(g));
        a[i] = bf16r(act * bf16r(b[i]));
      }
      if (col + 16 <= N_out) {
        store16_bf16(orow + col, a);
      } else {
#pragma unroll
        for (int i = 0; i < 16; ++i)
          if (col + i < N_out) orow[col + i] = __float2bfloat16_rn(a[i]);
      }
    }
  }
};

// Triangle-multiplication input projection.  Packed weight rows per 128-wide
// tile t < n_proj_tiles: 64 projection channels [64t, 64t+64) then the 64 gate
// channels with the same indices; the last tile holds the c output-gate rows.
//   p_ch = bf16( bf16(bf16(proj_ch) * mask) * bf16(sigmoid(bf16(gate_ch))) )
//   channel 2c -> a[c][i][j], channel 2c+1 -> b[c][i][j]   (a, b row pitch `pitch`)
//   g[pos][c'] = bf16(sigmoid(bf16(x . w_gating[c'])))
struct EpiTriProj {
  __nv_bfloat16* a;
  __nv_bfloat16* b;
  __nv_bfloat16* g;
  const float* mask;  // [n][n] or nullptr
  int64_t chan_stride;  // elements between channels of a / b (n * pitch)
  int n, pitch, c;      // pair side, padded row pitch of a/b, channels
  int M;                // n * n
  int n_proj_tiles;     // 2c / 64

  __device__ void operator()(const EpiRow& r) const {
    const bool row_ok = r.row < M;
    const int tile = r.n0 / 128;
    const int pos = row_ok ? r.row : 0;
    if (tile < n_proj_tiles) {
      const int i = pos / n;
      const int j = pos - i * n;
      const float mval = (mask != nullptr && row_ok) ? mask[pos] : 1.f;
      const int64_t poff = static_cast<int64_t>(i) * pitch + j;
#pragma unroll 1
      for (int c0 = 0; c0 < 64; c0 += 16) {
        float pv[16], gv[16];
        tmem_ld16(r.tmem + c0, pv);
        tmem_ld16(r.tmem + 64 + c0, gv);
        if (!row_ok) continue;
#pragma unroll
        for (int q = 0; q < 16; ++q) {
          const int ch = tile * 64 + c0 + q;
          const float p = bf16r(bf16r(pv[q]) * mval);
          const float s = bf16r(sigmoidf_stable(bf16r(gv[q])));
          const __nv_bfloat16 val = __float2bfloat16_rn(p * s);
          __nv_bfloat16* dst = ((ch & 1) ? b : a) + (ch >> 1) * chan_stride + poff;
          *dst = val;
        }
      }
    } else {
      __nv_bfloat16* grow = g + static_cast<int64_t>(pos) * c;
#pragma unroll 1
      for (int c0 = 0; c0 < 128; c0 += 16) {
        float v[16];
        tmem_ld16(r.tmem + c0, v);
        if (!row_ok || c0 >= c) continue;
#pragma unroll
        for (int q = 0; q < 16; ++q) v[q] = bf16r(sigmoidf_stable(bf16r(v[q])));
        store16_bf16(grow + c0, v);
      }
    }
  }
};

// Triangle-attention input projection.  Packed weight rows: q (c), k (c), v (c),
// gate (c), in 128-wide tiles.  Position pos = i*n + j belongs to batch row
// b = i, token t = j (starting node) or b = j, t = i (ending node).
//   q/k/v[b][h][t][dd] (head pitch dp >= d, padding left untouched)
//   q is scaled by d^-0.5 after rounding, as the reference scales the bf16 q.
//   g[pos][col] = bf16(sigmoid(bf16(x . w_gate[col])))
struct EpiAttProj {
  __nv_bfloat16* q;
  __nv_bfloat16* k;
  __nv_bfloat16* v;
  __nv_bfloat16* g;
  int n, c, heads, d, dp;
  int transpose;
  int M;
  float q_scale;
  const float* q_bias;  // [c] or null: bias of the q projection (SelfAttention)

  __device__ void operator()(const EpiRow& r) const {
    const bool row_ok = r.row < M;
    const int pos = row_ok ? r.row : 0;
    const int i = pos / n;
    const int j = pos - i * n;
    const int bidx = transpose ? j : i;
    const int tok = transpose ? i : j;
#pragma unroll 1
    for (int c0 = 0; c0 < 128; c0 += 16) {
      float x[16];
      tmem_ld16(r.tmem + c0, x);
      const int colg = r.n0 + c0;  // column of the packed [q|k|v|gate] output
      const int which = colg / c;  // 0 q, 1 k, 2 v, 3 gate
      const int cc = colg - which * c;
      if (!row_ok || which > 3) continue;
      if (which == 3) {
#pragma unroll
        for (int e = 0; e < 16; ++e) x[e] = bf16r(sigmoidf_stable(bf16r(x[e])));
        store16_bf16(g + static_cast<int64_t>(pos) * c + cc, x);
        continue;
      }
      __nv_bfloat16* base = which == 0 ? q : (which == 1 ? k : v);
#pragma unroll
      for (int e = 0; e < 16; ++e) {
        if (which == 0) {
          const float qb = q_bias ? q_bias[cc + e] : 0.f;
          x[e] = bf16r(bf16r(x[e] + qb) * q_scale);
        } else {
          x[e] = bf16r(x[e]);
        }
      }
      if (d % 16 == 0) {
        const int h = cc / d;
        const int dd = cc - h * d;
        __nv_bfloat16* dst =
            base + ((static_cast<int64_t>(bidx) * heads + h) * n + tok) * dp + dd;
        store16_bf16(dst, x);
      } else {
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
  }
};

}  // namespace xfb
