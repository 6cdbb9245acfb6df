// LayerNorm kernels (HBM-bound, one pass over the input).
//
// ln_rows_kernel: one warp per row of C channels, vectorised 16-byte loads,
//   f32 statistics (mean, then variance of the centred values) with warp
//   shuffles.  Writes bf16 y = LN(x)*w + b, optionally followed by the
//   adaptive modulation y = scale*y + shift, and optionally a small head
//   projection heads[h][row] = sum_c y[c] * wh[h][c] (the pair-bias / pair-logit
//   projections, H <= 16) reduced with a transposing butterfly.
//
// ln_channel_major_kernel: one thread per position of a channel-major
//   [C][rows][pitch] bf16 tensor (the triangle contraction output, n valid
//   columns); writes the normalised row-major [rows*n][C] bf16 tensor the output
//   projection reads.
#pragma once

#include "common.cuh"

namespace xfb {

template <typename T>
__device__ __forceinline__ void load_vec4(const T* p, float (&v)[4]);

template <>
__device__ __forceinline__ void load_vec4<float>(const float* p, float (&v)[4]) {
  const float4 a = *reinterpret_cast<const float4*>(p);
  v[0] = a.x;
  v[1] = a.y;
  v[2] = a.z;
  v[3] = a.w;
}

template <>
__device__ __forceinline__ void load_vec4<__nv_bfloat16>(const __nv_bfloat16* p, float (&v)[4]) {
  const uint2 a = *reinterpret_cast<const uint2*>(p);
  v[0] = __uint_as_float(a.x << 16);
  v[1] = __uint_as_float(a.x & 0xFFFF0000u);
  v[2] = __uint_as_float(a.y << 16);
  v[3] = __uint_as_float(a.y & 0xFFFF0000u);
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

struct LnArgs {
  const void* x;
  int64_t rows;
  int64_t ldx;
  const float* w;      // [C] or null (no affine)
  const float* b;      // [C] or null
  float eps;
  __nv_bfloat16* y;    // [rows][ldy] or null
  int64_t ldy;
  const __nv_bfloat16* mod_scale;  // [rows][C] (already squashed) or null
  const __nv_bfloat16* mod_shift;  // [rows][C] or null
  const __nv_bfloat16* wh;         // head projection [H][C] or null
  int heads;
  __nv_bfloat16* head_out;         // [H][head_ld]
  int64_t head_ld;
  float head_scale;                // multiplies the head projection before rounding
  const int64_t* gather_idx;       // [rows] source row of each output row, or null
  const uint8_t* gather_valid;     // [rows] zero = the output row reads zeros; or null
  int64_t src_rows;                // rows of x that gather_idx may address
  int64_t perm_outer, perm_inner;  // > 0: input row b*inner + k writes y row k*outer + b
  // ln_heads_tc_kernel only: with route = 1, y row r = i * route_n + j (pair row
  // i of this rank's block, column j) goes to rank s = j / route_rows as row
  // (j % route_rows) * route_n + route_rank * route_rows + i of y_dst[s] -- the
  // row <-> column transpose of a row-sharded pair, done by the producer.
  int route = 0;
  int route_rank, route_rows, route_n;
  __nv_bfloat16* y_dst[16];
};

// C = 32 * 4 * R channels: each lane holds R groups of 4 consecutive channels.
template <int C, typename InT, int HP>
__global__ void __launch_bounds__(256) ln_rows_kernel(LnArgs a) {
  static_assert(C % 128 == 0 || C == 64, "C must be 64 or a multiple of 128");
  constexpr int R = (C >= 128) ? C / 128 : 1;
  constexpr int V = (C >= 128) ? 4 : 2;  // channels per group
  const int lane = threadIdx.x & 31;
  const int64_t warps_total = static_cast<int64_t>(gridDim.x) * (blockDim.x >> 5);
  const int64_t warp_id = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);

  // Head projection weights for this lane's channels (loaded once per warp).
  float whr[HP > 0 ? HP : 1][R][V];
  if constexpr (HP > 0) {
#pragma unroll
    for (int h = 0; h < HP; ++h)
#pragma unroll
      for (int r = 0; r < R; ++r)
#pragma unroll
        for (int e = 0; e < V; ++e) {
          const int ch = r * 32 * V + lane * V + e;
          whr[h][r][e] = (h < a.heads) ? __bfloat162float(a.wh[h * C + ch]) : 0.f;
        }
  }
  float wv[R][V], bv[R][V];
#pragma unroll
  for (int r = 0; r < R; ++r)
#pragma unroll
    for (int e = 0; e < V; ++e) {
      const int ch = r * 32 * V + lane * V + e;
      wv[r][e] = a.w ? a.w[ch] : 1.f;
      bv[r][e] = a.b ? a.b[ch] : 0.f;
    }

  for (int64_t row = warp_id; row < a.rows; row += warps_total) {
    // optional row gather (the atom layout's queries -> keys): masked-out rows
    // and indices outside the source read zeros
    int64_t src = row;
    bool zero = false;
    if (a.gather_idx != nullptr) {
      src = a.gather_idx[row];
      zero = a.gather_valid != nullptr && a.gather_valid[row] == 0;
      if (!zero && (src < 0 || src >= a.src_rows)) {
        if (lane == 0) record_error(kErrIndex);
        zero = true;
      }
      if (zero) src = 0;
    }
    const InT* xr = reinterpret_cast<const InT*>(a.x) + src * a.ldx;
    float v[R][V];
#pragma unroll
    for (int r = 0; r < R; ++r) {
      const int ch = r * 32 * V + lane * V;
      if (zero) {
#pragma unroll
        for (int e = 0; e < V; ++e) v[r][e] = 0.f;
      } else if constexpr (V == 4) {
        load_vec4<InT>(xr + ch, v[r]);
      } else {
        v[r][0] = static_cast<float>(xr[ch]);
        v[r][1] = static_cast<float>(xr[ch + 1]);
      }
    }
    float s = 0.f;
#pragma unroll
    for (int r = 0; r < R; ++r)
#pragma unroll
      for (int e = 0; e < V; ++e) s += v[r][e];
    const float mean = warp_sum(s) * (1.f / C);
    float ss = 0.f;
#pragma unroll
    for (int r = 0; r < R; ++r)
#pragma unroll
      for (int e = 0; e < V; ++e) {
        const float dlt = v[r][e] - mean;
        ss += dlt * dlt;
      }
    const float var = warp_sum(ss) * (1.f / C);
    const float rstd = rsqrtf(var + a.eps);
#pragma unroll
    for (int r = 0; r < R; ++r)
#pragma unroll
      for (int e = 0; e < V; ++e) v[r][e] = (v[r][e] - mean) * rstd * wv[r][e] + bv[r][e];

    if (a.mod_scale != nullptr) {
#pragma unroll
      for (int r = 0; r < R; ++r)
#pragma unroll
        for (int e = 0; e < V; ++e) {
          const int64_t off = row * C + r * 32 * V + lane * V + e;
          const float sc = __bfloat162float(a.mod_scale[off]);
          const float sh = a.mod_shift ? __bfloat162float(a.mod_shift[off]) : 0.f;
          v[r][e] = sc * v[r][e] + sh;
        }
    }
    // bf16 rounding of the normalised activations (the GEMM input)
#pragma unroll
    for (int r = 0; r < R; ++r)
#pragma unroll
      for (int e = 0; e < V; ++e) v[r][e] = bf16r(v[r][e]);

    if (a.y != nullptr) {
      const int64_t yrow =
          a.perm_outer > 0 ? (row % a.perm_inner) * a.perm_outer + row / a.perm_inner : row;
      __nv_bfloat16* yr = a.y + yrow * a.ldy;
#pragma unroll
      for (int r = 0; r < R; ++r) {
        const int ch = r * 32 * V + lane * V;
        if constexpr (V == 4) {
          uint2 w;
          w.x = pack_bf16x2(v[r][0], v[r][1]);
          w.y = pack_bf16x2(v[r][2], v[r][3]);
          *reinterpret_cast<uint2*>(yr + ch) = w;
        } else {
          *reinterpret_cast<uint32_t*>(yr + ch) = pack_bf16x2(v[r][0], v[r][1]);
        }
      }
    }

    if constexpr (HP > 0) {
      float p[HP];
#pragma unroll
      for (int h = 0; h < HP; ++h) {
        float acc = 0.f;
#pragma unroll
        for (int r = 0; r < R; ++r)
#pragma unroll
          for (int e = 0; e < V; ++e) acc = fmaf(v[r][e], whr[h][r][e], acc);
        p[h] = acc;
      }
      // Transposing butterfly: after log2(HP) halving steps lane L holds head
      // bits taken from lane bits 4, 3, ... ; the remaining steps sum the rest.
      int off = 16;
#pragma unroll
      for (int w = HP / 2; w >= 1; w >>= 1) {
        const bool upper = (lane & off) != 0;
#pragma unroll
        for (int i = 0; i < w; ++i) {
          const float send = upper ? p[i] : p[i + w];
          const float keep = upper ? p[i + w] : p[i];
          p[i] = keep + __shfl_xor_sync(0xffffffffu, send, off);
        }
        off >>= 1;
      }
      float tot = p[0];
      for (int o = off; o >= 1; o >>= 1) tot += __shfl_xor_sync(0xffffffffu, tot, o);
      // lane L now holds head index formed by its top log2(HP) bits (bit 4 first)
      const int shift = 5 - __ffs(HP) + 1;  // number of low bits summed away
      if ((lane & ((1 << shift) - 1)) == 0) {
        const int hidx = lane >> shift;
        if (hidx < a.heads)
          a.head_out[hidx * a.head_ld + row] = __float2bfloat16_rn(tot * a.head_scale);
      }
    }
  }
}

// LayerNorm of 128-wide rows into bf16 y, without head projection, gather,
// permutation or modulation (the pair LayerNorms before the triangle
// multiplication and the transition): ln_rows_kernel's arithmetic, but each
// warp takes K rows per step so K rows' loads are in flight.
template <typename InT, int K>
__global__ void __launch_bounds__(256) ln_rows128_multi_kernel(LnArgs a) {
  const int lane = threadIdx.x & 31;
  const int64_t warps_total = static_cast<int64_t>(gridDim.x) * (blockDim.x >> 5);
  const int64_t warp_id = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
  float wv[4], bv[4];
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    wv[e] = a.w ? a.w[lane * 4 + e] : 1.f;
    bv[e] = a.b ? a.b[lane * 4 + e] : 0.f;
  }
  for (int64_t r0 = K * warp_id; r0 < a.rows; r0 += K * warps_total) {
    float v[K][4];
#pragma unroll
    for (int k = 0; k < K; ++k) {
      if (r0 + k < a.rows) {
        load_vec4<InT>(reinterpret_cast<const InT*>(a.x) + (r0 + k) * a.ldx + lane * 4, v[k]);
      } else {
        v[k][0] = v[k][1] = v[k][2] = v[k][3] = 0.f;
      }
    }
    float mean[K], rstd[K];
#pragma unroll
    for (int k = 0; k < K; ++k) {
      float s = 0.f;
#pragma unroll
      for (int e = 0; e < 4; ++e) s += v[k][e];
      mean[k] = warp_sum(s) * (1.f / 128);
    }
#pragma unroll
    for (int k = 0; k < K; ++k) {
      float ss = 0.f;
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float dlt = v[k][e] - mean[k];
        ss += dlt * dlt;
      }
      rstd[k] = rsqrtf(warp_sum(ss) * (1.f / 128) + a.eps);
    }
#pragma unroll
    for (int k = 0; k < K; ++k) {
      if (r0 + k >= a.rows) break;
      float o[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) o[e] = bf16r((v[k][e] - mean[k]) * rstd[k] * wv[e] + bv[e]);
      uint2 w;
      w.x = pack_bf16x2(o[0], o[1]);
      w.y = pack_bf16x2(o[2], o[3]);
      *reinterpret_cast<uint2*>(a.y + (r0 + k) * a.ldy + lane * 4) = w;
    }
  }
}

// LayerNorm of 64-wide rows without a head projection: four rows per warp at a
// time (8 lanes per row, 8 channels per lane), so a warp keeps four rows'
// loads in flight; statistics by 3-step shuffles within the 8 lanes.  Same
// arithmetic and options (gather, modulation, output-row permutation) as
// ln_rows_kernel.
template <typename InT>
__global__ void __launch_bounds__(256) ln_rows64_kernel(LnArgs a) {
  const int lane = threadIdx.x & 31;
  const int sub = lane & 7;   // channels 8*sub .. 8*sub+7
  const int grp = lane >> 3;  // which of the warp's four rows
  const int64_t warps_total = static_cast<int64_t>(gridDim.x) * (blockDim.x >> 5);
  const int64_t warp_id = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
  float wv[8], bv[8];
#pragma unroll
  for (int e = 0; e < 8; ++e) {
    wv[e] = a.w ? a.w[sub * 8 + e] : 1.f;
    bv[e] = a.b ? a.b[sub * 8 + e] : 0.f;
  }
  for (int64_t row0 = warp_id * 4; row0 < a.rows; row0 += warps_total * 4) {
    const int64_t row = row0 + grp;
    const bool live = row < a.rows;
    int64_t src = row;
    bool zero = !live;
    if (live && a.gather_idx != nullptr) {
      src = a.gather_idx[row];
      zero = a.gather_valid != nullptr && a.gather_valid[row] == 0;
      if (!zero && (src < 0 || src >= a.src_rows)) {
        if (sub == 0) record_error(kErrIndex);
        zero = true;
      }
    }
    float v[8];
    if (zero) {
#pragma unroll
      for (int e = 0; e < 8; ++e) v[e] = 0.f;
    } else {
      const InT* xr = reinterpret_cast<const InT*>(a.x) + src * a.ldx + sub * 8;
      float q[4];
      load_vec4<InT>(xr, q);
      v[0] = q[0], v[1] = q[1], v[2] = q[2], v[3] = q[3];
      load_vec4<InT>(xr + 4, q);
      v[4] = q[0], v[5] = q[1], v[6] = q[2], v[7] = q[3];
    }
    float s = 0.f;
#pragma unroll
    for (int e = 0; e < 8; ++e) s += v[e];
#pragma unroll
    for (int o = 4; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    const float mean = s * (1.f / 64);
    float ss = 0.f;
#pragma unroll
    for (int e = 0; e < 8; ++e) ss += (v[e] - mean) * (v[e] - mean);
#pragma unroll
    for (int o = 4; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    const float rstd = rsqrtf(ss * (1.f / 64) + a.eps);
#pragma unroll
    for (int e = 0; e < 8; ++e) v[e] = (v[e] - mean) * rstd * wv[e] + bv[e];
    if (!live) continue;
    if (a.mod_scale != nullptr) {
      float sc[8], sh[8];
      unpack8_bf16(*reinterpret_cast<const uint4*>(a.mod_scale + row * 64 + sub * 8), sc);
      if (a.mod_shift) {
        unpack8_bf16(*reinterpret_cast<const uint4*>(a.mod_shift + row * 64 + sub * 8), sh);
      } else {
#pragma unroll
        for (int e = 0; e < 8; ++e) sh[e] = 0.f;
      }
#pragma unroll
      for (int e = 0; e < 8; ++e) v[e] = sc[e] * v[e] + sh[e];
    }
    if (a.y != nullptr) {
      const int64_t yrow =
          a.perm_outer > 0 ? (row % a.perm_inner) * a.perm_outer + row / a.perm_inner : row;
      uint4 w;
      w.x = pack_bf16x2(v[0], v[1]);
      w.y = pack_bf16x2(v[2], v[3]);
      w.z = pack_bf16x2(v[4], v[5]);
      w.w = pack_bf16x2(v[6], v[7]);
      *reinterpret_cast<uint4*>(a.y + yrow * a.ldy + sub * 8) = w;
    }
  }
}

// Channel-major LayerNorm: x(ch, i, j) = in[ch*chan_stride + i*pitch + j].
// ln_heads_tc_kernel: LayerNorm of 128-wide rows plus a projection onto up to
// 16 heads (the attention pair bias, the single track's pair logits) on the
// tensor core.  Per tile of 128 rows: 8 warps normalise 16 rows each into a
// 128B-swizzled bf16 A tile (and into y when requested); one thread issues
// M=128 N=16 K=16 MMAs against the head weights (B: 16 x 128 bf16, rows past
// `heads` zero) into TMEM; warps 0-3 read heads 0-7 and warps 4-7 heads 8-15
// back, one row per thread, and store them head-major, coalesced along rows.
// The products are those of ln_rows_kernel's head path: bf16(normalised x) times
// bf16 weights, accumulated in f32.
template <typename InT, bool ROUTE = false>
__global__ void __launch_bounds__(256) ln_heads_tc_kernel(LnArgs a) {
  __shared__ __align__(1024) uint8_t sA[2 * 16384];  // k-halves of 64 channels
  __shared__ __align__(1024) uint8_t sB[2 * 2048];   // 16 heads x 64 channels per half
  __shared__ uint64_t bar;
  __shared__ uint32_t tmem_slot;
  __shared__ int abort_flag;
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0) {
    tmem_alloc(&tmem_slot, 32);
    tmem_relinquish();
  }
  // head weights into the swizzled B tile (K-major, one 128-byte row per head and half)
  for (int idx = threadIdx.x; idx < 16 * 128; idx += blockDim.x) {
    const int n = idx >> 7, ch = idx & 127;
    const int h = ch >> 6, k = ch & 63;
    const __nv_bfloat16 w = n < a.heads ? a.wh[n * 128 + ch] : __float2bfloat16_rn(0.f);
    *reinterpret_cast<__nv_bfloat16*>(sB + h * 2048 + n * 128 + (((k >> 3) ^ (n & 7)) << 4) +
                                      (k & 7) * 2) = w;
  }
  float wv[4], bv[4];
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    wv[e] = a.w ? a.w[lane * 4 + e] : 1.f;
    bv[e] = a.b ? a.b[lane * 4 + e] : 0.f;
  }
  fence_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_slot;
  constexpr uint32_t kIdesc = idesc_bf16(128, 16, false, false);
  // this lane's 8 bytes in a row of the A tile: channels 4*lane .. 4*lane+3
  const int half = lane >> 4;
  const int chunk = (lane & 15) >> 1;
  const int within = (lane & 1) * 8;
  const int64_t tiles = (a.rows + 127) / 128;
  uint32_t phase = 0;
  for (int64_t tile = blockIdx.x; tile < tiles; tile += gridDim.x) {
    const int64_t row0 = tile * 128;
    // ---- LayerNorm of 16 rows per warp, next row's load in flight
    float nxt[4];
    auto load = [&](int r, float (&v)[4]) {
      const int64_t row = row0 + warp * 16 + r;
      if (row < a.rows) {
        load_vec4<InT>(reinterpret_cast<const InT*>(a.x) + row * a.ldx + lane * 4, v);
      } else {
        v[0] = v[1] = v[2] = v[3] = 0.f;
      }
    };
    load(0, nxt);
#pragma unroll 1
    for (int r = 0; r < 16; ++r) {
      float v[4] = {nxt[0], nxt[1], nxt[2], nxt[3]};
      if (r + 1 < 16) load(r + 1, nxt);
      const int trow = warp * 16 + r;
      const int64_t row = row0 + trow;
      const float mean = warp_sum(v[0] + v[1] + v[2] + v[3]) * (1.f / 128);
      float ss = 0.f;
#pragma unroll
      for (int e = 0; e < 4; ++e) ss += (v[e] - mean) * (v[e] - mean);
      const float rstd = rsqrtf(warp_sum(ss) * (1.f / 128) + a.eps);
      uint2 pk = make_uint2(0u, 0u);
      if (row < a.rows) {
#pragma unroll
        for (int e = 0; e < 4; ++e) v[e] = (v[e] - mean) * rstd * wv[e] + bv[e];
        pk.x = pack_bf16x2(v[0], v[1]);
        pk.y = pack_bf16x2(v[2], v[3]);
        if (a.y != nullptr) {
          __nv_bfloat16* yrow = a.y + row * a.ldy;
          if constexpr (ROUTE) {
            const int64_t i = row / a.route_n;
            const int64_t j = row - i * a.route_n;
            const int s = static_cast<int>(j / a.route_rows);
            yrow = a.y_dst[s] + ((j - static_cast<int64_t>(s) * a.route_rows) * a.route_n +
                                 static_cast<int64_t>(a.route_rank) * a.route_rows + i) * a.ldy;
          }
          *reinterpret_cast<uint2*>(yrow + lane * 4) = pk;
        }
      }
      *reinterpret_cast<uint2*>(sA + half * 16384 + trow * 128 + ((chunk ^ (trow & 7)) << 4) +
                                within) = pk;
    }
    fence_async_smem();
    tc_fence_before();
    __syncthreads();
    // ---- head projection on the tensor core
    if (threadIdx.x == 0) {
      tc_fence_after();
      const uint32_t a_addr = smem_u32(sA), b_addr = smem_u32(sB);
#pragma unroll
      for (int h = 0; h < 2; ++h)
#pragma unroll
        for (int j = 0; j < 4; ++j)
          umma_bf16(tmem, sw128_desc(a_addr + h * 16384 + j * 32, 16, 1024),
                    sw128_desc(b_addr + h * 2048 + j * 32, 16, 1024), kIdesc, (h | j) ? 1u : 0u);
      umma_commit(&bar);
    }
    const bool ok = mbar_wait(&bar, phase, kErrWaitEpilogue, &abort_flag);
    phase ^= 1;
    tc_fence_after();
    // ---- heads back from TMEM: warps w and w+4 share lane quarter w % 4
    {
      const int quarter = warp & 3;
      const int hbase = (warp >> 2) * 8;
      float hv[8];
      uint32_t r8[8];
      __syncwarp();
      asm volatile(
          "tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
          : "=r"(r8[0]), "=r"(r8[1]), "=r"(r8[2]), "=r"(r8[3]), "=r"(r8[4]), "=r"(r8[5]),
            "=r"(r8[6]), "=r"(r8[7])
          : "r"(tmem + (static_cast<uint32_t>(quarter * 32) << 16) + hbase));
      asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
      for (int e = 0; e < 8; ++e) hv[e] = __uint_as_float(r8[e]);
      const int64_t row = row0 + quarter * 32 + lane;
      if (ok && row < a.rows) {
#pragma unroll
        for (int e = 0; e < 8; ++e)
          if (hbase + e < a.heads)
            a.head_out[(hbase + e) * a.head_ld + row] = __float2bfloat16_rn(hv[e] * a.head_scale);
      }
    }
    tc_fence_before();
    __syncthreads();  // TMEM and the A tile are reused by the next tile
  }
  if constexpr (ROUTE) __threadfence_system();  // publish the routed rows before the exchange barrier
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, 32);
  }
}

template <int C>
__global__ void __launch_bounds__(128) ln_channel_major_kernel(
    const __nv_bfloat16* in, int rows, int n, int pitch, int64_t chan_stride, const float* w,
    const float* b, float eps, __nv_bfloat16* y) {
  const int64_t total = static_cast<int64_t>(rows) * n;
  for (int64_t pos = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; pos < total;
       pos += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int i = static_cast<int>(pos / n);
    const int j = static_cast<int>(pos - static_cast<int64_t>(i) * n);
    const __nv_bfloat16* src = in + static_cast<int64_t>(i) * pitch + j;
    float v[C];
    float s = 0.f;
#pragma unroll
    for (int ch = 0; ch < C; ++ch) {
      v[ch] = __bfloat162float(src[ch * chan_stride]);
      s += v[ch];
    }
    const float mean = s * (1.f / C);
    float ss = 0.f;
#pragma unroll
    for (int ch = 0; ch < C; ++ch) {
      const float d = v[ch] - mean;
      ss += d * d;
    }
    const float rstd = rsqrtf(ss * (1.f / C) + eps);
    __nv_bfloat16* dst = y + pos * C;
#pragma unroll
    for (int ch = 0; ch < C; ch += 8) {
      float o[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const float wv = w ? w[ch + e] : 1.f;
        const float bv = b ? b[ch + e] : 0.f;
        o[e] = (v[ch + e] - mean) * rstd * wv + bv;
      }
      uint4 pk;
      pk.x = pack_bf16x2(o[0], o[1]);
      pk.y = pack_bf16x2(o[2], o[3]);
      pk.z = pack_bf16x2(o[4], o[5]);
      pk.w = pack_bf16x2(o[6], o[7]);
      *reinterpret_cast<uint4*>(dst + ch) = pk;
    }
  }
}

// LayerNorm statistics over the channels of a channel-major bf16 tensor with
// contiguous positions: x[ch * chan_stride + p], p < count (count even).  Writes
// stats[p] = (mean, 1 / sqrt(var + eps)).  Each thread takes two neighbouring
// positions, so a warp reads one 128-byte line per channel plane; the sums
// are shifted by the position's channel-0 value (a one-pass variance without
// the cancellation of E[x^2] - E[x]^2 at large means).
template <int C>
__global__ void __launch_bounds__(256) ln_stats_channel_major_kernel(
    const __nv_bfloat16* x, int64_t count, int64_t chan_stride, float eps, float2* stats) {
  const int64_t pairs = count / 2;
  for (int64_t t = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; t < pairs;
       t += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const uint32_t* src = reinterpret_cast<const uint32_t*>(x) + t;
    const int64_t stride_words = chan_stride / 2;
    const uint32_t w0 = src[0];
    const float k0 = __uint_as_float(w0 << 16), k1 = __uint_as_float(w0 & 0xFFFF0000u);
    float s0 = 0.f, s1 = 0.f, q0 = 0.f, q1 = 0.f;
#pragma unroll 16
    for (int ch = 1; ch < C; ++ch) {
      const uint32_t w = src[ch * stride_words];
      const float d0 = __uint_as_float(w << 16) - k0;
      const float d1 = __uint_as_float(w & 0xFFFF0000u) - k1;
      s0 += d0;
      s1 += d1;
      q0 = fmaf(d0, d0, q0);
      q1 = fmaf(d1, d1, q1);
    }
    const float m0 = s0 * (1.f / C), m1 = s1 * (1.f / C);
    const float v0 = fmaxf(q0 * (1.f / C) - m0 * m0, 0.f);
    const float v1 = fmaxf(q1 * (1.f / C) - m1 * m1, 0.f);
    reinterpret_cast<float4*>(stats)[t] =
        make_float4(k0 + m0, rsqrtf(v0 + eps), k1 + m1, rsqrtf(v1 + eps));
  }
}

// Row gather used to pack weights: dst[r][:] = src[map(r)][:] (bf16), zero rows
// where map(r) < 0.  `src_is_f32` selects the source element type.
__global__ void pack_rows_kernel(const void* src, int src_is_f32, const int* map, int rows,
                                 int k, __nv_bfloat16* dst) {
  const int64_t total = static_cast<int64_t>(rows) * k;
  for (int64_t idx = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; idx < total;
       idx += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int r = static_cast<int>(idx / k);
    const int c = static_cast<int>(idx - static_cast<int64_t>(r) * k);
    const int s = map[r];
    float v = 0.f;
    if (s >= 0) {
      v = src_is_f32 ? reinterpret_cast<const float*>(src)[static_cast<int64_t>(s) * k + c]
                     : __bfloat162float(
                           reinterpret_cast<const __nv_bfloat16*>(src)[static_cast<int64_t>(s) * k + c]);
    }
    dst[idx] = __float2bfloat16_rn(v);
  }
}

}  // namespace xfb
