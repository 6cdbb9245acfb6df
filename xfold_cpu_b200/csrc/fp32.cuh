// float32 compute path: the same operators in IEEE fp32 on the CUDA cores.
//
// The bf16 tensor-core path matches the reference's bf16 route (autocast) to
// about 1e-2; the reference's float32 route (no autocast: torch matmul /
// softmax in fp32, xfold/fastnn/native.py:31-43) is matched to about 1e-6 here
// by doing every product and sum in fp32 with FFMA, in the reference's order of
// operations where rounding could differ visibly (q scaled before q.k^T, the
// bias added and the mask applied before the softmax, gates multiplied after).
// These kernels serve that precision contract, not speed: tiled SIMT GEMM
// (64 x 64 tiles, 4 x 4 outputs per thread), one warp per row for LayerNorm, a
// one-warp-per-query online-softmax attention.  Every operand is addressed
// through strides, so transposes, head splits and the triangle multiplication's
// channel interleave are views, never copies.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace xfb {

__device__ __forceinline__ float f32_sigmoid(float x) { return 1.f / (1.f + expf(-x)); }

// C[b](i, j) (=|+=) epi( sum_k A[b](i, k) B[b](j, k) )
//   epi(v) = ((act(v + bias[j])) * row_scale[b](i)) * mul[b](i, j)
// act: 0 none, 1 sigmoid.  Null pointers skip their step.
struct F32Gemm {
  const float* A;
  int64_t a_sb, a_si, a_sk;
  const float* B;
  int64_t b_sb, b_sj, b_sk;
  float* C;
  int64_t c_sb, c_si, c_sj;
  int M, N, K, batch;
  const float* bias;
  int act;
  const float* row_scale;
  int64_t rs_sb, rs_si;
  const float* mul;
  int64_t m_sb, m_si, m_sj;
  int accumulate;
};

constexpr int kF32Tile = 64;
constexpr int kF32BK = 16;

__global__ void __launch_bounds__(256) f32_gemm_kernel(const F32Gemm g) {
  __shared__ float sA[kF32BK][kF32Tile + 4];
  __shared__ float sB[kF32BK][kF32Tile + 4];
  const int b = blockIdx.z;
  const int i0 = blockIdx.y * kF32Tile;
  const int j0 = blockIdx.x * kF32Tile;
  const int tx = threadIdx.x & 15;  // 4 columns each
  const int ty = threadIdx.x >> 4;  // 4 rows each
  const float* A = g.A + b * g.a_sb;
  const float* B = g.B + b * g.b_sb;
  float acc[4][4] = {};
  for (int k0 = 0; k0 < g.K; k0 += kF32BK) {
    // 64 x 16 elements of each operand, 4 per thread
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int idx = threadIdx.x + e * 256;
      const int kk = idx & 15, r = idx >> 4;
      const int k = k0 + kk;
      const int i = i0 + r, j = j0 + r;
      sA[kk][r] = (i < g.M && k < g.K) ? A[i * g.a_si + k * g.a_sk] : 0.f;
      sB[kk][r] = (j < g.N && k < g.K) ? B[j * g.b_sj + k * g.b_sk] : 0.f;
    }
    __syncthreads();
#pragma unroll
    for (int kk = 0; kk < kF32BK; ++kk) {
      float a[4], bb[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        a[e] = sA[kk][ty * 4 + e];
        bb[e] = sB[kk][tx * 4 + e];
      }
#pragma unroll
      for (int r = 0; r < 4; ++r)
#pragma unroll
        for (int c = 0; c < 4; ++c) acc[r][c] = fmaf(a[r], bb[c], acc[r][c]);
    }
    __syncthreads();
  }
#pragma unroll
  for (int r = 0; r < 4; ++r) {
    const int i = i0 + ty * 4 + r;
    if (i >= g.M) continue;
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      const int j = j0 + tx * 4 + c;
      if (j >= g.N) continue;
      float v = acc[r][c];
      if (g.bias != nullptr) v += g.bias[j];
      if (g.act == 1) v = f32_sigmoid(v);
      if (g.row_scale != nullptr) v *= g.row_scale[b * g.rs_sb + i * g.rs_si];
      if (g.mul != nullptr) v *= g.mul[b * g.m_sb + i * g.m_si + j * g.m_sj];
      float* dst = g.C + b * g.c_sb + i * g.c_si + j * g.c_sj;
      *dst = g.accumulate ? *dst + v : v;
    }
  }
}

// LayerNorm over the last dimension (C <= 1024), one warp per row, two-pass
// mean / variance in fp32; y[r] = (x[r] - mean) * rstd * w + b (w, b optional).
__global__ void __launch_bounds__(256) f32_layer_norm_kernel(const float* x, int64_t rows, int C,
                                                             int64_t ldx, const float* w,
                                                             const float* bias, float eps,
                                                             float* y, int64_t ldy) {
  const int lane = threadIdx.x & 31;
  const int64_t warps = static_cast<int64_t>(gridDim.x) * (blockDim.x >> 5);
  for (int64_t r = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
       r < rows; r += warps) {
    const float* xr = x + r * ldx;
    float v[32];
    float s = 0.f;
#pragma unroll
    for (int t = 0; t < 32; ++t) {
      const int c = lane + 32 * t;
      v[t] = c < C ? xr[c] : 0.f;
      s += v[t];
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    const float mean = s / C;
    float ss = 0.f;
#pragma unroll
    for (int t = 0; t < 32; ++t) {
      const int c = lane + 32 * t;
      const float dlt = c < C ? v[t] - mean : 0.f;
      ss = fmaf(dlt, dlt, ss);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    const float rstd = rsqrtf(ss / C + eps);
    float* yr = y + r * ldy;
#pragma unroll
    for (int t = 0; t < 32; ++t) {
      const int c = lane + 32 * t;
      if (c < C) {
        float o = (v[t] - mean) * rstd;
        if (w != nullptr) o *= w[c];
        if (bias != nullptr) o += bias[c];
        yr[c] = o;
      }
    }
  }
}

// out[b][h][i] = gate * sum_k softmax_k(q[b][h][i] . k[b][h][k] * scale + bias, mask) v[b][h][k]
// (xfold/fastnn/attention.py:45-66 in fp32): q scaled first, the bias added,
// masked keys (mask value 0) set to -1e9, softmax in fp32 (online, exact up to
// rounding), then the optional gate (already squashed) multiplied in.
// Head dims d, dv <= 64; rows of q / k / v / out / gate contiguous in d.
struct F32Attn {
  const float* q;
  int64_t q_sb, q_sh, q_si;
  const float* k;
  int64_t k_sb, k_sh, k_si;
  const float* v;
  int64_t v_sb, v_sh, v_si;
  const float* bias;  // bias[b*sb + h*sh + i*si + key] or null
  int64_t bias_sb, bias_sh, bias_si;
  const float* mask;  // mask[b*sb + key] or null (0 = masked)
  int64_t mask_sb;
  float* out;
  int64_t o_sb, o_sh, o_si;
  const float* gate;  // same strides as out, or null
  int64_t g_sb, g_sh, g_si;
  int B, H, Q, K, d, dv;
  float scale;
};

constexpr int kF32AttnWarps = 8;   // queries per CTA
constexpr int kF32AttnKeys = 32;   // keys per tile (one per lane)

__global__ void __launch_bounds__(256) f32_attention_kernel(const F32Attn p) {
  __shared__ float sK[kF32AttnKeys][65];
  __shared__ float sV[kF32AttnKeys][64];
  __shared__ float sQ[kF32AttnWarps][64];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int bh = blockIdx.y;
  const int b = bh / p.H, h = bh - (bh / p.H) * p.H;
  const int i = blockIdx.x * kF32AttnWarps + warp;
  const bool active = i < p.Q;
  const float* qrow = p.q + b * p.q_sb + h * p.q_sh + static_cast<int64_t>(i) * p.q_si;
  for (int dd = lane; dd < 64; dd += 32) sQ[warp][dd] = (active && dd < p.d) ? qrow[dd] * p.scale : 0.f;
  const float* kb = p.k + b * p.k_sb + h * p.k_sh;
  const float* vb = p.v + b * p.v_sb + h * p.v_sh;
  const float* brow = (p.bias && active)
                         ? p.bias + b * p.bias_sb + h * p.bias_sh + static_cast<int64_t>(i) * p.bias_si
                         : nullptr;
  const float* mrow = p.mask ? p.mask + b * p.mask_sb : nullptr;
  float m = -INFINITY, l = 0.f;
  float o0 = 0.f, o1 = 0.f;  // output dims lane and lane + 32
  for (int k0 = 0; k0 < p.K; k0 += kF32AttnKeys) {
    __syncthreads();  // the previous tile is consumed (and sQ written)
    for (int idx = threadIdx.x; idx < kF32AttnKeys * 64; idx += blockDim.x) {
      const int kk = idx >> 6, dd = idx & 63;
      const int key = k0 + kk;
      const bool ok = key < p.K;
      sK[kk][dd] = (ok && dd < p.d) ? kb[static_cast<int64_t>(key) * p.k_si + dd] : 0.f;
      sV[kk][dd] = (ok && dd < p.dv) ? vb[static_cast<int64_t>(key) * p.v_si + dd] : 0.f;
    }
    __syncthreads();
    const int key = k0 + lane;
    float s = -INFINITY;  // keys past the end take no part
    if (key < p.K) {
      float dot = 0.f;
      for (int dd = 0; dd < p.d; ++dd) dot = fmaf(sQ[warp][dd], sK[lane][dd], dot);
      s = dot;
      if (brow != nullptr) s += brow[key];
      if (mrow != nullptr && mrow[key] == 0.f) s = -1e9f;
    }
    float tmax = s;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) tmax = fmaxf(tmax, __shfl_xor_sync(0xffffffffu, tmax, o));
    const float m_new = fmaxf(m, tmax);
    const float alpha = m == -INFINITY ? 0.f : expf(m - m_new);
    const float pk = s == -INFINITY ? 0.f : expf(s - m_new);
    float psum = pk;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) psum += __shfl_xor_sync(0xffffffffu, psum, o);
    l = l * alpha + psum;
    o0 *= alpha;
    o1 *= alpha;
#pragma unroll 8
    for (int j = 0; j < kF32AttnKeys; ++j) {
      const float pj = __shfl_sync(0xffffffffu, pk, j);
      o0 = fmaf(pj, sV[j][lane], o0);
      o1 = fmaf(pj, sV[j][lane + 32], o1);
    }
    m = m_new;
  }
  if (!active) return;
  float* orow = p.out + b * p.o_sb + h * p.o_sh + static_cast<int64_t>(i) * p.o_si;
  const float* grow =
      p.gate ? p.gate + b * p.g_sb + h * p.g_sh + static_cast<int64_t>(i) * p.g_si : nullptr;
  const float inv = l > 0.f ? 1.f / l : 0.f;
  if (lane < p.dv) orow[lane] = grow ? (o0 * inv) * grow[lane] : o0 * inv;
  if (lane + 32 < p.dv) orow[lane + 32] = grow ? (o1 * inv) * grow[lane + 32] : o1 * inv;
}

// y = silu(h[:, :f]) * h[:, f:]  (gated_linear_unit_torch, fastnn/gated_linear_unit.py:103-107)
__global__ void f32_silu_mul_kernel(const float* h, int64_t rows, int f, float* y) {
  const int64_t total = rows * f;
  for (int64_t t = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; t < total;
       t += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t r = t / f;
    const int c = static_cast<int>(t - r * f);
    const float a = h[r * 2 * f + c];
    y[t] = (a / (1.f + expf(-a))) * h[r * 2 * f + f + c];
  }
}

// y = y * scale + shift, elementwise over n values (the conditioned LayerNorm's
// modulation, diffusion_transformer.py:57-62)
__global__ void f32_scale_shift_kernel(float* y, const float* scale, const float* shift,
                                       int64_t n) {
  for (int64_t t = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; t < n;
       t += static_cast<int64_t>(gridDim.x) * blockDim.x)
    y[t] = y[t] * scale[t] + shift[t];
}

}  // namespace xfb
