// MSA-stack operators of the Evoformer (MSAAttention, OuterProductMean).
//
// MSAAttention (xfold/nn/attention.py:108-144) attends over tokens with one
// [heads, N, N] weight matrix shared by every MSA row: the softmax of the pair
// logits plus a key mask.  The weighted average of every row's values is then
// one GEMM per head, weights[h] [N(q) x N(k)] times the head's values as a
// [N(k) x S*8] matrix.  For that the projection writes v and the gate
// head-major with rows ordered (token, sequence): vt[h][k][b][c] and
// gt[h][q][b][c]; the weighted average's output ot[h][q][b][c] then has the
// gate's layout, and a head merge gives the [S][N][64] rows the output
// projection reads.
#pragma once

#include "attention.cuh"
#include "gemm.cuh"

namespace xfb {

// v | gate projection epilogue (BN = 128): columns 0..63 are v (8 heads x 8),
// 64..127 the gate logits.  Row m of the tile is (token, sequence) row m of the
// normalised MSA.  Writes bf16 v to vt[h][m][8] and bf16 sigmoid(bf16 gate) to
// gt[h][m][8]; a warp's 32 consecutive rows store 512 contiguous bytes per head.
struct EpiMsaVG {
  static constexpr int kStagingBytes = 0;
  static constexpr int kStagingBufs = 1;
  static constexpr int kAuxBytes = 0;
  __nv_bfloat16* vt;
  __nv_bfloat16* gt;
  int64_t M;

  __device__ void load_aux(void*, uint64_t*, int, int, int) const {}
  __device__ void store(const EpiCtx&) const {}

  __device__ void compute(const EpiCtx& c) const {
    const int64_t m = static_cast<int64_t>(c.m0) + c.row;
    __nv_bfloat16* base = c.half ? gt : vt;
#pragma unroll 1
    for (int c0 = 0; c0 < 64; c0 += 16) {
      float v[16];
      tmem_ld16(c.tmem + c.half * 64 + c0, v);
      if (m >= M) continue;
      if (c.half) {
#pragma unroll
        for (int i = 0; i < 16; ++i) v[i] = sigmoid_ex2(bf16r(v[i]));
      }
#pragma unroll
      for (int q = 0; q < 2; ++q) {
        uint4 w;
        w.x = pack_bf16x2(v[8 * q + 0], v[8 * q + 1]);
        w.y = pack_bf16x2(v[8 * q + 2], v[8 * q + 3]);
        w.z = pack_bf16x2(v[8 * q + 4], v[8 * q + 5]);
        w.w = pack_bf16x2(v[8 * q + 6], v[8 * q + 7]);
        *reinterpret_cast<uint4*>(base + ((c0 / 8 + q) * M + m) * 8) = w;
      }
    }
  }
};

// kmask[k] = max over sequences s of mask[s][k] (the reference's
// torch.max(msa_mask, dim=0)).  A block of 1024 threads takes 32 tokens: lane
// = token (a warp reads 128 contiguous bytes of a row), warp = one of 32 row
// groups, then a shared-memory reduction over the groups.
__global__ void __launch_bounds__(1024) msa_key_mask_kernel(const float* mask, int64_t s,
                                                            int64_t n, float* kmask) {
  __shared__ float part[32][33];
  const int lane = threadIdx.x & 31, grp = threadIdx.x >> 5;
  const int64_t k = static_cast<int64_t>(blockIdx.x) * 32 + lane;
  float m = -INFINITY;
  if (k < n) {
    for (int64_t r = grp; r < s; r += 32) m = fmaxf(m, mask[r * n + k]);
  }
  part[grp][lane] = m;
  __syncthreads();
  if (grp == 0) {
#pragma unroll 8
    for (int g = 1; g < 32; ++g) m = fmaxf(m, part[g][lane]);
    if (k < n) kmask[k] = s > 0 ? m : 0.f;
  }
}

// weights[r][k] = bf16(softmax_k(bf16(logits[r][k] + 1e9 (kmask[k] - 1)))), one
// warp per row of n keys (n a multiple of 8), three passes over the row (max,
// sum, write; the row stays in L1).  The bf16 rounding of the masked logit is
// the reference's in-place add on its bf16 logits (attention.py:133).
__global__ void __launch_bounds__(256) msa_softmax_kernel(const __nv_bfloat16* logits,
                                                          const float* kmask, int64_t rows,
                                                          int64_t n, __nv_bfloat16* weights) {
  const int lane = threadIdx.x & 31;
  const int64_t warps = static_cast<int64_t>(gridDim.x) * (blockDim.x >> 5);
  auto logit8 = [&](const __nv_bfloat16* row, int64_t k0, float (&x)[8]) {
    const uint4 w = *reinterpret_cast<const uint4*>(row + k0);
    unpack8_bf16(w, x);
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const float km = kmask ? kmask[k0 + e] : 1.f;
      x[e] = bf16r(x[e] + 1e9f * (km - 1.f));
    }
  };
  for (int64_t r = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
       r < rows; r += warps) {
    const __nv_bfloat16* row = logits + r * n;
    float m = -INFINITY;
    for (int64_t k0 = lane * 8; k0 < n; k0 += 256) {
      float x[8];
      logit8(row, k0, x);
#pragma unroll
      for (int e = 0; e < 8; ++e) m = max_nan(m, x[e]);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = max_nan(m, __shfl_xor_sync(0xffffffffu, m, o));
    constexpr float kLog2e = 1.4426950408889634f;
    float l = 0.f;
    for (int64_t k0 = lane * 8; k0 < n; k0 += 256) {
      float x[8];
      logit8(row, k0, x);
#pragma unroll
      for (int e = 0; e < 8; ++e) l += ex2_approx((x[e] - m) * kLog2e);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) l += __shfl_xor_sync(0xffffffffu, l, o);
    const float inv = 1.f / l;
    __nv_bfloat16* out = weights + r * n;
    for (int64_t k0 = lane * 8; k0 < n; k0 += 256) {
      float x[8];
      logit8(row, k0, x);
      uint4 w;
      w.x = pack_bf16x2(ex2_approx((x[0] - m) * kLog2e) * inv, ex2_approx((x[1] - m) * kLog2e) * inv);
      w.y = pack_bf16x2(ex2_approx((x[2] - m) * kLog2e) * inv, ex2_approx((x[3] - m) * kLog2e) * inv);
      w.z = pack_bf16x2(ex2_approx((x[4] - m) * kLog2e) * inv, ex2_approx((x[5] - m) * kLog2e) * inv);
      w.w = pack_bf16x2(ex2_approx((x[6] - m) * kLog2e) * inv, ex2_approx((x[7] - m) * kLog2e) * inv);
      *reinterpret_cast<uint4*>(out + k0) = w;
    }
  }
}

// Head merge: o[b][q][h*8 + c] = ot[h][q][b][c] for 8 heads of 8 channels.  One
// thread per (q, b) with b fastest, so the reads (16 bytes per head) are
// coalesced along b and each thread writes its 128-byte output row.
__global__ void msa_merge_heads_kernel(const __nv_bfloat16* ot, int64_t s, int64_t n,
                                       __nv_bfloat16* o) {
  const int64_t total = s * n;
  for (int64_t idx = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; idx < total;
       idx += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t q = idx / s;
    const int64_t b = idx - q * s;
    uint4 w[8];
#pragma unroll
    for (int h = 0; h < 8; ++h) w[h] = reinterpret_cast<const uint4*>(ot)[h * total + idx];
    uint4* dst = reinterpret_cast<uint4*>(o + (b * n + q) * 64);
#pragma unroll
    for (int h = 0; h < 8; ++h) dst[h] = w[h];
  }
}

// ---------------------------------------------------------------- OuterProductMean
//
// OuterProductMean (xfold/nn/primitives.py:62-75): out[i][j][f] =
// (sum_{c,e} (sum_a left[a][i][c] right[a][j][e]) W[c][e][f] + b[f]) /
// (1e-3 + sum_a mask[a][i] mask[a][j]).  The left / right projections are
// written [S][N*32] (masked), the MN-major operands of the first GEMM over the
// sequences; for a chunk of rows i its output goes straight into the
// [(i, j)][(c, e)] layout the second GEMM (against W as [f][(c, e)]) reads, so
// the N*N*1024 outer products exist only one L2-sized chunk at a time.

// left | right projection epilogue (BN = 128, 64 used columns): row m = (a, n)
// of the normalised MSA; columns 0..31 left, 32..63 right, each times
// mask[m] (the reference's mask * projection), bf16 into [m][32].
struct EpiOpmLR {
  static constexpr int kStagingBytes = 0;
  static constexpr int kStagingBufs = 1;
  static constexpr int kAuxBytes = 0;
  __nv_bfloat16* left;
  __nv_bfloat16* right;
  const float* mask;  // [M] or null
  int64_t M;

  __device__ void load_aux(void*, uint64_t*, int, int, int) const {}
  __device__ void store(const EpiCtx&) const {}

  __device__ void compute(const EpiCtx& c) const {
    if (c.half) return;  // columns 64..127 are past the 64 projections
    const int64_t m = static_cast<int64_t>(c.m0) + c.row;
    const float mv = (m < M && mask) ? mask[m] : 1.f;
#pragma unroll 1
    for (int c0 = 0; c0 < 64; c0 += 16) {
      float v[16];
      tmem_ld16(c.tmem + c0, v);
      if (m >= M) continue;
      __nv_bfloat16* dst = (c0 < 32 ? left : right) + m * 32 + (c0 & 31);
#pragma unroll
      for (int q = 0; q < 2; ++q) {
        uint4 w;
        w.x = pack_bf16x2(bf16r(v[8 * q + 0]) * mv, bf16r(v[8 * q + 1]) * mv);
        w.y = pack_bf16x2(bf16r(v[8 * q + 2]) * mv, bf16r(v[8 * q + 3]) * mv);
        w.z = pack_bf16x2(bf16r(v[8 * q + 4]) * mv, bf16r(v[8 * q + 5]) * mv);
        w.w = pack_bf16x2(bf16r(v[8 * q + 6]) * mv, bf16r(v[8 * q + 7]) * mv);
        reinterpret_cast<uint4*>(dst)[q] = w;
      }
    }
  }
};

// First GEMM's epilogue (BN = 256): tile rows (i, c) of the chunk, columns
// (j, e); element ((i, c), (j, e)) goes to outer[((i * N + j) * 32 + c) * 32 + e]
// (bf16), i.e. row (i, j) and column (c, e) of the second GEMM's A operand.
struct EpiOpmOuter {
  static constexpr int kStagingBytes = 0;
  static constexpr int kStagingBufs = 1;
  static constexpr int kAuxBytes = 0;
  __nv_bfloat16* outer;
  int M;   // chunk rows * 32
  int N;   // tokens (columns / 32)

  __device__ void load_aux(void*, uint64_t*, int, int, int) const {}
  __device__ void store(const EpiCtx&) const {}

  __device__ void compute(const EpiCtx& c) const {
    const int m = c.m0 + c.row;
    const int i = m >> 5, ci = m & 31;
#pragma unroll 1
    for (int c0 = 0; c0 < 128; c0 += 16) {
      float v[16];
      tmem_ld16(c.tmem + c.half * 128 + c0, v);
      const int col = c.n0 + c.half * 128 + c0;  // (j, e0), e0 in {0, 16}
      if (m >= M || col >= N * 32) continue;
      const int j = col >> 5, e0 = col & 31;
      __nv_bfloat16* dst = outer + ((static_cast<int64_t>(i) * N + j) * 32 + ci) * 32 + e0;
      store16_bf16(dst, v);
    }
  }
};

// Second GEMM's epilogue (BN = 128, f32 out): (bf16(acc) + b[f]) /
// (1e-3 + norm[row]) staged like EpiOut and stored or reduce-added by TMA into
// the f32 pair rows of the chunk.
struct EpiOpmOut : EpiOut<128, true> {
  const float* norm;  // [rows of the chunk], the mask overlap counts
  float eps;
  int M;              // rows of the chunk (the TMA store drops rows past it)

  __device__ void compute(const EpiCtx& c) const {
    const int m = c.m0 + c.row;
    const float inv = m < M ? 1.f / (eps + norm[m]) : 0.f;
#pragma unroll 1
    for (int c0 = 0; c0 < 64; c0 += 16) {
      const int col = c.half * 64 + c0;
      float v[16];
      tmem_ld16(c.tmem + col, v);
#pragma unroll
      for (int i = 0; i < 16; ++i) v[i] = (bf16r(v[i]) + this->bias[c.n0 + col + i]) * inv;
      this->write(c, col, v);
    }
  }
};

// output_w [c][e][f] (f32 or bf16) -> packed [f][c*32 + e] bf16: the second
// GEMM's K-major B operand.
__global__ void pack_opm_weight_kernel(const void* w, int w_f32, int64_t f_out,
                                       __nv_bfloat16* packed) {
  const int64_t total = f_out * 1024;
  for (int64_t idx = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; idx < total;
       idx += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t f = idx / 1024, ce = idx - f * 1024;
    const int64_t src = ce * f_out + f;
    packed[idx] = w_f32 ? __float2bfloat16_rn(static_cast<const float*>(w)[src])
                        : static_cast<const __nv_bfloat16*>(w)[src];
  }
}

// f32 -> bf16 copy of the 0/1 mask (exact), the operand of the overlap-count GEMM.
__global__ void f32_to_bf16_kernel(const float* x, int64_t n, __nv_bfloat16* y) {
  for (int64_t k = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; k < n;
       k += static_cast<int64_t>(gridDim.x) * blockDim.x)
    y[k] = __float2bfloat16_rn(x[k]);
}

}  // namespace xfb
