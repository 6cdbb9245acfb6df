// Windowed cross-attention of the atom transformer and its pair logits.
//
// window_attention_kernel: one CTA per subset (a window of 32 query atoms and
//   the 128 key atoms around it), 4 heads of width 32 (c = 128).  The four
//   heads' queries are stacked into one M = 128 tile whose rows carry only
//   their own head's 32 channels (block-diagonal, K = 128), so one chain of
//   M=128 N=128 MMAs against the [128 keys x 128 channels] key tile gives every
//   head's 32 x 128 logits at once; row 32h+i of the accumulator is query i of
//   head h.  Each thread owns one row: it adds the pair logits and the
//   reference's mask term, takes the whole-row softmax (the 128 keys fit one
//   tile, no online rescaling), writes P to TMEM, and after P [V_0..V_3] (the
//   value tile as an MN-major B operand, N = 128) reads its head's 32 output
//   channels, normalises, applies sigmoid(gate) and stores bf16.  The O
//   accumulator reuses the logits' TMEM columns; P sits in the next 64.
//
// cross_pair_logits_kernel: LayerNorm over the 16 channels of every atom pair
//   and the projection onto blocks x heads pair logits, written in the layout
//   the attention kernel reads ([block][subset][head][query][key], bf16).
#pragma once

#include "attention.cuh"
#include "layer_norm.cuh"

namespace xfb {

constexpr int kWinQ = 32;    // queries per subset
constexpr int kWinK = 128;   // keys per subset
constexpr int kWinH = 4;     // heads
constexpr int kWinC = 128;   // channels (heads x 32)

struct WindowAttnArgs {
  const __nv_bfloat16* qg;    // [subsets*32][256]: q (projection + bias) | gate logits
  const __nv_bfloat16* kv;    // [subsets*128][256]: k | v
  const __nv_bfloat16* bias;  // [subsets][4][32][128] pair logits, or null
  const float* mask_q;        // [subsets*32] (0 = masked), or null
  const float* mask_k;        // [subsets*128], or null
  __nv_bfloat16* out;         // [subsets*32][128]
  float q_scale;
};

struct WinSmem {
  static constexpr int kA = 0;          // stacked queries: two K-halves of 128 x 128 B
  static constexpr int kK = 32768;      // keys: two channel halves of 128 x 128 B
  static constexpr int kV = 65536;      // values: same layout as the keys
  static constexpr int kBar = 98304;    // two mbarriers
  static constexpr int kTotal = kBar + 16;
  static constexpr int kLaunchBytes = kTotal + 1024;  // 1024-byte alignment slack
};

// Byte offset of 16-byte chunk `c` (0..7) of row `r` in a 128B-swizzled tile.
__device__ __forceinline__ uint32_t sw128_chunk(int r, int c) {
  return static_cast<uint32_t>(r * 128 + ((c ^ (r & 7)) << 4));
}

__device__ __forceinline__ uint4 scale_bf16x8(uint4 v, float s) {
  uint32_t* w = reinterpret_cast<uint32_t*>(&v);
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    const float lo = __uint_as_float(w[e] << 16) * s;
    const float hi = __uint_as_float(w[e] & 0xFFFF0000u) * s;
    w[e] = pack_bf16x2(lo, hi);
  }
  return v;
}

__global__ void __launch_bounds__(128) window_attention_kernel(const __grid_constant__ WindowAttnArgs a) {
  extern __shared__ uint8_t win_smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(win_smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + WinSmem::kBar);
  __shared__ uint32_t tmem_slot;
  __shared__ int abort_flag;
  __shared__ uint32_t key_masked[4];
  const int t = threadIdx.x;
  const int warp = t >> 5;  // head of this thread's row, and its TMEM lane quarter
  const int lane = t & 31;  // query of this thread's row
  const int64_t s = blockIdx.x;
  if (t == 0) {
    mbar_init(&bars[0], 1);
    mbar_init(&bars[1], 1);
    abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0) {
    tmem_alloc(&tmem_slot, 256);
    tmem_relinquish();
  }
  // ---- masks: bit j of key_masked set when key j is masked out
  {
    const bool km = a.mask_k != nullptr && a.mask_k[s * kWinK + t] == 0.f;
    const uint32_t bits = __ballot_sync(0xffffffffu, km);
    if (lane == 0) key_masked[warp] = bits;
  }
  const bool q_masked = a.mask_q != nullptr && a.mask_q[s * kWinQ + lane] == 0.f;
  // ---- stacked queries: row t holds head `warp`'s channels of query `lane`, scaled
  {
    const uint4* src = reinterpret_cast<const uint4*>(a.qg + (s * kWinQ + lane) * 256 + warp * 32);
    uint4 q[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) q[e] = scale_bf16x8(src[e], a.q_scale);
    const uint4 zero = make_uint4(0u, 0u, 0u, 0u);
    uint8_t* mine = smem + WinSmem::kA + (warp >> 1) * 16384;
    uint8_t* other = smem + WinSmem::kA + ((warp >> 1) ^ 1) * 16384;
    const int first = (warp & 1) * 4;
#pragma unroll
    for (int c = 0; c < 8; ++c) {
      const int e = c - first;
      *reinterpret_cast<uint4*>(mine + sw128_chunk(t, c)) = (e >= 0 && e < 4) ? q[e & 3] : zero;
      *reinterpret_cast<uint4*>(other + sw128_chunk(t, c)) = zero;
    }
  }
  // ---- keys and values: row t is key t
  {
    const uint4* src = reinterpret_cast<const uint4*>(a.kv + (s * kWinK + t) * 256);
    uint4 kx[16];
#pragma unroll
    for (int c = 0; c < 16; ++c) kx[c] = src[c];
#pragma unroll
    for (int c = 0; c < 16; ++c)
      *reinterpret_cast<uint4*>(smem + WinSmem::kK + (c >> 3) * 16384 + sw128_chunk(t, c & 7)) = kx[c];
#pragma unroll
    for (int c = 0; c < 16; ++c) kx[c] = src[16 + c];
#pragma unroll
    for (int c = 0; c < 16; ++c)
      *reinterpret_cast<uint4*>(smem + WinSmem::kV + (c >> 3) * 16384 + sw128_chunk(t, c & 7)) = kx[c];
  }
  fence_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_slot;
  constexpr uint32_t kIdescS = idesc_bf16(128, 128, false, false);
  constexpr uint32_t kIdescO = idesc_bf16(128, 128, false, true);
  constexpr uint32_t kPCol = 128;  // P: 64 columns after the logits / output
  if (t == 0) {
    const uint32_t a_addr = smem_u32(smem + WinSmem::kA);
    const uint32_t k_addr = smem_u32(smem + WinSmem::kK);
#pragma unroll
    for (int kk = 0; kk < 8; ++kk) {
      const uint32_t off = (kk >> 2) * 16384 + (kk & 3) * 32;
      umma_bf16(tmem, sw128_desc(a_addr + off, 16, 1024), sw128_desc(k_addr + off, 16, 1024),
                kIdescS, kk > 0 ? 1u : 0u);
    }
    umma_commit(&bars[0]);
  }
  bool ok = mbar_wait(&bars[0], 0, kErrWaitSoftmax, &abort_flag);
  tc_fence_after();
  const uint32_t trow = tmem + (static_cast<uint32_t>(warp * 32) << 16);
  float x[128];
#pragma unroll
  for (int cc = 0; cc < 4; ++cc) tmem_ld32_to(trow + 32 * cc, x + 32 * cc);
  tmem_wait_ld();
  // ---- logits: (q.k + 1e9 where query and key are both masked) + pair logits
  const uint4* brow =
      a.bias ? reinterpret_cast<const uint4*>(a.bias + ((s * kWinH + warp) * kWinQ + lane) * kWinK)
             : nullptr;
  float m = -INFINITY;
#pragma unroll
  for (int c = 0; c < 16; ++c) {
    uint4 bv = brow ? brow[c] : make_uint4(0u, 0u, 0u, 0u);
    const uint32_t* bw = reinterpret_cast<const uint32_t*>(&bv);
    const uint32_t km = q_masked ? (key_masked[c >> 2] >> ((c & 3) * 8)) & 0xFFu : 0u;
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const int j = c * 8 + e;
      float v = x[j];
      if ((km >> e) & 1u) v += 1e9f;
      v += (e & 1) ? __uint_as_float(bw[e >> 1] & 0xFFFF0000u) : __uint_as_float(bw[e >> 1] << 16);
      x[j] = v;
      m = max_nan(m, v);
    }
  }
  // ---- softmax numerators (bf16 P into TMEM) and the f32 row sum
  // (x - max) before the scaling: rows of the mask term sit near 1e9, where
  // x * log2(e) - max * log2(e) would keep the rounding error of both products
  constexpr float kLog2e = 1.4426950408889634f;
  float l = 0.f;
#pragma unroll
  for (int half = 0; half < 2; ++half) {
    uint32_t p[32];
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      const float p0 = ex2_approx((x[64 * half + 2 * j] - m) * kLog2e);
      const float p1 = ex2_approx((x[64 * half + 2 * j + 1] - m) * kLog2e);
      l += p0 + p1;
      p[j] = pack_bf16x2(p0, p1);
    }
    tmem_st32_u(trow + kPCol + 32 * half, p);
  }
  tmem_wait_st();
  tc_fence_before();
  __syncthreads();
  if (t == 0) {
    tc_fence_after();
    const uint32_t v_addr = smem_u32(smem + WinSmem::kV);
#pragma unroll
    for (int kk = 0; kk < 8; ++kk)
      umma_bf16_ts(tmem, tmem + kPCol + 8 * kk, sw128_desc(v_addr + kk * 2048, 16384, 1024),
                   kIdescO, kk > 0 ? 1u : 0u);
    umma_commit(&bars[1]);
  }
  ok = mbar_wait(&bars[1], 0, kErrWaitSoftmax, &abort_flag) && ok;
  tc_fence_after();
  float o[32];
  tmem_ld32_to(trow + 32 * warp, o);
  tmem_wait_ld();
  if (ok) {
    const float inv = 1.f / l;
    const uint4* gsrc = reinterpret_cast<const uint4*>(a.qg + (s * kWinQ + lane) * 256 + 128 + warp * 32);
    uint4* dst = reinterpret_cast<uint4*>(a.out + (s * kWinQ + lane) * kWinC + warp * 32);
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      uint4 g = gsrc[c];
      const uint32_t* gw = reinterpret_cast<const uint32_t*>(&g);
      uint4 r;
      uint32_t* rw = reinterpret_cast<uint32_t*>(&r);
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float g0 = sigmoidf_stable(__uint_as_float(gw[e] << 16));
        const float g1 = sigmoidf_stable(__uint_as_float(gw[e] & 0xFFFF0000u));
        rw[e] = pack_bf16x2(o[c * 8 + 2 * e] * inv * g0, o[c * 8 + 2 * e + 1] * inv * g1);
      }
      dst[c] = r;
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, 256);
  }
}

// One thread per atom pair: LayerNorm over its 16 channels (weight, optional
// bias), bf16 rounding of the normalised values (the projection's input), and
// outs = blocks * heads dot products with the bf16 projection rows, rounded to
// bf16 at out[((b * subsets + n) * heads + h) * pairs + r] for pair r of subset n.
template <typename InT>
__global__ void __launch_bounds__(256) cross_pair_logits_kernel(
    const InT* x, int64_t subsets, int pairs, int heads, int outs, const float* lw,
    const float* lb, float eps, const __nv_bfloat16* w, __nv_bfloat16* out) {
  __shared__ float sw[16][16];
  for (int i = threadIdx.x; i < 256; i += blockDim.x) {
    const int o = i >> 4;
    sw[o][i & 15] = o < outs ? __bfloat162float(w[i]) : 0.f;
  }
  __syncthreads();
  float gw[16], gb[16];
#pragma unroll
  for (int c = 0; c < 16; ++c) {
    gw[c] = lw ? lw[c] : 1.f;
    gb[c] = lb ? lb[c] : 0.f;
  }
  const int64_t total = subsets * pairs;
  for (int64_t pos = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; pos < total;
       pos += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    float v[16];
    const InT* src = x + pos * 16;
#pragma unroll
    for (int c = 0; c < 16; c += 4) {
      float q[4];
      load_vec4<InT>(src + c, q);
      v[c] = q[0];
      v[c + 1] = q[1];
      v[c + 2] = q[2];
      v[c + 3] = q[3];
    }
    float sum = 0.f;
#pragma unroll
    for (int c = 0; c < 16; ++c) sum += v[c];
    const float mean = sum * (1.f / 16);
    float ss = 0.f;
#pragma unroll
    for (int c = 0; c < 16; ++c) ss += (v[c] - mean) * (v[c] - mean);
    const float rstd = rsqrtf(ss * (1.f / 16) + eps);
#pragma unroll
    for (int c = 0; c < 16; ++c) v[c] = bf16r((v[c] - mean) * rstd * gw[c] + gb[c]);
    const int64_t n = pos / pairs;
    const int64_t r = pos - n * pairs;
    for (int o = 0; o < outs; ++o) {
      float acc = 0.f;
#pragma unroll
      for (int c = 0; c < 16; ++c) acc = fmaf(v[c], sw[o][c], acc);
      const int b = o / heads, h = o - b * heads;
      out[((static_cast<int64_t>(b) * subsets + n) * heads + h) * pairs + r] = __float2bfloat16_rn(acc);
    }
  }
}

}  // namespace xfb
