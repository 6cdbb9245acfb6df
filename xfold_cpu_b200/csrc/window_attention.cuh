// Windowed cross-attention of the atom transformer and its pair logits.
//
// window_attention_kernel: one CTA per subset (a window of 32 query atoms and
//   the 128 key atoms around it), 4 heads of width 32 (c = 128).  The four
//   heads' queries are stacked into one M = 128 tile whose rows carry only
//   their own head's 32 channels (block-diagonal, K = 128), so one chain of
//   M=128 N=128 MMAs against the [128 keys x 128 channels] key tile gives every
//   head's 32 x 128 logits at once; row 32h+i of the accumulator is query i of
//   head h.  The subset's keys and values (one contiguous [128 x 256] block of
//   the projection output) arrive by four TMA boxes whose 128B swizzle is the
//   operand layout.  Two threads share each row (warps w and w + 4 read the
//   same TMEM lane quarter), 64 keys each: their pair logits are loaded at the
//   start, in flight while the tiles land and the MMAs run; each adds the pair
//   logits and the reference's mask term to its 64 logits, the two exchange
//   their maxima through shared memory and take the whole-row softmax (the 128
//   keys fit one tile, no online rescaling), P goes to TMEM, and after
//   P [V_0..V_3] (the value tile as an MN-major B operand, N = 128) each reads
//   16 of its head's 32 output channels, normalises by the pair's summed
//   denominators, applies sigmoid(gate) and stores bf16.  The O accumulator
//   reuses the logits' TMEM columns; P sits in the next 64.
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
  CUtensorMap kv_map;         // kv as 2-D {256, subsets*128}, box {64, 128}, 128B swizzle
  const __nv_bfloat16* qg;    // [subsets*32][256]: q (projection + bias) | gate logits
  const __nv_bfloat16* bias;  // [subsets][4][32][128] pair logits, or null
  const float* mask_q;        // [subsets*32] (0 = masked), or null
  const float* mask_k;        // [subsets*128], or null
  __nv_bfloat16* out;         // [subsets*32][128]
  float q_scale;
};

struct WinSmem {
  static constexpr int kA = 0;          // stacked queries: two K-halves of 128 x 128 B
  static constexpr int kK = 32768;      // keys: two channel halves of 128 x 128 B (TMA)
  static constexpr int kV = 65536;      // values: same layout as the keys (TMA)
  static constexpr int kBar = 98304;    // three mbarriers
  static constexpr int kTotal = kBar + 24;
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

constexpr int kWinThreads = 256;  // two threads per logits row (64 keys each)

// Logits of 32 consecutive keys (chunk `cc` of this thread's 64) of its row:
// the accumulator plus the mask term plus the pair logits, in the reference's
// order.
__device__ __forceinline__ void window_logits32(float* x, const uint4 (&bias)[8], int cc,
                                                uint32_t km) {
#pragma unroll
  for (int e = 0; e < 32; ++e) {
    const uint32_t bw = reinterpret_cast<const uint32_t*>(&bias[cc * 4 + (e >> 3)])[(e & 7) >> 1];
    float v = x[e];
    if ((km >> e) & 1u) v += 1e9f;
    x[e] = v + ((e & 1) ? __uint_as_float(bw & 0xFFFF0000u) : __uint_as_float(bw << 16));
  }
}

__global__ void __launch_bounds__(kWinThreads, 2) window_attention_kernel(
    const __grid_constant__ WindowAttnArgs a) {
  extern __shared__ uint8_t win_smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(win_smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + WinSmem::kBar);  // kv, S, O
  __shared__ uint32_t tmem_slot;
  __shared__ int abort_flag;
  __shared__ uint32_t key_masked[4];
  __shared__ float row_max[kWinThreads];
  __shared__ float row_sum[kWinThreads];
  const int t = threadIdx.x;
  const int warp = t >> 5;
  const int head = warp & 3;  // head of this thread's row, and its TMEM lane quarter
  const int hf = warp >> 2;   // which 64 keys of the row (and 16 of the head's outputs)
  const int lane = t & 31;    // query of this thread's row
  const int row = head * 32 + lane;
  const int64_t s = blockIdx.x;
  if (t == 0) {
#pragma unroll
    for (int b = 0; b < 3; ++b) mbar_init(&bars[b], 1);
    abort_flag = 0;
    fence_mbar_init();
    // keys and values of this subset: rows s*128.. of kv, four 64-column boxes
    mbar_arrive_expect_tx(&bars[0], 4 * 16384);
#pragma unroll
    for (int b = 0; b < 4; ++b)
      tma_load_2d(smem + (b < 2 ? WinSmem::kK : WinSmem::kV) + (b & 1) * 16384, &a.kv_map,
                  &bars[0], b * 64, static_cast<int>(s * kWinK));
  }
  if (warp == 0) {
    tmem_alloc(&tmem_slot, 256);
    tmem_relinquish();
  }
  // ---- this thread's 64 pair logits, in flight during the MMAs
  uint4 bias[8];
  {
    const uint4* brow = reinterpret_cast<const uint4*>(
        a.bias + ((s * kWinH + head) * kWinQ + lane) * kWinK + hf * 64);
#pragma unroll
    for (int c = 0; c < 8; ++c) bias[c] = a.bias ? brow[c] : make_uint4(0u, 0u, 0u, 0u);
  }
  // ---- masks: bit j of key_masked set when key j is masked out
  if (t < kWinK) {
    const bool km = a.mask_k != nullptr && a.mask_k[s * kWinK + t] == 0.f;
    const uint32_t bits = __ballot_sync(0xffffffffu, km);
    if (lane == 0) key_masked[warp] = bits;
  }
  const bool q_masked = a.mask_q != nullptr && a.mask_q[s * kWinQ + lane] == 0.f;
  // ---- stacked queries: row `row` holds head `head`'s channels of query
  // `lane`, scaled; this thread writes K-half `hf` of the row
  {
    const uint4 zero = make_uint4(0u, 0u, 0u, 0u);
    uint8_t* dst = smem + WinSmem::kA + hf * 16384;
    if ((head >> 1) == hf) {
      const uint4* src = reinterpret_cast<const uint4*>(a.qg + (s * kWinQ + lane) * 256 + head * 32);
      uint4 q[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) q[e] = scale_bf16x8(src[e], a.q_scale);
      const int first = (head & 1) * 4;
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        const int e = c - first;
        *reinterpret_cast<uint4*>(dst + sw128_chunk(row, c)) = (e >= 0 && e < 4) ? q[e & 3] : zero;
      }
    } else {
#pragma unroll
      for (int c = 0; c < 8; ++c) *reinterpret_cast<uint4*>(dst + sw128_chunk(row, c)) = zero;
    }
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
    if (mbar_wait(&bars[0], 0, kErrWaitMma, &abort_flag)) {
      tc_fence_after();
      const uint32_t a_addr = smem_u32(smem + WinSmem::kA);
      const uint32_t k_addr = smem_u32(smem + WinSmem::kK);
#pragma unroll
      for (int kk = 0; kk < 8; ++kk) {
        const uint32_t off = (kk >> 2) * 16384 + (kk & 3) * 32;
        umma_bf16(tmem, sw128_desc(a_addr + off, 16, 1024), sw128_desc(k_addr + off, 16, 1024),
                  kIdescS, kk > 0 ? 1u : 0u);
      }
    }
    umma_commit(&bars[1]);
  }
  bool ok = mbar_wait(&bars[1], 0, kErrWaitSoftmax, &abort_flag);
  tc_fence_after();
  const uint32_t trow = tmem + (static_cast<uint32_t>(head * 32) << 16);
  // ---- logits of this thread's 64 keys: (q.k + 1e9 where query and key are
  // both masked) + pair logits; the row max shared with the partner thread
  float x[64];
  tmem_ld32_to(trow + 64 * hf, x);
  tmem_ld32_to(trow + 64 * hf + 32, x + 32);
  tmem_wait_ld();
#pragma unroll
  for (int u = 0; u < 2; ++u)
    window_logits32(x + 32 * u, bias, u, q_masked ? key_masked[2 * hf + u] : 0u);
  float m = -INFINITY;
#pragma unroll
  for (int e = 0; e < 64; ++e) m = max_nan(m, x[e]);
  row_max[t] = m;
  __syncthreads();
  m = max_nan(m, row_max[t ^ 128]);
  // ---- softmax numerators (bf16 P into TMEM) and this half's f32 sum.
  // (x - max) before the scaling: rows of the mask term sit near 1e9, where
  // x * log2(e) - max * log2(e) would keep the rounding error of both products.
  constexpr float kLog2e = 1.4426950408889634f;
  float l = 0.f;
  {
    uint32_t p[32];
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      const float p0 = ex2_approx((x[2 * j] - m) * kLog2e);
      const float p1 = ex2_approx((x[2 * j + 1] - m) * kLog2e);
      l += p0 + p1;
      p[j] = pack_bf16x2(p0, p1);
    }
    tmem_st32_u(trow + kPCol + 32 * hf, p);
  }
  row_sum[t] = l;
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
    umma_commit(&bars[2]);
  }
  // ---- output: this thread's 16 of its head's 32 channels
  const int ocol = head * 32 + hf * 16;
  uint4 gate[2];  // gate logits, loaded while the PV MMAs run
  {
    const uint4* gsrc = reinterpret_cast<const uint4*>(a.qg + (s * kWinQ + lane) * 256 + 128 + ocol);
    gate[0] = gsrc[0];
    gate[1] = gsrc[1];
  }
  const float inv = 1.f / (row_sum[t] + row_sum[t ^ 128]);
  ok = mbar_wait(&bars[2], 0, kErrWaitSoftmax, &abort_flag) && ok;
  tc_fence_after();
  float o[16];
  tmem_ld16(trow + ocol, o);
  if (ok) {
    uint4* dst = reinterpret_cast<uint4*>(a.out + (s * kWinQ + lane) * kWinC + ocol);
#pragma unroll
    for (int c = 0; c < 2; ++c) {
      const uint32_t* gw = reinterpret_cast<const uint32_t*>(&gate[c]);
      uint4 r;
      uint32_t* rw = reinterpret_cast<uint32_t*>(&r);
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float g0 = sigmoid_ex2(__uint_as_float(gw[e] << 16));
        const float g1 = sigmoid_ex2(__uint_as_float(gw[e] & 0xFFFF0000u));
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
