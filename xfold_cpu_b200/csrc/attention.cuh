// Flash attention with pair bias, key mask and fused sigmoid output gate on
// tcgen05 (sm_100a).
//
// Persistent CTAs (two per SM for head dim <= 32) walk work items (batch row b,
// head h, 128-query tile).  Per 64-key tile t of an item:
//   S_t  = bias_t + Q K_t^T tcgen05.mma from TMA-loaded swizzled SMEM into TMEM
//                           (double-buffered S); the bf16 bias tile enters the
//                           accumulator exactly through MMAs against a 16 x 16
//                           identity, so the softmax never touches it
//   P_t  = 2^(S_t - m_ref)  softmax warps, one query row per thread; P goes
//                           back to TMEM as bf16 (tcgen05.st)
//   O   += P_t V_t          tcgen05.mma with A = P from TMEM, V read MN-major
//   l   += P_t 1            a second MMA against a tile of ones: the row sums of
//                           the bf16 probabilities, next to O in TMEM
// With PRE, q carries d^-0.5 * log2(e) and the bias log2(e) from their
// producers, so scores are in log2 units; otherwise the exponent's FMA scales
// them by log2(e).  The running reference max m_ref only moves when a tile's
// max exceeds it by more than 8 (a factor 256), so O and l in TMEM are rescaled
// (tcgen05.ld / st) rarely.  A fixed share of the exponentials runs as a
// polynomial on the FMA pipe instead of the MUFU unit (exp2_poly2).
//
// Mask semantics follow the reference: a masked key gets the logit -1e9 (so a
// fully masked row is a uniform average), keys past the sequence end get
// probability exactly 0, and a NaN logit makes the row NaN.
#pragma once

#include "common.cuh"

namespace xfb {

// warpgroup 0: softmax warps 0-3; warpgroup 1: TMA producer (4), S-MMA issuer
// (5, owns TMEM), PV-MMA issuer (6), idle (7).  With two CTAs per SM the
// kernel launches at 128 registers per thread and moves registers from
// warpgroup 1 (down to 64) to the softmax (up to 192): 128*64 + 128*192 is
// exactly the 256*128 the CTA was launched with.
constexpr int kAttnThreads = 256;
constexpr int kAttnRegsLaunch = 128, kAttnRegsSoftmax = 192, kAttnRegsOther = 64;
static_assert(kAttnRegsSoftmax + kAttnRegsOther == 2 * kAttnRegsLaunch, "register split");
constexpr int kAttnKvStages = 3;    // K / V ring, freed by the PV MMA
constexpr int kAttnBiasStages = 3;  // bias ring, freed by the S MMA
constexpr int kAttnBK = 64;  // keys per tile
constexpr float kLog2e = 1.4426950408889634f;
// Of every 8 pairs of probabilities in a row tile, this many are computed by
// exp2_poly2 (FMA pipe) and the rest by ex2.approx (MUFU).
#ifndef XFB_FLASH_POLY_PAIRS
#define XFB_FLASH_POLY_PAIRS 0
#endif
constexpr int kAttnPolyPairs = XFB_FLASH_POLY_PAIRS;
// 1: the TMA bias tile enters S through identity MMAs; 0: the softmax warps add
// it from shared memory.
#ifndef XFB_FLASH_BIAS_MMA
#define XFB_FLASH_BIAS_MMA 1
#endif
constexpr bool kAttnBiasMma = XFB_FLASH_BIAS_MMA != 0;

// Bias source: streamed bf16 tiles through TMA, or per-thread global loads.
enum AttnBiasMode : int { kBiasTma = 0, kBiasGlobalBf16 = 1, kBiasGlobalF32 = 2 };

struct AttnArgs {
  int B, H, nq, nk, d;        // d: real head dim (<= DP)
  int q_tiles;                // ceil(nq / 128)
  const uint32_t* mask_bits;  // [B or 1][ceil(nk/32)] keep bits (bit k%32 of word k/32), or null
  int64_t mask_sb;            // words between batch rows (0 = shared)
  const void* bias;           // bias[b*sb + h*sh + q*sq + key], or null
  int64_t bias_sb, bias_sh, bias_sq;
  int bias_batched;           // TMA bias map: z = b*H + h when set, else z = h
  __nv_bfloat16* out;         // out[b*sb + h*sh + q*sq + dd]
  int64_t out_sb, out_sh, out_sq;
  const __nv_bfloat16* gate;  // optional gate, same indexing as out (already squashed)
  int64_t gate_sb, gate_sh, gate_sq;
};

template <int DP>
struct AttnSmem {
  static constexpr int kQBytes = 128 * DP * 2;
  static constexpr int kKVBytes = kAttnBK * DP * 2;
  static constexpr int kBiasBytes = 128 * kAttnBK * 2;  // one 64-key swizzle atom per row
  static constexpr int kQOff = 0;
  static constexpr int kKOff = kQOff + 2 * kQBytes;
  static constexpr int kVOff = kKOff + kAttnKvStages * kKVBytes;
  static constexpr int kBiasOff = kVOff + kAttnKvStages * kKVBytes;
  static constexpr int kOnesOff = kBiasOff + kAttnBiasStages * kBiasBytes;
  // ones as one extra N chunk of the V operand (one swizzle atom wide, all keys):
  // the PV MMA then also writes the row sums next to O
  static constexpr int kOnesBytes = kAttnBK * (DP == 32 ? 64 : 128);
  static constexpr int kIdentOff = kOnesOff + kOnesBytes;
  static constexpr int kIdentBytes = 16 * 128;  // 16 x 16 identity in 128-byte swizzled rows
  static constexpr int kBarOff = kIdentOff + kIdentBytes;
  // q_full[2], q_empty[2], kv_full[S], kv_empty[S], b_full[SB], b_empty[SB],
  // s_full[2], s_free[2],
  // p_full[2], o_done[2], o_free
  static constexpr int kNumBars = 4 + 2 * kAttnKvStages + 2 * kAttnBiasStages + 9;
  static constexpr int kTotal = kBarOff + kNumBars * 8 + 16;
  static constexpr int kLaunchBytes = kTotal + 1024;
  static constexpr int kCtasPerSm = kLaunchBytes * 2 <= 220 * 1024 ? 2 : 1;
};

// Operand descriptors for the Q / K tiles (K-major, head dim contiguous).
template <int DP>
__device__ __forceinline__ uint64_t qk_desc(uint32_t addr, int k) {
  if constexpr (DP == 32) {
    return sw64_desc(addr + k * 32, 16, 512);
  } else {
    return sw128_desc(addr + k * 32, 16, 1024);
  }
}

// [V | ones] as the MN-major B operand of [O | l] = P [V | 1] (N = head dim + 16,
// K = keys): the first swizzle-atom-wide N chunk is the V tile, the next one
// (at byte offset `lbo`) the ones block.
template <int DP>
__device__ __forceinline__ uint64_t v_desc(uint32_t addr, int kstep, uint32_t lbo) {
  if constexpr (DP == 32) {
    return sw64_desc(addr + kstep * 16 * 64, lbo, 512);
  } else {
    return sw128_desc(addr + kstep * 16 * 128, lbo, 1024);
  }
}

// Bias tile (128 queries x 64 keys, K-major, one 128-byte swizzle atom per row)
// as the A operand of the identity MMAs; kstep selects 16 keys.
__device__ __forceinline__ uint64_t p_desc(uint32_t addr, int kstep) {
  return sw128_desc(addr + kstep * 32, 16, 1024);
}

// Loads 32 consecutive TMEM columns of this thread's lane into dst[0..31].
__device__ __forceinline__ void tmem_ld32_to(uint32_t taddr, float* dst) {
  uint32_t r[32];
  __syncwarp();  // warp-collective
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
        "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]),
        "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]),
        "=r"(r[31])
      : "r"(taddr));
#pragma unroll
  for (int i = 0; i < 32; ++i) dst[i] = __uint_as_float(r[i]);
}

// Stores 32 consecutive TMEM columns of this thread's lane from src[0..31].
__device__ __forceinline__ void tmem_st32_from(uint32_t taddr, const float* src) {
  __syncwarp();
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16, "
      "%17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};" ::"r"(taddr),
      "r"(__float_as_uint(src[0])), "r"(__float_as_uint(src[1])), "r"(__float_as_uint(src[2])),
      "r"(__float_as_uint(src[3])), "r"(__float_as_uint(src[4])), "r"(__float_as_uint(src[5])),
      "r"(__float_as_uint(src[6])), "r"(__float_as_uint(src[7])), "r"(__float_as_uint(src[8])),
      "r"(__float_as_uint(src[9])), "r"(__float_as_uint(src[10])), "r"(__float_as_uint(src[11])),
      "r"(__float_as_uint(src[12])), "r"(__float_as_uint(src[13])), "r"(__float_as_uint(src[14])),
      "r"(__float_as_uint(src[15])), "r"(__float_as_uint(src[16])), "r"(__float_as_uint(src[17])),
      "r"(__float_as_uint(src[18])), "r"(__float_as_uint(src[19])), "r"(__float_as_uint(src[20])),
      "r"(__float_as_uint(src[21])), "r"(__float_as_uint(src[22])), "r"(__float_as_uint(src[23])),
      "r"(__float_as_uint(src[24])), "r"(__float_as_uint(src[25])), "r"(__float_as_uint(src[26])),
      "r"(__float_as_uint(src[27])), "r"(__float_as_uint(src[28])), "r"(__float_as_uint(src[29])),
      "r"(__float_as_uint(src[30])), "r"(__float_as_uint(src[31]))
      : "memory");
}

__device__ __forceinline__ void tmem_wait_ld() {
  __syncwarp();
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_wait_st() {
  __syncwarp();
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

// Stores 32 consecutive TMEM columns of this thread's lane from raw words.
__device__ __forceinline__ void tmem_st32_u(uint32_t taddr, const uint32_t* v) {
  __syncwarp();
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16, "
      "%17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};" ::"r"(taddr),
      "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]),
      "r"(v[8]), "r"(v[9]), "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15]),
      "r"(v[16]), "r"(v[17]), "r"(v[18]), "r"(v[19]), "r"(v[20]), "r"(v[21]), "r"(v[22]), "r"(v[23]),
      "r"(v[24]), "r"(v[25]), "r"(v[26]), "r"(v[27]), "r"(v[28]), "r"(v[29]), "r"(v[30]), "r"(v[31])
      : "memory");
}

// Stores 16 consecutive TMEM columns of this thread's lane from src[0..15].
__device__ __forceinline__ void tmem_st16_from(uint32_t taddr, const float* src) {
  __syncwarp();
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
      "{%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16};" ::"r"(taddr),
      "r"(__float_as_uint(src[0])), "r"(__float_as_uint(src[1])), "r"(__float_as_uint(src[2])),
      "r"(__float_as_uint(src[3])), "r"(__float_as_uint(src[4])), "r"(__float_as_uint(src[5])),
      "r"(__float_as_uint(src[6])), "r"(__float_as_uint(src[7])), "r"(__float_as_uint(src[8])),
      "r"(__float_as_uint(src[9])), "r"(__float_as_uint(src[10])), "r"(__float_as_uint(src[11])),
      "r"(__float_as_uint(src[12])), "r"(__float_as_uint(src[13])), "r"(__float_as_uint(src[14])),
      "r"(__float_as_uint(src[15]))
      : "memory");
}

// max with NaN propagation (a NaN logit must poison its row, as in the
// reference); the three-operand form is native on sm_100.
__device__ __forceinline__ float max_nan(float a, float b) {
  float r;
  asm("max.NaN.f32 %0, %1, %2;" : "=f"(r) : "f"(a), "f"(b));
  return r;
}
__device__ __forceinline__ float max3_nan(float a, float b, float c) {
  float r;
  asm("max.NaN.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
  return r;
}

// Maximum of 64 scores: 32 three-operand maxima in a tree of depth 4.
__device__ __forceinline__ float tile_max64(const float* s) {
  float a[22];
#pragma unroll
  for (int i = 0; i < 21; ++i) a[i] = max3_nan(s[3 * i], s[3 * i + 1], s[3 * i + 2]);
  a[21] = s[63];
  float b[8];
#pragma unroll
  for (int i = 0; i < 7; ++i) b[i] = max3_nan(a[3 * i], a[3 * i + 1], a[3 * i + 2]);
  b[7] = a[21];
  return max3_nan(max3_nan(b[0], b[1], b[2]), max3_nan(b[3], b[4], b[5]), max_nan(b[6], b[7]));
}

// 2^x for a pair of values on the FMA pipe (Cody-Waite range reduction plus a
// minimax polynomial).  x = j + f with j = rint(x) from the 1.5 * 2^23
// rounding constant and f in [-0.5, 0.5]; 2^f is the degree-3 polynomial
// below, fitted here to minimise the relative error on that interval (max
// 7.5e-5, well under the 2^-9 of the bf16 probabilities it feeds); 2^j is
// added to the exponent field as an integer.  Inputs are clamped at -125 so the
// exponent cannot underflow: 2^-125 stands for anything smaller, which is
// below f32 resolution next to the row max's 2^0.  A NaN input gives a finite
// value here; the MUFU share of the same row carries the NaN.
__device__ __forceinline__ float2 exp2_poly2(float2 x) {
  constexpr float kRound = 12582912.f;  // 1.5 * 2^23
  constexpr float c0 = 0.99992805719375610f, c1 = 0.69326096773147583f,
                  c2 = 0.24261112511157990f, c3 = 0.05517166852951050f;
  x.x = fmaxf(x.x, -125.f);
  x.y = fmaxf(x.y, -125.f);
  const float2 t = add2(x, make_float2(kRound, kRound));
  const float2 r = add2(t, make_float2(-kRound, -kRound));
  const float2 f = fma2(r, make_float2(-1.f, -1.f), x);
  float2 p = fma2(make_float2(c3, c3), f, make_float2(c2, c2));
  p = fma2(p, f, make_float2(c1, c1));
  p = fma2(p, f, make_float2(c0, c0));
  return make_float2(__uint_as_float(__float_as_uint(t.x) * 8388608u + __float_as_uint(p.x)),
                     __uint_as_float(__float_as_uint(t.y) * 8388608u + __float_as_uint(p.y)));
}

// Work item w -> (b, h, q-tile), query tiles fastest so concurrent CTAs share K / V.
__device__ __forceinline__ void attn_item(const AttnArgs& a, int w, int& b, int& h, int& qt) {
  qt = w % a.q_tiles;
  const int bh = w / a.q_tiles;
  b = bh / a.H;
  h = bh - b * a.H;
}

template <int DP, int BMODE, bool PRE>
__global__ void __launch_bounds__(kAttnThreads, AttnSmem<DP>::kCtasPerSm)
    flash_attn_kernel(const __grid_constant__ CUtensorMap tmQ,
                      const __grid_constant__ CUtensorMap tmK,
                      const __grid_constant__ CUtensorMap tmV,
                      const __grid_constant__ CUtensorMap tmBias, AttnArgs args) {
  static_assert(DP == 32 || DP == 64, "padded head dim must be 32 or 64");
  using L = AttnSmem<DP>;
  constexpr uint32_t kIdescS = idesc_bf16(128, kAttnBK, false, false);
  constexpr uint32_t kIdescO = idesc_bf16(128, DP + 16, false, true);  // O and l
  constexpr uint32_t kIdescL = idesc_bf16(128, 16, false, false);  // also the bias MMAs
  // TMEM columns: S 2 x 64 at 0, O at 128, l (16) after O, P 2 x 32 (bf16 pairs)
  constexpr uint32_t kOCol = 128;
  constexpr uint32_t kLCol = kOCol + DP;
  constexpr uint32_t kPCol = DP == 32 ? 192 : 224;
  constexpr uint32_t kTmemCols = kPCol + 64 <= 256 ? 256 : 512;

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint8_t* sQ = smem + L::kQOff;
  uint8_t* sK = smem + L::kKOff;
  uint8_t* sV = smem + L::kVOff;
  uint8_t* sBias = smem + L::kBiasOff;
  uint8_t* sOnes = smem + L::kOnesOff;
  uint8_t* sIdent = smem + L::kIdentOff;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::kBarOff);
  uint64_t* q_full = bars;
  uint64_t* q_empty = q_full + 2;
  uint64_t* kv_full = q_empty + 2;
  uint64_t* kv_empty = kv_full + kAttnKvStages;
  uint64_t* b_full = kv_empty + kAttnKvStages;
  uint64_t* b_empty = b_full + kAttnBiasStages;
  uint64_t* s_full = b_empty + kAttnBiasStages;
  uint64_t* s_free = s_full + 2;
  uint64_t* p_full = s_free + 2;
  uint64_t* o_done = p_full + 2;
  uint64_t* o_free = o_done + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + L::kNumBars);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int n_tiles = (args.nk + kAttnBK - 1) / kAttnBK;
  const int n_items = args.B * args.H * args.q_tiles;
  // this CTA's items are blockIdx.x, blockIdx.x + gridDim.x, ...
  const int my_items = static_cast<int>(blockIdx.x) < n_items
                           ? (n_items - 1 - static_cast<int>(blockIdx.x)) / gridDim.x + 1
                           : 0;
  const int total = my_items * n_tiles;
  const bool has_bias = args.bias != nullptr;

  if (threadIdx.x == 0) {
    for (int i = 0; i < 2; ++i) {
      mbar_init(&q_full[i], 1);
      mbar_init(&q_empty[i], 1);
      mbar_init(&s_full[i], 1);
      mbar_init(&s_free[i], 128);
      mbar_init(&p_full[i], 128);
      mbar_init(&o_done[i], 1);
    }
    for (int s = 0; s < kAttnKvStages; ++s) {
      mbar_init(&kv_full[s], 1);
      mbar_init(&kv_empty[s], 1);
    }
    for (int s = 0; s < kAttnBiasStages; ++s) {
      mbar_init(&b_full[s], 1);
      mbar_init(&b_empty[s], kAttnBiasMma ? 1 : 128);
    }
    mbar_init(o_free, 128);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 5) {
    tmem_alloc(tmem_slot, kTmemCols);
    tmem_relinquish();
  }
  if (warp < 4) {
    // the ones tile of the row-sum MMA (every element 1.0, so no swizzle matters)
    for (int i = threadIdx.x; i < L::kOnesBytes / 16; i += 128)
      reinterpret_cast<uint4*>(sOnes)[i] = make_uint4(0x3F803F80u, 0x3F803F80u, 0x3F803F80u,
                                                     0x3F803F80u);
    // identity: row n holds 1.0 at k = n, in the 128-byte swizzle (16-byte
    // chunk c of row n stored at chunk position c ^ (n % 8))
    for (int i = threadIdx.x; i < L::kIdentBytes / 16; i += 128) {
      const int n = i >> 3;
      const int c = (i & 7) ^ (n & 7);
      const uint32_t one = (n & 1) ? 0x3F800000u : 0x00003F80u;
      const int word = c == (n >> 3) ? (n & 7) >> 1 : -1;
      reinterpret_cast<uint4*>(sIdent)[i] =
          make_uint4(word == 0 ? one : 0u, word == 1 ? one : 0u, word == 2 ? one : 0u,
                     word == 3 ? one : 0u);
    }
    fence_async_smem();
  }
  if (warp == 4 && lane == 0) {
    tma_prefetch(&tmQ);
    tma_prefetch(&tmK);
    tma_prefetch(&tmV);
    if (BMODE == kBiasTma && has_bias) tma_prefetch(&tmBias);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp >= 4) {
  if constexpr (AttnSmem<DP>::kCtasPerSm == 2)
    asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(kAttnRegsOther));
  if (warp == 4) {
    // ------------------------------------------------ TMA producer
    if (lane == 0) {
      const bool tma_bias = BMODE == kBiasTma && has_bias;
      int g = 0;   // global key-tile counter (ring index)
      int it = 0;  // item counter of this CTA
      bool ok = true;
      for (int w = blockIdx.x; ok && w < n_items; w += gridDim.x, ++it) {
        int b, h, qt;
        attn_item(args, w, b, h, qt);
        const int bh = b * args.H + h;
        const int qb = it & 1;
        if (!mbar_wait(&q_empty[qb], ((it >> 1) & 1) ^ 1, kErrWaitProducer, abort_flag)) break;
        mbar_arrive_expect_tx(&q_full[qb], L::kQBytes);
        tma_load_3d(sQ + qb * L::kQBytes, &tmQ, &q_full[qb], 0, qt * 128, bh);
        const int bz = args.bias_batched ? bh : h;
        for (int t = 0; t < n_tiles; ++t, ++g) {
          const int st = g % kAttnKvStages;
          if (!mbar_wait(&kv_empty[st], ((g / kAttnKvStages) & 1) ^ 1, kErrWaitProducer,
                         abort_flag)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&kv_full[st], 2 * L::kKVBytes);
          tma_load_3d(sK + st * L::kKVBytes, &tmK, &kv_full[st], 0, t * kAttnBK, bh);
          tma_load_3d(sV + st * L::kKVBytes, &tmV, &kv_full[st], 0, t * kAttnBK, bh);
          if (tma_bias) {
            const int sb = g % kAttnBiasStages;
            if (!mbar_wait(&b_empty[sb], ((g / kAttnBiasStages) & 1) ^ 1, kErrWaitProducer,
                           abort_flag)) {
              ok = false;
              break;
            }
            mbar_arrive_expect_tx(&b_full[sb], L::kBiasBytes);
            tma_load_3d(sBias + sb * L::kBiasBytes, &tmBias, &b_full[sb], t * kAttnBK, qt * 128,
                        bz);
          }
        }
      }
    }
  } else if (warp == 5) {
    // ------------------------------------------------ S-MMA issuer
    // The CTA's key tiles form one sequence g = item * n_tiles + t.  S(g) is
    // issued as soon as its K / bias tiles have landed and the softmax has loaded
    // S(g - 2) from the same TMEM buffer; PV runs on its own issuer (warp 6), so
    // neither waits for the other's inputs.
    if (lane == 0) {
      const bool tma_bias = kAttnBiasMma && BMODE == kBiasTma && has_bias;
      const uint64_t ident_desc = sw128_desc(smem_u32(sIdent), 16, 1024);
      for (int gs = 0; gs < total; ++gs) {
        const int it = gs / n_tiles;
        const int t = gs - it * n_tiles;
        const int qb = it & 1;
        const int st = gs % kAttnKvStages;
        const int sb = gs & 1;
        const int sbias = gs % kAttnBiasStages;
        if (t == 0 && !mbar_wait(&q_full[qb], (it >> 1) & 1, kErrWaitMma, abort_flag)) break;
        if (!mbar_wait(&kv_full[st], (gs / kAttnKvStages) & 1, kErrWaitMma, abort_flag) ||
            !mbar_wait(&s_free[sb], ((gs >> 1) & 1) ^ 1, kErrWaitMma, abort_flag))
          break;
        if (tma_bias &&
            !mbar_wait(&b_full[sbias], (gs / kAttnBiasStages) & 1, kErrWaitMma, abort_flag))
          break;
        tc_fence_after();
        const uint32_t q_addr = smem_u32(sQ + qb * L::kQBytes);
        const uint32_t k_addr = smem_u32(sK + st * L::kKVBytes);
        if (tma_bias) {
          // S[:, 16j + n] = sum_k bias[:, 16j + k] * I[k][n]: exact in the f32 accumulator
          const uint32_t b_addr = smem_u32(sBias + sbias * L::kBiasBytes);
#pragma unroll
          for (int j = 0; j < kAttnBK / 16; ++j)
            umma_bf16(tmem_base + sb * kAttnBK + 16 * j, p_desc(b_addr, j), ident_desc, kIdescL, 0u);
        }
#pragma unroll
        for (int k = 0; k < DP / 16; ++k)
          umma_bf16(tmem_base + sb * kAttnBK, qk_desc<DP>(q_addr, k), qk_desc<DP>(k_addr, k),
                    kIdescS, (tma_bias || k > 0) ? 1u : 0u);
        umma_commit(&s_full[sb]);
        if (tma_bias) umma_commit(&b_empty[sbias]);
        if (t == n_tiles - 1) umma_commit(&q_empty[qb]);
      }
    }
  } else if (warp == 6) {
    // ------------------------------------------------ PV-MMA issuer
    // [O | l] += P(g) [V(g) | 1] once the softmax stored P(g) in TMEM.  S(g) read
    // K(g) before the softmax could produce P(g), so this commit frees the K / V
    // stage for both.
    if (lane == 0) {
      const uint32_t ones_addr = smem_u32(sOnes);
      for (int gp = 0; gp < total; ++gp) {
        const int it = gp / n_tiles;
        const int t = gp - it * n_tiles;
        const int st = gp % kAttnKvStages;
        const int pb = gp & 1;
        // the previous item's O must have been read before the first PV overwrites it
        if (t == 0 && it > 0 && !mbar_wait(o_free, (it - 1) & 1, kErrWaitMma, abort_flag)) break;
        if (!mbar_wait(&p_full[pb], (gp >> 1) & 1, kErrWaitMma, abort_flag)) break;
        tc_fence_after();
        const uint32_t v_addr = smem_u32(sV + st * L::kKVBytes);
        const uint32_t p_tmem = tmem_base + kPCol + pb * (kAttnBK / 2);  // 8 columns per 16 keys
#pragma unroll
        for (int j = 0; j < kAttnBK / 16; ++j)
          umma_bf16_ts(tmem_base + kOCol, p_tmem + 8 * j, v_desc<DP>(v_addr, j, ones_addr - v_addr),
                       kIdescO, (t > 0 || j > 0) ? 1u : 0u);
        umma_commit(&o_done[pb]);
        umma_commit(&kv_empty[st]);  // K and V of that tile are no longer read
      }
    }
  }
  } else {
    if constexpr (AttnSmem<DP>::kCtasPerSm == 2)
      asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(kAttnRegsSoftmax));
    // ------------------------------------------------ softmax warps 0-3
    const int row = warp * 32 + lane;
    const uint32_t t_row = tmem_base + (static_cast<uint32_t>(warp * 32) << 16);
    const int words = (args.nk + 31) / 32;
    // Scores stay in the units the MMA produced (log2 with PRE, natural
    // otherwise); kScale converts inside the exponent's FMA.
    constexpr float kScale = PRE ? 1.f : kLog2e;
    constexpr float kMasked = PRE ? -1e9f * kLog2e : -1e9f;
    const float2 scale2 = make_float2(kScale, kScale);
    int g = 0;
    bool ok = true;
    for (int w = blockIdx.x; w < n_items; w += gridDim.x) {
      int b, h, qt;
      attn_item(args, w, b, h, qt);
      const int q = qt * 128 + row;
      const bool q_ok = q < args.nq;
      const uint32_t* mrow = args.mask_bits ? args.mask_bits + b * args.mask_sb : nullptr;
      const void* brow = nullptr;
      if (BMODE != kBiasTma && has_bias && q_ok) {
        const int64_t off =
            b * args.bias_sb + h * args.bias_sh + static_cast<int64_t>(q) * args.bias_sq;
        brow = (BMODE == kBiasGlobalF32)
                   ? static_cast<const void*>(reinterpret_cast<const float*>(args.bias) + off)
                   : static_cast<const void*>(reinterpret_cast<const __nv_bfloat16*>(args.bias) + off);
      }
      float m_ref = -INFINITY;  // reference max, log2 units
      for (int t = 0; t < n_tiles; ++t) {
        const int gt = g + t;
        const int sb = gt & 1;
        const int key0 = t * kAttnBK;
        // mask words of this tile, loaded ahead of the waits
        uint32_t w0 = 0xFFFFFFFFu, w1 = 0xFFFFFFFFu;
        if (mrow != nullptr) {
          w0 = mrow[2 * t];
          w1 = (2 * t + 1 < words) ? mrow[2 * t + 1] : 0u;
        }
        // ---- S_t from TMEM
        ok = mbar_wait(&s_full[sb], (gt >> 1) & 1, kErrWaitSoftmax, abort_flag) && ok;
        tc_fence_after();
        float s[kAttnBK];
        tmem_ld32_to(t_row + sb * kAttnBK, s);
        tmem_ld32_to(t_row + sb * kAttnBK + 32, s + 32);
        tmem_wait_ld();
        tc_fence_before();
        mbar_arrive(&s_free[sb]);
        float2* s2 = reinterpret_cast<float2*>(s);
        // ---- bias (with kAttnBiasMma the TMA bias entered S in the MMA)
        if (!kAttnBiasMma && BMODE == kBiasTma && has_bias) {
          const int sbias = gt % kAttnBiasStages;
          ok = mbar_wait(&b_full[sbias], (gt / kAttnBiasStages) & 1, kErrWaitSoftmax, abort_flag) &&
               ok;
          const uint8_t* bt = sBias + sbias * L::kBiasBytes + row * 128;
#pragma unroll
          for (int c = 0; c < 8; ++c) {
            const uint4 wv = *reinterpret_cast<const uint4*>(bt + ((c ^ (row & 7)) << 4));
            const uint32_t ww[4] = {wv.x, wv.y, wv.z, wv.w};
#pragma unroll
            for (int e = 0; e < 4; ++e)
              s2[c * 4 + e] = add2(s2[c * 4 + e], make_float2(__uint_as_float(ww[e] << 16),
                                                              __uint_as_float(ww[e] & 0xFFFF0000u)));
          }
          mbar_arrive(&b_empty[sbias]);  // the values are in registers: the slot may refill
        } else if (brow != nullptr) {
#pragma unroll
          for (int j = 0; j < kAttnBK; ++j) {
            float bj = 0.f;
            if (key0 + j < args.nk) {
              bj = (BMODE == kBiasGlobalF32)
                       ? reinterpret_cast<const float*>(brow)[key0 + j]
                       : __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(brow)[key0 + j]);
            }
            s[j] += bj;
          }
        }
        // ---- key mask: masked -> -1e9, past the end -> -inf
        if (key0 + kAttnBK > args.nk || (w0 & w1) != 0xFFFFFFFFu) {
#pragma unroll
          for (int j = 0; j < kAttnBK; ++j) {
            const uint32_t bit = ((j < 32 ? w0 : w1) >> (j & 31)) & 1u;
            if (key0 + j >= args.nk) {
              s[j] = -INFINITY;
            } else if (!bit) {
              s[j] = kMasked;
            }
          }
        }
        // ---- tile max and lazy reference update (a NaN max always "grows")
        const float mt = tile_max64(s) * kScale;
        const bool grow = !(mt <= m_ref + 8.f);
        float factor = 1.f;
        if (grow) {
          factor = ex2_approx(m_ref - mt);  // 0 when m_ref = -inf
          m_ref = mt;
        }
        // O and l already hold earlier tiles of this item: rescale them in TMEM (rare).
        if (t > 0 && __any_sync(0xffffffffu, grow)) {
          const int gp = gt - 1;
          ok = mbar_wait(&o_done[gp & 1], (gp >> 1) & 1, kErrWaitSoftmax, abort_flag) && ok;
          tc_fence_after();
          float o[DP];
          float lv[16];
#pragma unroll
          for (int c = 0; c < DP / 32; ++c) tmem_ld32_to(t_row + kOCol + c * 32, o + c * 32);
          tmem_ld16(t_row + kLCol, lv);
#pragma unroll
          for (int i = 0; i < DP; ++i) o[i] *= factor;
#pragma unroll
          for (int i = 0; i < 16; ++i) lv[i] *= factor;
#pragma unroll
          for (int c = 0; c < DP / 32; ++c) tmem_st32_from(t_row + kOCol + c * 32, o + c * 32);
          tmem_st16_from(t_row + kLCol, lv);
          tmem_wait_st();
        }
        // ---- probabilities: 2^(s * kScale - m_ref), split between MUFU and FMA pipes
        {
          const float2 neg = make_float2(-m_ref, -m_ref);
#pragma unroll
          for (int j = 0; j < kAttnBK / 2; ++j) {
            float2 x = fma2(s2[j], scale2, neg);
            if ((j & 7) < kAttnPolyPairs) {
              x = exp2_poly2(x);
            } else {
              x.x = ex2_approx(x.x);
              x.y = ex2_approx(x.y);
            }
            s2[j] = x;
          }
        }
        // ---- P (bf16 pairs) into the TMEM columns of this parity; the PV MMA
        //      that read them last (tile g-2) must have completed.
        const int pb = gt & 1;
        if (gt >= 2) {
          ok = mbar_wait(&o_done[pb], ((gt - 2) >> 1) & 1, kErrWaitSoftmax, abort_flag) && ok;
        }
        uint32_t pk[kAttnBK / 2];
#pragma unroll
        for (int j = 0; j < kAttnBK / 2; ++j) pk[j] = pack_bf16x2(s[2 * j], s[2 * j + 1]);
        tmem_st32_u(t_row + kPCol + pb * (kAttnBK / 2), pk);
        tmem_wait_st();
        tc_fence_before();
        mbar_arrive(&p_full[pb]);
      }
      // ---- item epilogue: wait for the last PV, normalise, gate, store
      const int gl = g + n_tiles - 1;
      ok = mbar_wait(&o_done[gl & 1], (gl >> 1) & 1, kErrWaitSoftmax, abort_flag) && ok;
      tc_fence_after();
      float o[DP];
      float lv[16];
#pragma unroll
      for (int c = 0; c < DP / 32; ++c) tmem_ld32_to(t_row + kOCol + c * 32, o + c * 32);
      tmem_ld16(t_row + kLCol, lv);
      tc_fence_before();
      mbar_arrive(o_free);
      if (q_ok && ok) {
        const float inv_l = 1.f / lv[0];
        __nv_bfloat16* orow =
            args.out + b * args.out_sb + h * args.out_sh + static_cast<int64_t>(q) * args.out_sq;
        const __nv_bfloat16* grow_p =
            args.gate == nullptr ? nullptr
                                 : args.gate + b * args.gate_sb + h * args.gate_sh +
                                       static_cast<int64_t>(q) * args.gate_sq;
        const bool vec = (args.d == DP) && ((reinterpret_cast<uintptr_t>(orow) & 15) == 0) &&
                         (grow_p == nullptr || (reinterpret_cast<uintptr_t>(grow_p) & 15) == 0);
        if (vec) {
#pragma unroll
          for (int c = 0; c < DP / 8; ++c) {
            float v[8];
#pragma unroll
            for (int e = 0; e < 8; ++e) v[e] = o[c * 8 + e] * inv_l;
            if (grow_p != nullptr) {
              const uint4 gw = reinterpret_cast<const uint4*>(grow_p)[c];
              const uint32_t gg[4] = {gw.x, gw.y, gw.z, gw.w};
#pragma unroll
              for (int e = 0; e < 4; ++e) {
                v[2 * e] = bf16r(v[2 * e]) * __uint_as_float(gg[e] << 16);
                v[2 * e + 1] = bf16r(v[2 * e + 1]) * __uint_as_float(gg[e] & 0xFFFF0000u);
              }
            }
            uint4 pk;
            pk.x = pack_bf16x2(v[0], v[1]);
            pk.y = pack_bf16x2(v[2], v[3]);
            pk.z = pack_bf16x2(v[4], v[5]);
            pk.w = pack_bf16x2(v[6], v[7]);
            reinterpret_cast<uint4*>(orow)[c] = pk;
          }
        } else {
#pragma unroll
          for (int i = 0; i < DP; ++i) {
            if (i < args.d) {
              float v = bf16r(o[i] * inv_l);
              if (grow_p != nullptr) v = v * __bfloat162float(grow_p[i]);
              orow[i] = __float2bfloat16_rn(v);
            }
          }
        }
      }
      g += n_tiles;
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 5) {
    tc_fence_after();
    tmem_dealloc(tmem_base, kTmemCols);
  }
}

// Packs a key mask (f32 or uint8, nonzero = keep) into bits: out[r][k/32] bit k%32.
// Keys past nk are 0.
__global__ void pack_mask_bits_kernel(const void* mask, int is_float, int64_t rows, int nk,
                                      int64_t in_stride, uint32_t* out, int words) {
  const int64_t total = rows * words;
  for (int64_t idx = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; idx < total;
       idx += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t r = idx / words;
    const int wd = static_cast<int>(idx - r * words);
    uint32_t bits = 0;
    for (int j = 0; j < 32; ++j) {
      const int k = wd * 32 + j;
      if (k >= nk) break;
      bool keep;
      if (is_float) {
        keep = reinterpret_cast<const float*>(mask)[r * in_stride + k] != 0.f;
      } else {
        keep = reinterpret_cast<const uint8_t*>(mask)[r * in_stride + k] != 0;
      }
      bits |= static_cast<uint32_t>(keep) << j;
    }
    out[idx] = bits;
  }
}

}  // namespace xfb
