// Triangle attention (head dim <= 32, one bias shared by every batch row) on
// tcgen05 with three query tiles in flight per SM.
//
// With head dim 32 one score costs 4 d = 128 MMA FLOP but one ex2 on the MUFU
// unit (16 per clock per SM), and the MMAs are small (M = 128, N <= 64,
// K = 16), so the softmax warps and the tensor pipe bound this attention
// together, not the tensor FLOPs.  The one-tile-per-CTA kernel in attention.cuh
// keeps two softmax warps per SM sub-partition and leaves the MUFU unit idle
// half of the time while they wait on TMEM loads, stores and barriers.  This
// kernel runs one persistent CTA per SM with three softmax warpgroups, each
// owning its own query tile ("slot"), so three softmax warps share each
// sub-partition and cover each other's latencies.
//
// Work group = (head h, 128-query tile qt, batch rows 3j, 3j+1, 3j+2): slot s
// handles batch row 3j+s.  The bias tile bias[h, qt-rows, key-tile] is the
// same for the three rows, so it is loaded once per key tile and read by all
// three slots' S MMAs.  Per 64-key tile of a slot:
//   S   = bias + Q K^T   four identity MMAs (the bf16 bias enters the f32
//                        accumulator exactly) then the QK^T MMAs, into one of
//                        the slot's two 64-column S buffers (XFB_TRI_BIAS_MMA=0:
//                        the softmax adds the bias from shared memory instead)
//   P   = 2^(S - m_ref)  softmax warps, one query row per thread; P (bf16
//                        pairs) is written back over the first 32 columns of
//                        the same S buffer, and the row sum of the f32
//                        probabilities is kept in registers
//   O  += P V            tcgen05.mma with A = P from TMEM, V MN-major
// TMEM: slot s owns columns [160 s, 160 s + 160): S buffers at +0 and +64, O
// (32 columns) at +128; 480 of the 512 columns.
//
// Semantics are those of flash_attn_kernel (attention.cuh): masked keys get
// the logit -1e9, keys past the end probability 0, a NaN logit poisons its
// row, and the reference max m_ref moves lazily (only when a tile exceeds it
// by more than 2^8), rescaling O in TMEM and the row sum in registers.
#pragma once

#include "attention.cuh"
#include "common.cuh"

namespace xfb {

// Kernel shapes: TriCfg<SLOTS, BK> -- SLOTS query tiles in flight per SM (one
// softmax warpgroup each), key tiles of BK keys.  (3, 64) fills 480 of the 512
// TMEM columns with two 64-column S buffers and a 32-column O per slot; (4, 32)
// fills 384 with two 32-column S buffers and O per slot, for four softmax
// warps per SM sub-partition instead of three.  Control warpgroups follow the
// softmax ones: the TMA producer, then one MMA issuer per slot (the first
// issuer warp owns TMEM).
template <int SLOTS, int BK>
struct TriCfg {
  static constexpr int kSlots = SLOTS;
  static constexpr int kBK = BK;
  static constexpr int kCtlGroups = (SLOTS + 1 + 3) / 4;
  static constexpr int kThreads = (SLOTS + kCtlGroups) * 128;
  static constexpr int kProducerWarp = SLOTS * 4;
  static constexpr int kIssuerWarp0 = SLOTS * 4 + 1;
  static constexpr int kRegsLaunch = SLOTS == 3 ? 128 : 80;
  static constexpr int kRegsSoftmax = SLOTS == 3 ? 152 : 88;
  static constexpr int kRegsOther = SLOTS == 3 ? 56 : 64;
  static_assert(SLOTS * 128 * kRegsSoftmax + kCtlGroups * 128 * kRegsOther ==
                    kThreads * kRegsLaunch,
                "register split must add up to the launch allocation");
  static_assert(kThreads * kRegsLaunch <= 65536, "registers");
  static constexpr int kKvStages = 3;                    // per slot, freed by its PV MMA
  static constexpr int kBiasStages = SLOTS == 3 ? 3 : 4;  // shared, freed by every slot
  static constexpr int kSlotCols = 2 * BK + 32;          // two S buffers and O
  static constexpr int kOCol = 2 * BK;                   // within a slot
  static_assert(SLOTS * kSlotCols <= 512, "TMEM");
  static_assert(BK == 32 || BK == 64, "key tiles of 32 or 64");
};

// 1: the bias tile enters S through identity MMAs (tensor pipe); 0: the
// softmax warps add it from shared memory (ALU / FMA pipes; 64-key tiles only).
#ifndef XFB_TRI_BIAS_MMA
#define XFB_TRI_BIAS_MMA 1
#endif
constexpr bool kTriBiasMma = XFB_TRI_BIAS_MMA != 0;
// Of every 8 pairs of probabilities in a row tile, this many are computed by
// exp2_poly2 on the FMA pipe instead of ex2.approx on the MUFU unit.
#ifndef XFB_TRI_POLY_PAIRS
#define XFB_TRI_POLY_PAIRS 0
#endif
constexpr int kTriPolyPairs = XFB_TRI_POLY_PAIRS;

template <class C>
struct TriSmem {
  static constexpr int kQBytes = 128 * 32 * 2;          // 8 KB, 64-byte swizzle
  static constexpr int kKVBytes = C::kBK * 32 * 2;      // 64-byte swizzle
  static constexpr int kBiasBytes = 128 * C::kBK * 2;   // one swizzle atom per row
  static constexpr int kQOff = 0;                                            // [slot][2]
  static constexpr int kKOff = kQOff + C::kSlots * 2 * kQBytes;              // [slot][stage]
  static constexpr int kVOff = kKOff + C::kSlots * C::kKvStages * kKVBytes;  // [slot][stage]
  static constexpr int kBiasOff = kVOff + C::kSlots * C::kKvStages * kKVBytes;
  static constexpr int kIdentOff = kBiasOff + C::kBiasStages * kBiasBytes;
  static constexpr int kIdentBytes = 16 * 128;
  static constexpr int kBarOff = kIdentOff + kIdentBytes;
  // per slot: q_full[2], q_empty[2], kv_full[S], kv_empty[S], s_full[2],
  // p_full[2], pv_done[2], o_free;  shared: b_full[SB], b_empty[SB]
  static constexpr int kSlotBars = 4 + 2 * C::kKvStages + 7;
  static constexpr int kNumBars = C::kSlots * kSlotBars + 2 * C::kBiasStages;
  static constexpr int kTotal = kBarOff + kNumBars * 8 + 16;
  static constexpr int kLaunchBytes = kTotal + 1024;
  static_assert(kBiasOff % 1024 == 0 && kIdentOff % 1024 == 0, "swizzle alignment");
  static_assert(kKOff % 512 == 0 && kVOff % 512 == 0, "64-byte swizzle alignment");
  static_assert(kLaunchBytes <= 227 * 1024, "shared memory");
};

struct TriBars {
  uint64_t* q_full;   // [2]
  uint64_t* q_empty;  // [2]
  uint64_t* kv_full;  // [kKvStages]
  uint64_t* kv_empty;
  uint64_t* s_full;   // [2]
  uint64_t* p_full;   // [2]
  uint64_t* pv_done;  // [2]
  uint64_t* o_free;   // [1]
};

template <class C>
__device__ __forceinline__ TriBars tri_bars(uint64_t* base, int slot) {
  uint64_t* p = base + slot * TriSmem<C>::kSlotBars;
  TriBars b;
  b.q_full = p;
  b.q_empty = p + 2;
  b.kv_full = p + 4;
  b.kv_empty = p + 4 + C::kKvStages;
  b.s_full = p + 4 + 2 * C::kKvStages;
  b.p_full = b.s_full + 2;
  b.pv_done = b.p_full + 2;
  b.o_free = b.pv_done + 2;
  return b;
}

// Group index -> (head, query tile, first batch row); query tiles fastest so
// the CTAs running at the same time read the same rows' K / V from L2.
template <int SLOTS>
__device__ __forceinline__ void tri_group(const AttnArgs& a, int gi, int& h, int& qt, int& b0) {
  qt = gi % a.q_tiles;
  const int jh = gi / a.q_tiles;
  h = jh % a.H;
  b0 = (jh / a.H) * SLOTS;
}

// Maximum of 32 scores (NaN-propagating three-operand maxima).
__device__ __forceinline__ float tile_max32(const float* s) {
  float a[11];
#pragma unroll
  for (int i = 0; i < 10; ++i) a[i] = max3_nan(s[3 * i], s[3 * i + 1], s[3 * i + 2]);
  a[10] = max_nan(s[30], s[31]);
  const float b0 = max3_nan(a[0], a[1], a[2]), b1 = max3_nan(a[3], a[4], a[5]),
              b2 = max3_nan(a[6], a[7], a[8]), b3 = max_nan(a[9], a[10]);
  return max_nan(max3_nan(b0, b1, b2), b3);
}

// Stores 16 consecutive TMEM columns of this thread's lane from raw words.
__device__ __forceinline__ void tmem_st16_u(uint32_t taddr, const uint32_t* v) {
  __syncwarp();
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
      "{%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16};" ::"r"(taddr),
      "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]),
      "r"(v[8]), "r"(v[9]), "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15])
      : "memory");
}

// Bias tile as the A operand of the identity MMAs; kstep selects 16 keys.
template <int BK>
__device__ __forceinline__ uint64_t tri_bias_desc(uint32_t addr, int kstep) {
  if constexpr (BK == 64) {
    return sw128_desc(addr + kstep * 32, 16, 1024);
  } else {
    return sw64_desc(addr + kstep * 32, 16, 512);
  }
}

template <bool PRE, class C>
__global__ void __launch_bounds__(C::kThreads, 1)
    flash_tri_kernel(const __grid_constant__ CUtensorMap tmQ,
                     const __grid_constant__ CUtensorMap tmK,
                     const __grid_constant__ CUtensorMap tmV,
                     const __grid_constant__ CUtensorMap tmBias, AttnArgs args) {
  using L = TriSmem<C>;
  constexpr int kSlots = C::kSlots;
  constexpr int kBK = C::kBK;
  static_assert(kTriBiasMma || kBK == 64, "the softmax-side bias reads 64-key rows");
  constexpr uint32_t kIdescS = idesc_bf16(128, kBK, false, false);
  constexpr uint32_t kIdescO = idesc_bf16(128, 32, false, true);
  constexpr uint32_t kIdescB = idesc_bf16(128, 16, false, false);  // bias identity MMAs
  constexpr uint32_t kOCol = C::kOCol;  // within a slot

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint8_t* sQ = smem + L::kQOff;
  uint8_t* sK = smem + L::kKOff;
  uint8_t* sV = smem + L::kVOff;
  uint8_t* sBias = smem + L::kBiasOff;
  uint8_t* sIdent = smem + L::kIdentOff;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::kBarOff);
  uint64_t* b_full = bars + kSlots * L::kSlotBars;
  uint64_t* b_empty = b_full + C::kBiasStages;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + L::kNumBars);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int n_tiles = (args.nk + kBK - 1) / kBK;
  const int row_groups = (args.B + kSlots - 1) / kSlots;
  const int n_groups = row_groups * args.H * args.q_tiles;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kSlots; ++s) {
      const TriBars tb = tri_bars<C>(bars, s);
      for (int i = 0; i < 2; ++i) {
        mbar_init(&tb.q_full[i], 1);
        mbar_init(&tb.q_empty[i], 1);
        mbar_init(&tb.s_full[i], 1);
        mbar_init(&tb.p_full[i], 128);
        mbar_init(&tb.pv_done[i], 1);
      }
      for (int i = 0; i < C::kKvStages; ++i) {
        mbar_init(&tb.kv_full[i], 1);
        mbar_init(&tb.kv_empty[i], 1);
      }
      mbar_init(tb.o_free, 128);
    }
    for (int i = 0; i < C::kBiasStages; ++i) {
      mbar_init(&b_full[i], 1);
      // one MMA commit per slot, or one arrive per softmax warp
      mbar_init(&b_empty[i], kTriBiasMma ? kSlots : kSlots * 4);
    }
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == C::kIssuerWarp0) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  if (warp < 4) {
    // 16 x 16 identity in the 128-byte swizzle (chunk c of row n at c ^ (n % 8))
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
  if (warp == C::kProducerWarp && lane == 0) {
    tma_prefetch(&tmQ);
    tma_prefetch(&tmK);
    tma_prefetch(&tmV);
    tma_prefetch(&tmBias);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp >= C::kProducerWarp) {
    asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(C::kRegsOther));
    if (warp == C::kProducerWarp && lane == 0) {
      // ------------------------------------------------ TMA producer
      // Per group: the three slots' Q tiles, then per key tile the shared bias
      // tile and each slot's K / V.  Rows past B (only in the last row group)
      // read as zeros (TMA fills boxes outside the tensor) and are not stored.
      int it = 0, g = 0;
      bool ok = true;
      for (int gi = blockIdx.x; ok && gi < n_groups; gi += gridDim.x, ++it) {
        int h, qt, b0;
        tri_group<kSlots>(args, gi, h, qt, b0);
        const int qb = it & 1;
#pragma unroll
        for (int s = 0; s < kSlots; ++s) {
          const TriBars tb = tri_bars<C>(bars, s);
          if (!mbar_wait(&tb.q_empty[qb], ((it >> 1) & 1) ^ 1, kErrWaitProducer, abort_flag)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&tb.q_full[qb], L::kQBytes);
          tma_load_3d(sQ + (s * 2 + qb) * L::kQBytes, &tmQ, &tb.q_full[qb], 0, qt * 128,
                      (b0 + s) * args.H + h);
        }
        for (int t = 0; ok && t < n_tiles; ++t, ++g) {
          const int sb = g % C::kBiasStages;
          if (!mbar_wait(&b_empty[sb], ((g / C::kBiasStages) & 1) ^ 1, kErrWaitProducer,
                         abort_flag)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&b_full[sb], L::kBiasBytes);
          tma_load_3d(sBias + sb * L::kBiasBytes, &tmBias, &b_full[sb], t * kBK, qt * 128, h);
          const int st = g % C::kKvStages;
#pragma unroll
          for (int s = 0; s < kSlots; ++s) {
            const TriBars tb = tri_bars<C>(bars, s);
            if (!mbar_wait(&tb.kv_empty[st], ((g / C::kKvStages) & 1) ^ 1, kErrWaitProducer,
                           abort_flag)) {
              ok = false;
              break;
            }
            const int bh = (b0 + s) * args.H + h;
            mbar_arrive_expect_tx(&tb.kv_full[st], 2 * L::kKVBytes);
            tma_load_3d(sK + (s * C::kKvStages + st) * L::kKVBytes, &tmK, &tb.kv_full[st], 0,
                        t * kBK, bh);
            tma_load_3d(sV + (s * C::kKvStages + st) * L::kKVBytes, &tmV, &tb.kv_full[st], 0,
                        t * kBK, bh);
          }
        }
      }
    } else if (warp >= C::kIssuerWarp0 && warp < C::kIssuerWarp0 + kSlots && lane == 0) {
      // ------------------------------------------------ MMA issuer of one slot
      // Tile sequence g = item * n_tiles + t (the same for every slot, and the
      // index of the shared bias tile).  One tile of lookahead:
      //   S(g + 1) once PV(g - 1), which read P from the same TMEM buffer, is done;
      //   PV(g)    once the softmax stored P(g).
      const int s = warp - C::kIssuerWarp0;
      const TriBars tb = tri_bars<C>(bars, s);
      const uint32_t slot_tmem = tmem_base + s * C::kSlotCols;
      const uint64_t ident_desc = sw128_desc(smem_u32(sIdent), 16, 1024);
      const int my_groups =
          static_cast<int>(blockIdx.x) < n_groups
              ? (n_groups - 1 - static_cast<int>(blockIdx.x)) / static_cast<int>(gridDim.x) + 1
              : 0;
      const int total = my_groups * n_tiles;
      // issues S(gs); false if a wait gave up
      auto issue_s = [&](int gs) -> bool {
        const int it = gs / n_tiles;
        const int t = gs - it * n_tiles;
        const int qb = it & 1;
        const int st = gs % C::kKvStages;
        const int sb = gs % C::kBiasStages;
        const int buf = gs & 1;
        if ((t == 0 && !mbar_wait(&tb.q_full[qb], (it >> 1) & 1, kErrWaitMma, abort_flag)) ||
            (kTriBiasMma &&
             !mbar_wait(&b_full[sb], (gs / C::kBiasStages) & 1, kErrWaitMma, abort_flag)) ||
            !mbar_wait(&tb.kv_full[st], (gs / C::kKvStages) & 1, kErrWaitMma, abort_flag) ||
            (gs >= 2 &&
             !mbar_wait(&tb.pv_done[buf], ((gs - 2) >> 1) & 1, kErrWaitMma, abort_flag)))
          return false;
        tc_fence_after();
        const uint32_t d_tmem = slot_tmem + buf * kBK;
        const uint32_t q_addr = smem_u32(sQ + (s * 2 + qb) * L::kQBytes);
        const uint32_t k_addr = smem_u32(sK + (s * C::kKvStages + st) * L::kKVBytes);
        if (kTriBiasMma) {
          // S[:, 16j + n] = sum_k bias[:, 16j + k] I[k][n]: exact in the f32 accumulator
          const uint32_t b_addr = smem_u32(sBias + sb * L::kBiasBytes);
#pragma unroll
          for (int j = 0; j < kBK / 16; ++j)
            umma_bf16(d_tmem + 16 * j, tri_bias_desc<kBK>(b_addr, j), ident_desc, kIdescB, 0u);
        }
#pragma unroll
        for (int k = 0; k < 2; ++k)
          umma_bf16(d_tmem, qk_desc<32>(q_addr, k), qk_desc<32>(k_addr, k), kIdescS,
                    (kTriBiasMma || k > 0) ? 1u : 0u);
        umma_commit(&tb.s_full[buf]);
        if (kTriBiasMma) umma_commit(&b_empty[sb]);  // this slot is done with the bias tile
        if (t == n_tiles - 1) umma_commit(&tb.q_empty[qb]);
        return true;
      };
      bool ok = total == 0 || issue_s(0);
      for (int gp = 0; ok && gp < total; ++gp) {
        if (gp + 1 < total && !issue_s(gp + 1)) break;
        const int it = gp / n_tiles;
        const int t = gp - it * n_tiles;
        const int st = gp % C::kKvStages;
        const int buf = gp & 1;
        // the previous item must have read O before its first PV overwrites it
        if ((t == 0 && it > 0 && !mbar_wait(tb.o_free, (it - 1) & 1, kErrWaitMma, abort_flag)) ||
            !mbar_wait(&tb.p_full[buf], (gp >> 1) & 1, kErrWaitMma, abort_flag))
          break;
        tc_fence_after();
        const uint32_t v_addr = smem_u32(sV + (s * C::kKvStages + st) * L::kKVBytes);
        const uint32_t p_tmem = slot_tmem + buf * kBK;  // 8 columns per 16 keys
#pragma unroll
        for (int j = 0; j < kBK / 16; ++j)
          umma_bf16_ts(slot_tmem + kOCol, p_tmem + 8 * j, v_desc<32>(v_addr, j, L::kKVBytes),
                       kIdescO, (t > 0 || j > 0) ? 1u : 0u);
        umma_commit(&tb.pv_done[buf]);
        umma_commit(&tb.kv_empty[st]);  // K (read by S) and V of this tile are done
      }
    }
  } else {
    asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(C::kRegsSoftmax));
    // ------------------------------------------------ softmax warpgroups
    const int slot = warp >> 2;
    const int row = (warp & 3) * 32 + lane;
    const TriBars tb = tri_bars<C>(bars, slot);
    const uint32_t t_row =
        tmem_base + (static_cast<uint32_t>((warp & 3) * 32) << 16) + slot * C::kSlotCols;
    const int words = (args.nk + 31) / 32;
    constexpr float kScale = PRE ? 1.f : kLog2e;
    constexpr float kMasked = PRE ? -1e9f * kLog2e : -1e9f;
    const float2 scale2 = make_float2(kScale, kScale);
    int g = 0;
    bool ok = true;
    for (int gi = blockIdx.x; gi < n_groups; gi += gridDim.x) {
      int h, qt, b0;
      tri_group<kSlots>(args, gi, h, qt, b0);
      const int b = b0 + slot;
      const bool b_ok = b < args.B;  // rows past B (last row group) run on zeros, unstored
      const int q = qt * 128 + row;
      const uint32_t* mrow =
          (args.mask_bits != nullptr && b_ok) ? args.mask_bits + b * args.mask_sb : nullptr;
      float m_ref = -INFINITY;  // reference max, log2 units
      float2 lsum[4] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f),
                        make_float2(0.f, 0.f)};
      for (int t = 0; t < n_tiles; ++t, ++g) {
        const int buf = g & 1;
        const int key0 = t * kBK;
        uint32_t w0 = 0xFFFFFFFFu, w1 = 0xFFFFFFFFu;
        if (mrow != nullptr) {
          if constexpr (kBK == 64) {
            w0 = mrow[2 * t];
            w1 = (2 * t + 1 < words) ? mrow[2 * t + 1] : 0u;
          } else {
            w0 = mrow[t];
          }
        }
        // this row of the shared bias tile (128-byte swizzle: 16-byte chunk c of
        // row r sits at chunk c ^ (r % 8)), read before S is waited for
        uint4 bw[kBK / 8];
        if (!kTriBiasMma) {
          const int sbias = g % C::kBiasStages;
          ok = mbar_wait(&b_full[sbias], (g / C::kBiasStages) & 1, kErrWaitSoftmax, abort_flag) &&
               ok;
          const uint8_t* brow = sBias + sbias * L::kBiasBytes + row * 128;
#pragma unroll
          for (int c = 0; c < kBK / 8; ++c)
            bw[c] = *reinterpret_cast<const uint4*>(brow + ((c ^ (row & 7)) << 4));
          __syncwarp();
          if (lane == 0) mbar_arrive(&b_empty[sbias]);  // the warp's values are in registers
        }
        ok = mbar_wait(&tb.s_full[buf], (g >> 1) & 1, kErrWaitSoftmax, abort_flag) && ok;
        tc_fence_after();
        float s[kBK];
        float2* s2 = reinterpret_cast<float2*>(s);
        // S of this tile from TMEM, with the bias (softmax-side variant) and the
        // key mask applied: masked -> -1e9, past the end -> -inf
        auto load_scores = [&]() {
          tmem_ld32_to(t_row + buf * kBK, s);
          if constexpr (kBK == 64) tmem_ld32_to(t_row + buf * kBK + 32, s + 32);
          tmem_wait_ld();
          if (!kTriBiasMma) {
#pragma unroll
            for (int c = 0; c < kBK / 8; ++c) {
              const uint32_t ww[4] = {bw[c].x, bw[c].y, bw[c].z, bw[c].w};
#pragma unroll
              for (int e = 0; e < 4; ++e)
                s2[c * 4 + e] = add2(s2[c * 4 + e],
                                     make_float2(__uint_as_float(ww[e] << 16),
                                                 __uint_as_float(ww[e] & 0xFFFF0000u)));
            }
          }
          if (key0 + kBK > args.nk || (w0 & w1) != 0xFFFFFFFFu) {
#pragma unroll
            for (int j = 0; j < kBK; ++j) {
              const uint32_t bit = ((j < 32 ? w0 : w1) >> (j & 31)) & 1u;
              if (key0 + j >= args.nk) {
                s[j] = -INFINITY;
              } else if (!bit) {
                s[j] = kMasked;
              }
            }
          }
        };
        load_scores();
        uint32_t pk[kBK / 2];
        // probabilities 2^(s * kScale - m) of this tile into pk, their f32 sum into ts
        float2 ts[4];
        auto exponentiate = [&](float m) {
          const float2 neg = make_float2(-m, -m);
#pragma unroll
          for (int i = 0; i < 4; ++i) ts[i] = make_float2(0.f, 0.f);
#pragma unroll
          for (int j = 0; j < kBK / 2; ++j) {
            float2 x = fma2(s2[j], scale2, neg);
            if ((j & 7) < kTriPolyPairs) {
              x = exp2_poly2(x);
            } else {
              x.x = ex2_approx(x.x);
              x.y = ex2_approx(x.y);
            }
            ts[j & 3] = add2(ts[j & 3], x);
            pk[j] = pack_bf16x2(x.x, x.y);
          }
        };
        // rescales O (earlier tiles of this item) by `factor` once PV(g - 1) is done
        auto rescale_o = [&](float factor) {
          const int gp = g - 1;
          ok = mbar_wait(&tb.pv_done[gp & 1], (gp >> 1) & 1, kErrWaitSoftmax, abort_flag) && ok;
          tc_fence_after();
          float o[32];
          tmem_ld32_to(t_row + kOCol, o);
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 32; ++i) o[i] *= factor;
          tmem_st32_from(t_row + kOCol, o);
          tmem_wait_st();
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            lsum[i].x *= factor;
            lsum[i].y *= factor;
          }
        };
        // ---- tile max and lazy reference update (a NaN max always "grows")
        {
          const float mt = (kBK == 64 ? tile_max64(s) : tile_max32(s)) * kScale;
          const bool grow = !(mt <= m_ref + 8.f);
          float factor = 1.f;
          if (grow) {
            factor = ex2_approx(m_ref - mt);  // 0 when m_ref = -inf
            m_ref = mt;
          }
          if (t > 0 && __any_sync(0xffffffffu, grow)) rescale_o(factor);
          exponentiate(m_ref);
        }
#pragma unroll
        for (int i = 0; i < 4; ++i) lsum[i] = add2(lsum[i], ts[i]);
        // P over the S columns this thread just read (the next S MMA into this
        // buffer waits for the PV MMA that reads P)
        if constexpr (kBK == 64) {
          tmem_st32_u(t_row + buf * kBK, pk);
        } else {
          tmem_st16_u(t_row + buf * kBK, pk);
        }
        tmem_wait_st();
        tc_fence_before();
        mbar_arrive(&tb.p_full[buf]);
      }
      // ---- item epilogue: last PV, normalise, gate, store
      const bool store = b_ok && q < args.nq;
      __nv_bfloat16* orow =
          args.out + b * args.out_sb + h * args.out_sh + static_cast<int64_t>(q) * args.out_sq;
      const __nv_bfloat16* grow_p =
          args.gate == nullptr ? nullptr
                               : args.gate + b * args.gate_sb + h * args.gate_sh +
                                     static_cast<int64_t>(q) * args.gate_sq;
      const bool vec = (args.d == 32) && ((reinterpret_cast<uintptr_t>(orow) & 15) == 0) &&
                       (grow_p == nullptr || (reinterpret_cast<uintptr_t>(grow_p) & 15) == 0);
      const int gl = g - 1;
      ok = mbar_wait(&tb.pv_done[gl & 1], (gl >> 1) & 1, kErrWaitSoftmax, abort_flag) && ok;
      tc_fence_after();
      float o[32];
      tmem_ld32_to(t_row + kOCol, o);
      tmem_wait_ld();
      tc_fence_before();
      mbar_arrive(tb.o_free);
      if (store && ok) {
        const float l = (lsum[0].x + lsum[0].y) + (lsum[1].x + lsum[1].y) +
                        ((lsum[2].x + lsum[2].y) + (lsum[3].x + lsum[3].y));
        const float inv_l = 1.f / l;
        if (vec) {
#pragma unroll
          for (int c = 0; c < 4; ++c) {
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
            uint4 pkd;
            pkd.x = pack_bf16x2(v[0], v[1]);
            pkd.y = pack_bf16x2(v[2], v[3]);
            pkd.z = pack_bf16x2(v[4], v[5]);
            pkd.w = pack_bf16x2(v[6], v[7]);
            reinterpret_cast<uint4*>(orow)[c] = pkd;
          }
        } else {
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            if (i < args.d) {
              float v = bf16r(o[i] * inv_l);
              if (grow_p != nullptr) v = v * __bfloat162float(grow_p[i]);
              orow[i] = __float2bfloat16_rn(v);
            }
          }
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == C::kIssuerWarp0) {
    tc_fence_after();
    tmem_dealloc(tmem_base, 512);
  }
}

}  // namespace xfb
