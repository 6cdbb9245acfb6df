// Flash attention with pair bias, key mask and fused sigmoid output gate on
// tcgen05 (sm_100a).
//
// One CTA owns 128 queries of one (batch row, head).  Per 128-key tile:
//   S  = Q K^T            tcgen05.mma, Q/K from TMA-loaded swizzled SMEM, S in TMEM
//   P  = exp(S + bias - m) online softmax in f32 by 4 warps (one query row per
//                          thread); the bias tile is TMA-streamed into swizzled
//                          SMEM with K and V; P is written as bf16 into a
//                          128B-swizzled SMEM tile
//   O_t = P V             tcgen05.mma with V read MN-major straight from its
//                          [key][head_dim] layout, O_t in TMEM
//   O  = O * 2^(m_old-m_new) + O_t   accumulated in registers
// S and O_t are double-buffered in TMEM so the S MMA of tile t+1 overlaps the
// softmax of tile t.
//
// Mask semantics follow the reference: a masked key gets the logit -1e9 (so a
// fully masked row is a uniform average), keys past the sequence end (tile
// padding) get probability exactly 0, and a NaN logit makes the row NaN.
#pragma once

#include "common.cuh"

namespace xfb {

constexpr int kAttnThreads = 192;
constexpr int kAttnKvStages = 2;

// Bias source: streamed bf16 tiles through TMA, or per-thread global loads.
enum AttnBiasMode : int { kBiasTma = 0, kBiasGlobalBf16 = 1, kBiasGlobalF32 = 2 };

struct AttnArgs {
  int B, H, nq, nk, d;      // d: real head dim (<= DP)
  const void* mask;         // key mask [B][nk] (row stride mask_sb, 0 = shared), or null
  int mask_is_float;        // 1: f32 mask (!= 0 is kept), 0: uint8 / bool mask
  int64_t mask_sb;
  const void* bias;         // bias[b*sb + h*sh + q*sq + key], or null
  int64_t bias_sb, bias_sh, bias_sq;
  int bias_batched;         // TMA bias map: z = b*H + h when set, else z = h
  __nv_bfloat16* out;       // out[b*sb + h*sh + q*sq + dd]
  int64_t out_sb, out_sh, out_sq;
  const __nv_bfloat16* gate;  // optional gate, same indexing as out (already squashed)
  int64_t gate_sb, gate_sh, gate_sq;
};

template <int DP>
struct AttnSmem {
  static constexpr int kQBytes = 128 * DP * 2;
  static constexpr int kKVBytes = 128 * DP * 2;
  static constexpr int kBiasBytes = 128 * 128 * 2;  // two 64-key swizzle atoms
  static constexpr int kPBytes = 128 * 128 * 2;
  static constexpr int kKVStride = ((kKVBytes + 1023) / 1024) * 1024;
  static constexpr int kQOff = 0;
  static constexpr int kKOff = kQOff + ((kQBytes + 1023) / 1024) * 1024;
  static constexpr int kVOff = kKOff + kAttnKvStages * kKVStride;
  static constexpr int kBiasOff = kVOff + kAttnKvStages * kKVStride;
  static constexpr int kPOff = kBiasOff + kAttnKvStages * kBiasBytes;
  static constexpr int kMaskOff = kPOff + 2 * kPBytes;
  static constexpr int kMaxKeys = 8192;
  static constexpr int kFlagOff = kMaskOff + kMaxKeys;       // one byte per key tile
  static constexpr int kBarOff = kFlagOff + kMaxKeys / 128;  // 8-byte aligned
  // q_full, kv_full[S], kv_empty[S], s_full[2], s_free[2], p_full[2], o_full[2], o_free[2]
  static constexpr int kNumBars = 1 + 2 * kAttnKvStages + 10;
  static constexpr int kTotal = kBarOff + kNumBars * 8 + 16;
  static constexpr int kLaunchBytes = kTotal + 1024;
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

// V tile as the MN-major B operand of O = P V (N = head dim, K = keys).
template <int DP>
__device__ __forceinline__ uint64_t v_desc(uint32_t addr, int kstep) {
  if constexpr (DP == 32) {
    return sw64_desc(addr + kstep * 16 * 64, 8192, 512);
  } else {
    return sw128_desc(addr + kstep * 16 * 128, 8192, 1024);
  }
}

// P tile (128 queries x 128 keys, K-major, two 64-key swizzle atoms).
__device__ __forceinline__ uint64_t p_desc(uint32_t addr, int kstep) {
  return sw128_desc(addr + (kstep >> 2) * 16384 + (kstep & 3) * 32, 16, 1024);
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

__device__ __forceinline__ void tmem_wait_ld() {
  __syncwarp();
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

template <int DP, int BMODE>
__global__ void __launch_bounds__(kAttnThreads, 1)
    flash_attn_kernel(const __grid_constant__ CUtensorMap tmQ,
                      const __grid_constant__ CUtensorMap tmK,
                      const __grid_constant__ CUtensorMap tmV,
                      const __grid_constant__ CUtensorMap tmBias, AttnArgs args) {
  static_assert(DP == 32 || DP == 64, "padded head dim must be 32 or 64");
  using L = AttnSmem<DP>;
  constexpr uint32_t kIdescS = idesc_bf16(128, 128, false, false);
  constexpr uint32_t kIdescO = idesc_bf16(128, DP, false, true);
  constexpr uint32_t kTmemCols = 512;  // S: 2 x 128 columns, O_t: 2 x DP columns
  constexpr float kLog2e = 1.4426950408889634f;

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint8_t* sQ = smem + L::kQOff;
  uint8_t* sK = smem + L::kKOff;
  uint8_t* sV = smem + L::kVOff;
  uint8_t* sBias = smem + L::kBiasOff;
  uint8_t* sP = smem + L::kPOff;
  uint8_t* sMask = smem + L::kMaskOff;
  uint8_t* sFlag = smem + L::kFlagOff;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::kBarOff);
  uint64_t* q_full = bars;
  uint64_t* kv_full = bars + 1;
  uint64_t* kv_empty = kv_full + kAttnKvStages;
  uint64_t* s_full = kv_empty + kAttnKvStages;
  uint64_t* s_free = s_full + 2;
  uint64_t* p_full = s_free + 2;
  uint64_t* o_full = p_full + 2;
  uint64_t* o_free = o_full + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + L::kNumBars);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int q0 = blockIdx.x * 128;
  const int bh = blockIdx.y;
  const int b = bh / args.H;
  const int h = bh - b * args.H;
  const int n_tiles = (args.nk + 127) / 128;
  const bool has_bias = args.bias != nullptr;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int s = 0; s < kAttnKvStages; ++s) {
      mbar_init(&kv_full[s], 1);
      mbar_init(&kv_empty[s], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&s_free[i], 128);
      mbar_init(&p_full[i], 128);
      mbar_init(&o_full[i], 1);
      mbar_init(&o_free[i], 128);
    }
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 5) {
    tmem_alloc(tmem_slot, kTmemCols);
    tmem_relinquish();
  }
  if (warp == 4 && lane == 0) {
    tma_prefetch(&tmQ);
    tma_prefetch(&tmK);
    tma_prefetch(&tmV);
    if (BMODE == kBiasTma && has_bias) tma_prefetch(&tmBias);
  }
  // Stage this batch row's key mask (1 = keep) and per-tile "all kept" flags.
  if (warp < 4) {
    for (int kk = threadIdx.x; kk < n_tiles * 128; kk += 128) {
      uint8_t keep = 0;
      if (kk < args.nk) {
        if (args.mask == nullptr) {
          keep = 1;
        } else if (args.mask_is_float) {
          keep = reinterpret_cast<const float*>(args.mask)[b * args.mask_sb + kk] != 0.f;
        } else {
          keep = reinterpret_cast<const uint8_t*>(args.mask)[b * args.mask_sb + kk] != 0;
        }
      }
      sMask[kk] = keep;
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp < 4) {
    for (int t = threadIdx.x; t < n_tiles; t += 128) {
      int all = 1;
      for (int j = 0; j < 128; ++j) all &= sMask[t * 128 + j];
      sFlag[t] = static_cast<uint8_t>(all);
    }
  }
  __syncthreads();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 4) {
    // ------------------------------------------------ TMA producer
    if (lane == 0) {
      const bool tma_bias = BMODE == kBiasTma && has_bias;
      const int bz = args.bias_batched ? bh : h;
      const uint32_t stage_bytes = 2 * L::kKVBytes + (tma_bias ? L::kBiasBytes : 0);
      mbar_arrive_expect_tx(q_full, L::kQBytes);
      tma_load_3d(sQ, &tmQ, q_full, 0, q0, bh);
      for (int t = 0; t < n_tiles; ++t) {
        const int st = t % kAttnKvStages;
        const uint32_t ph = (t / kAttnKvStages) & 1;
        if (!mbar_wait(&kv_empty[st], ph ^ 1, kErrWaitProducer, abort_flag)) break;
        mbar_arrive_expect_tx(&kv_full[st], stage_bytes);
        tma_load_3d(sK + st * L::kKVStride, &tmK, &kv_full[st], 0, t * 128, bh);
        tma_load_3d(sV + st * L::kKVStride, &tmV, &kv_full[st], 0, t * 128, bh);
        if (tma_bias) {
          uint8_t* dst = sBias + st * L::kBiasBytes;
          tma_load_3d(dst, &tmBias, &kv_full[st], t * 128, q0, bz);
          tma_load_3d(dst + 16384, &tmBias, &kv_full[st], t * 128 + 64, q0, bz);
        }
      }
    }
  } else if (warp == 5) {
    // ------------------------------------------------ MMA issuer
    if (lane == 0) {
      bool ok = mbar_wait(q_full, 0, kErrWaitMma, abort_flag);
      const uint32_t q_addr = smem_u32(sQ);
      const uint32_t p_addr0 = smem_u32(sP);
      for (int t = 0; ok && t <= n_tiles; ++t) {
        if (t < n_tiles) {
          const int st = t % kAttnKvStages;
          if (!mbar_wait(&kv_full[st], (t / kAttnKvStages) & 1, kErrWaitMma, abort_flag)) break;
          if (!mbar_wait(&s_free[t & 1], ((t >> 1) & 1) ^ 1, kErrWaitMma, abort_flag)) break;
          tc_fence_after();
          const uint32_t k_addr = smem_u32(sK + st * L::kKVStride);
          const uint32_t s_col = (t & 1) * 128;
#pragma unroll
          for (int k = 0; k < DP / 16; ++k)
            umma_bf16(tmem_base + s_col, qk_desc<DP>(q_addr, k), qk_desc<DP>(k_addr, k),
                      kIdescS, k > 0 ? 1u : 0u);
          umma_commit(&s_full[t & 1]);
        }
        if (t >= 1) {
          const int u = t - 1;
          const int st = u % kAttnKvStages;
          if (!mbar_wait(&p_full[u & 1], (u >> 1) & 1, kErrWaitMma, abort_flag)) break;
          if (!mbar_wait(&o_free[u & 1], ((u >> 1) & 1) ^ 1, kErrWaitMma, abort_flag)) break;
          tc_fence_after();
          const uint32_t v_addr = smem_u32(sV + st * L::kKVStride);
          const uint32_t p_addr = p_addr0 + (u & 1) * L::kPBytes;
          const uint32_t o_col = 256 + (u & 1) * DP;
#pragma unroll
          for (int j = 0; j < 8; ++j)
            umma_bf16(tmem_base + o_col, p_desc(p_addr, j), v_desc<DP>(v_addr, j), kIdescO,
                      j > 0 ? 1u : 0u);
          umma_commit(&o_full[u & 1]);
          umma_commit(&kv_empty[st]);  // K, V and bias of tile u are no longer read
        }
      }
    }
  } else {
    // ------------------------------------------------ softmax warps 0-3
    const int row = warp * 32 + lane;
    const int q = q0 + row;
    const bool q_ok = q < args.nq;
    const uint32_t t_row = tmem_base + (static_cast<uint32_t>(warp * 32) << 16);
    const void* brow = nullptr;  // global bias row (non-TMA modes)
    if (BMODE != kBiasTma && has_bias && q_ok) {
      const int64_t off = b * args.bias_sb + h * args.bias_sh + static_cast<int64_t>(q) * args.bias_sq;
      brow = (BMODE == kBiasGlobalF32)
                 ? static_cast<const void*>(reinterpret_cast<const float*>(args.bias) + off)
                 : static_cast<const void*>(reinterpret_cast<const __nv_bfloat16*>(args.bias) + off);
    }
    // Running maxima are kept in the log2 domain.
    float m_run = -INFINITY, l_run = 0.f;
    float m_prev = -INFINITY;  // max used for the P of the previous tile
    float m_acc = -INFINITY;   // reference max of o_acc
    float o_acc[DP];
#pragma unroll
    for (int i = 0; i < DP; ++i) o_acc[i] = 0.f;
    bool ok = true;

    for (int t = 0; t < n_tiles; ++t) {
      const int key0 = t * 128;
      const int st = t % kAttnKvStages;
      if (!mbar_wait(&s_full[t & 1], (t >> 1) & 1, kErrWaitSoftmax, abort_flag)) {
        ok = false;
        break;
      }
      tc_fence_after();
      float s[128];
      const uint32_t s_col = (t & 1) * 128;
#pragma unroll
      for (int c = 0; c < 4; ++c) tmem_ld32_to(t_row + s_col + c * 32, s + c * 32);
      tmem_wait_ld();
      tc_fence_before();
      mbar_arrive(&s_free[t & 1]);

      // Work in the log2 domain: s2 = (qk + bias) * log2(e).  Masked keys all get
      // the same constant, so a fully masked row stays exactly uniform.
      if (BMODE == kBiasTma && has_bias) {
        // The bias tile landed with K/V of this stage (already complete: the S
        // MMA of this tile waited for it); observe the phase for visibility.
        if (!mbar_wait(&kv_full[st], (t / kAttnKvStages) & 1, kErrWaitSoftmax, abort_flag)) {
          ok = false;
          break;
        }
        const uint8_t* bt = sBias + st * L::kBiasBytes + row * 128;
#pragma unroll
        for (int c = 0; c < 16; ++c) {
          const int phys = (c & 7) ^ (row & 7);
          const uint4 w = *reinterpret_cast<const uint4*>(bt + (c >> 3) * 16384 + phys * 16);
          const uint32_t ww[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            s[c * 8 + 2 * e] = (s[c * 8 + 2 * e] + __uint_as_float(ww[e] << 16)) * kLog2e;
            s[c * 8 + 2 * e + 1] =
                (s[c * 8 + 2 * e + 1] + __uint_as_float(ww[e] & 0xFFFF0000u)) * kLog2e;
          }
        }
      } else if (brow != nullptr) {
#pragma unroll
        for (int j = 0; j < 128; ++j) {
          float bj = 0.f;
          if (key0 + j < args.nk) {
            bj = (BMODE == kBiasGlobalF32)
                     ? reinterpret_cast<const float*>(brow)[key0 + j]
                     : __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(brow)[key0 + j]);
          }
          s[j] = (s[j] + bj) * kLog2e;
        }
      } else {
#pragma unroll
        for (int j = 0; j < 128; ++j) s[j] *= kLog2e;
      }
      // key mask: masked -> -1e9 (scaled), past the end -> -inf
      if (!sFlag[t]) {
        constexpr float kMasked = -1e9f * kLog2e;
#pragma unroll
        for (int j = 0; j < 128; ++j) {
          const int kk = key0 + j;
          if (kk >= args.nk) {
            s[j] = -INFINITY;
          } else if (!sMask[kk]) {
            s[j] = kMasked;
          }
        }
      }
      float mt = s[0];
#pragma unroll
      for (int j = 1; j < 128; ++j) mt = fmaxf(mt, s[j]);
      const float m_new = fmaxf(m_run, mt);  // log2 domain
      const float alpha = ex2_approx(m_run - m_new);
      float rs = 0.f;
#pragma unroll
      for (int j = 0; j < 128; ++j) {
        s[j] = ex2_approx(s[j] - m_new);
        rs += s[j];
      }
      l_run = l_run * alpha + rs;
      m_run = m_new;

      // P (bf16) into the swizzled SMEM tile of this parity.  The PV MMA that
      // last read this buffer (tile t-2) completed before O_{t-2} was consumed.
      uint8_t* pbuf = sP + (t & 1) * L::kPBytes + row * 128;
#pragma unroll
      for (int c = 0; c < 16; ++c) {
        uint4 w;
        w.x = pack_bf16x2(s[c * 8 + 0], s[c * 8 + 1]);
        w.y = pack_bf16x2(s[c * 8 + 2], s[c * 8 + 3]);
        w.z = pack_bf16x2(s[c * 8 + 4], s[c * 8 + 5]);
        w.w = pack_bf16x2(s[c * 8 + 6], s[c * 8 + 7]);
        const int phys = (c & 7) ^ (row & 7);
        *reinterpret_cast<uint4*>(pbuf + (c >> 3) * 16384 + phys * 16) = w;
      }
      fence_async_smem();
      mbar_arrive(&p_full[t & 1]);

      if (t >= 1) {
        const int u = t - 1;
        if (!mbar_wait(&o_full[u & 1], (u >> 1) & 1, kErrWaitSoftmax, abort_flag)) {
          ok = false;
          break;
        }
        tc_fence_after();
        float ot[DP];
#pragma unroll
        for (int c = 0; c < DP / 32; ++c) tmem_ld32_to(t_row + 256 + (u & 1) * DP + c * 32, ot + c * 32);
        tmem_wait_ld();
        tc_fence_before();
        mbar_arrive(&o_free[u & 1]);
        const float beta = ex2_approx(m_acc - m_prev);
#pragma unroll
        for (int i = 0; i < DP; ++i) o_acc[i] = o_acc[i] * beta + ot[i];
        m_acc = m_prev;
      }
      m_prev = m_new;
    }

    if (ok && n_tiles > 0) {
      const int u = n_tiles - 1;
      if (mbar_wait(&o_full[u & 1], (u >> 1) & 1, kErrWaitSoftmax, abort_flag)) {
        tc_fence_after();
        float ot[DP];
#pragma unroll
        for (int c = 0; c < DP / 32; ++c) tmem_ld32_to(t_row + 256 + (u & 1) * DP + c * 32, ot + c * 32);
        tmem_wait_ld();
        const float beta = ex2_approx(m_acc - m_prev);
#pragma unroll
        for (int i = 0; i < DP; ++i) o_acc[i] = o_acc[i] * beta + ot[i];
        if (q_ok) {
          const float inv_l = 1.f / l_run;
          __nv_bfloat16* orow = args.out + b * args.out_sb + h * args.out_sh +
                                static_cast<int64_t>(q) * args.out_sq;
          const __nv_bfloat16* grow =
              args.gate == nullptr ? nullptr
                                   : args.gate + b * args.gate_sb + h * args.gate_sh +
                                         static_cast<int64_t>(q) * args.gate_sq;
#pragma unroll
          for (int i = 0; i < DP; ++i) {
            if (i < args.d) {
              float o = bf16r(o_acc[i] * inv_l);
              if (grow != nullptr) o = o * __bfloat162float(grow[i]);
              orow[i] = __float2bfloat16_rn(o);
            }
          }
        }
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

}  // namespace xfb
