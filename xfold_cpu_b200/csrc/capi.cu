// extern "C" entry points of libxfold_b200.so (declared in include/xfold_b200.h).
//
// Single translation unit: it includes every kernel header so the device
// error word and all template instantiations live in one module.
#include <cudaTypedefs.h>

#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <atomic>
#include <mutex>
#include <string>
#include <type_traits>

#include "../../include/xfold_b200.h"
#include "attention.cuh"
#include "tri_attention.cuh"
#include "transition.cuh"
#include "exchange.cuh"
#include "common.cuh"
#include "gemm.cuh"
#include "layer_norm.cuh"
#include "window_attention.cuh"
#include "msa.cuh"
#include "fp32.cuh"
#include "checkpoint.cuh"

#ifndef XFB_NVCC_FLAGS
#define XFB_NVCC_FLAGS "unknown"
#endif

namespace {

using bf16 = __nv_bfloat16;

thread_local std::string g_last_error;

int fail(int code, const std::string& msg) {
  g_last_error = msg;
  return code;
}

#define XFB_REQUIRE(cond, msg)                                        \
  do {                                                                \
    if (!(cond)) return fail(XFB_ERR_INVALID, std::string(msg));      \
  } while (0)

#define XFB_CUDA(call)                                                                     \
  do {                                                                                     \
    cudaError_t e_ = (call);                                                               \
    if (e_ != cudaSuccess)                                                                 \
      return fail(XFB_ERR_CUDA, std::string(#call) + ": " + cudaGetErrorString(e_));       \
  } while (0)

#define XFB_TRY(expr)           \
  do {                          \
    int rc_ = (expr);           \
    if (rc_ != XFB_OK) return rc_; \
  } while (0)

#define XFB_LAUNCHED()                                                                 \
  do {                                                                                 \
    g_launches.fetch_add(1, std::memory_order_relaxed);                                \
    cudaError_t e_ = cudaGetLastError();                                               \
    if (e_ != cudaSuccess)                                                             \
      return fail(XFB_ERR_CUDA, std::string("kernel launch: ") + cudaGetErrorString(e_)); \
  } while (0)

// Number of kernels this library has launched (all devices, all threads).
std::atomic<unsigned long long> g_launches{0};

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }
int64_t round_up(int64_t x, int64_t m) { return (x + m - 1) / m * m; }
int64_t pad_pitch(int64_t n) { return round_up(n, 8); }

// ------------------------------------------------------------------ device info

constexpr int kMaxDevices = 64;
int g_sm_count[kMaxDevices];
std::once_flag g_dev_once[kMaxDevices];

int current_device(int* dev) {
  XFB_CUDA(cudaGetDevice(dev));
  if (*dev < 0 || *dev >= kMaxDevices) return fail(XFB_ERR_INVALID, "device index out of range");
  return XFB_OK;
}

int sm_count(int* out) {
  int dev;
  XFB_TRY(current_device(&dev));
  std::call_once(g_dev_once[dev], [dev]() {
    int v = 0;
    cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev);
    g_sm_count[dev] = v;
  });
  *out = g_sm_count[dev] > 0 ? g_sm_count[dev] : 148;
  return XFB_OK;
}

// ------------------------------------------------------------------ tensor maps

PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;
std::once_flag g_encode_once;

int get_encoder() {
  std::call_once(g_encode_once, []() {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess) {
      g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
    }
  });
  if (g_encode == nullptr) return fail(XFB_ERR_CUDA, "cuTensorMapEncodeTiled is unavailable");
  return XFB_OK;
}

// N-D tensor map (rank 2..5) over bf16 or f32 data.  dims[0] is contiguous;
// strides[i] is the byte stride of dims[i+1].  Size-1 trailing dimensions
// get a consistent stride.  The base must be 16-byte aligned and every stride
// a multiple of 16 bytes (the TMA rules).
int make_map_nd(CUtensorMap* map, bool f32, int rank, const void* base, const uint64_t* dims,
                const uint64_t* strides, const uint32_t* box, CUtensorMapSwizzle swz) {
  XFB_TRY(get_encoder());
  if (!aligned16(base)) return fail(XFB_ERR_INVALID, "TMA operand base is not 16-byte aligned");
  cuuint64_t d[5], s[4];
  cuuint32_t bx[5], estr[5];
  for (int i = 0; i < rank; ++i) {
    d[i] = dims[i];
    bx[i] = box[i];
    estr[i] = 1;
  }
  for (int i = 0; i + 1 < rank; ++i) {
    uint64_t st = strides[i];
    if (dims[i + 1] == 1 && i > 0) st = std::max<uint64_t>(st, s[i - 1] * dims[i]);
    st = static_cast<uint64_t>(round_up(static_cast<int64_t>(st), 16));
    if (strides[i] % 16 != 0 && dims[i + 1] != 1)
      return fail(XFB_ERR_INVALID, "TMA operand stride is not a multiple of 16 bytes");
    s[i] = st;
  }
  CUresult r = g_encode(map, f32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16,
                        rank, const_cast<void*>(base), d, s, bx, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, swz, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                        CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    char buf[256];
    snprintf(buf, sizeof(buf), "cuTensorMapEncodeTiled failed (%d): rank %d dims %llu %llu %llu box %u %u",
             static_cast<int>(r), rank, (unsigned long long)dims[0],
             (unsigned long long)(rank > 1 ? dims[1] : 0), (unsigned long long)(rank > 2 ? dims[2] : 0),
             box[0], rank > 1 ? box[1] : 0);
    return fail(XFB_ERR_CUDA, buf);
  }
  return XFB_OK;
}

// 3-D bf16 tensor map: element (x, y, z) at base + x*2 + y*stride1 + z*stride2.
int make_map(CUtensorMap* map, const void* base, uint64_t dx, uint64_t dy, uint64_t dz,
             uint64_t stride1, uint64_t stride2, uint32_t bx, uint32_t by,
             CUtensorMapSwizzle swz) {
  if (dz == 1) stride2 = std::max<uint64_t>(stride2, stride1 * dy);
  const uint64_t dims[3] = {dx, dy, dz};
  const uint64_t strides[2] = {stride1, stride2};
  const uint32_t box[3] = {bx, by, 1};
  return make_map_nd(map, false, 3, base, dims, strides, box, swz);
}

// Row-major [batch][rows][ld] output map with a box of 128 rows and one
// 128-byte swizzle atom of columns (32 f32 or 64 bf16).
int make_out_map(CUtensorMap* map, const void* base, bool f32, int64_t cols, int64_t rows,
                 int64_t batch, int64_t ld, int64_t bstride) {
  const int64_t es = f32 ? 4 : 2;
  const uint64_t dims[3] = {static_cast<uint64_t>(cols), static_cast<uint64_t>(rows),
                            static_cast<uint64_t>(batch)};
  const uint64_t strides[2] = {static_cast<uint64_t>(ld * es),
                               static_cast<uint64_t>((batch > 1 ? bstride : ld * rows) * es)};
  const uint32_t box[3] = {f32 ? 32u : 64u, 128u, 1u};
  return make_map_nd(map, f32, 3, base, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B);
}

template <class Kernel>
int set_smem(Kernel kernel, int bytes) {
  XFB_CUDA(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes));
  return XFB_OK;
}

// ------------------------------------------------------------------ GEMM launcher

// Deepest operand pipeline that fits next to the epilogue's buffers.
template <int BN, class Epi>
constexpr int gemm_stages() {
  constexpr int stage = (128 + BN) * 64 * 2;
  constexpr int aux = ((Epi::kAuxBytes + 1023) / 1024) * 1024 * 2;
  constexpr int staging = ((Epi::kStagingBytes + 1023) / 1024) * 1024 * Epi::kStagingBufs;
  constexpr int budget = 200 * 1024 - aux - staging;
  // Epilogues with large buffers (an f32 output plus an aux ring) would keep
  // only two operand stages, i.e. no prefetch of the next tile when K = 128:
  // those take a third stage out of the last 24 KB of shared memory.
  constexpr int wide = 224 * 1024 - aux - staging;
  if (budget / stage <= 2 && wide / stage >= 3) return 3;
  return budget / stage > 6 ? 6 : budget / stage;
}

// A: K-major -> element (m, k) at A[bat*a_bs + m*lda + k]; MN-major -> A[bat*a_bs + k*lda + m].
// B: K-major -> element (n, k) at B[bb*b_bs + n*ldb + k]; MN-major -> B[bb*b_bs + k*ldb + n],
// with bb = 0 when b_shared (one weight for every batch index) else bb = bat.
template <int BN, bool A_MN, bool B_MN, class Epi>
int run_gemm(const void* A, int64_t lda, int64_t a_bs, const void* B, int64_t ldb, int64_t b_bs,
             int64_t M, int64_t N, int64_t K, int64_t batch, const Epi& epi, cudaStream_t st,
             bool b_shared = false) {
  constexpr int STAGES = gemm_stages<BN, Epi>();
  static_assert(STAGES >= 2, "epilogue buffers leave no room for the operand pipeline");
  if (M <= 0 || N <= 0 || batch <= 0) return XFB_OK;
  if (K <= 0) return fail(XFB_ERR_INVALID, "GEMM with empty reduction dimension");
  if (M > (1ll << 31) - 256 || N > (1 << 30)) return fail(XFB_ERR_INVALID, "GEMM too large");
  const int64_t b_batch = b_shared ? 1 : batch;
  CUtensorMap ta, tb;
  if (A_MN) {
    XFB_TRY(make_map(&ta, A, M, K, batch, lda * 2, a_bs * 2, 64, 64, CU_TENSOR_MAP_SWIZZLE_128B));
  } else {
    XFB_TRY(make_map(&ta, A, K, M, batch, lda * 2, a_bs * 2, 64, 128, CU_TENSOR_MAP_SWIZZLE_128B));
  }
  if (B_MN) {
    XFB_TRY(make_map(&tb, B, N, K, b_batch, ldb * 2, b_bs * 2, 64, 64, CU_TENSOR_MAP_SWIZZLE_128B));
  } else {
    XFB_TRY(make_map(&tb, B, K, N, b_batch, ldb * 2, b_bs * 2, 64, BN, CU_TENSOR_MAP_SWIZZLE_128B));
  }
  xfb::GemmShape sh;
  sh.M = static_cast<int>(M);
  sh.N = static_cast<int>(N);
  sh.K = static_cast<int>(K);
  sh.batch = static_cast<int>(batch);
  sh.m_tiles = static_cast<int>((M + 127) / 128);
  sh.n_tiles = static_cast<int>((N + BN - 1) / BN);
  sh.k_blocks = static_cast<int>((K + 63) / 64);
  sh.b_shared = b_shared ? 1 : 0;
  const int64_t total = static_cast<int64_t>(sh.m_tiles) * sh.n_tiles * sh.batch;
  if (total > (1ll << 31) - 1) return fail(XFB_ERR_INVALID, "GEMM has too many tiles");
  int sms;
  XFB_TRY(sm_count(&sms));
  const int grid = static_cast<int>(std::min<int64_t>(total, sms));
  using L = xfb::GemmSmem<BN, STAGES, Epi>;
  auto kernel = xfb::gemm_bf16_kernel<BN, STAGES, A_MN, B_MN, Epi>;
  XFB_TRY(set_smem(kernel, L::kLaunchBytes));
  kernel<<<grid, xfb::GemmWarps<Epi>::kThreads, L::kLaunchBytes, st>>>(ta, tb, sh, epi);
  XFB_LAUNCHED();
  return XFB_OK;
}

template <class EPI>
int linear_tma(const bf16* x, int64_t m, int64_t k, int64_t ldx, const bf16* w, int64_t n,
               const float* bias, const bf16* gate, void* out, int accumulate, cudaStream_t st) {
  constexpr bool kF32 = EPI::kColsPerBox == 32;
  EPI epi;
  XFB_TRY(make_out_map(&epi.out_map, out, kF32, n, m, 1, n, 0));
  epi.bias = bias;
  epi.accumulate = accumulate;
  if constexpr (EPI::kAuxBytes > 0) {
    const uint64_t dims[3] = {static_cast<uint64_t>(n), static_cast<uint64_t>(m), 1};
    const uint64_t strides[2] = {static_cast<uint64_t>(n * 2), static_cast<uint64_t>(n * m * 2)};
    const uint32_t box[3] = {64, 128, 1};
    XFB_TRY(make_map_nd(&epi.gate_map, false, 3, gate, dims, strides, box,
                        CU_TENSOR_MAP_SWIZZLE_128B));
  }
  return run_gemm<128, false, false>(x, ldx, 0, w, k, 0, m, n, k, 1, epi, st);
}

// y[m][n] (=|+=) bf16(x[m][k] w[n][k]^T + bias) [* gate], BN = 128, output via
// TMA store / reduce-add (f32 or bf16 y with row stride n).  Needs n % 8 == 0
// and 16-byte aligned pointers; anything else takes the direct-store epilogue.
int linear_core(const bf16* x, int64_t m, int64_t k, int64_t ldx, const bf16* w, int64_t n,
                const float* bias, const bf16* gate, int64_t ld_gate, void* out, int out_f32,
                int accumulate, int64_t ld_out, cudaStream_t st) {
  const bool tma_ok = n % 8 == 0 && ld_out == n && aligned16(out) &&
                      (gate == nullptr || (ld_gate == n && aligned16(gate)));
  if (!tma_ok) {
    xfb::EpiDirect<128> epi;
    epi.out = out;
    epi.ld_out = ld_out;
    epi.bstride_out = 0;
    epi.out_f32 = out_f32;
    epi.accumulate = accumulate;
    epi.bias = bias;
    epi.gate = gate;
    epi.ld_gate = ld_gate;
    epi.M = static_cast<int>(m);
    epi.N = static_cast<int>(n);
    return run_gemm<128, false, false>(x, ldx, 0, w, k, 0, m, n, k, 1, epi, st);
  }
  if (gate != nullptr) {
    return out_f32 ? linear_tma<xfb::EpiOutGated<128, true>>(x, m, k, ldx, w, n, bias, gate, out,
                                                             accumulate, st)
                   : linear_tma<xfb::EpiOutGated<128, false>>(x, m, k, ldx, w, n, bias, gate, out,
                                                              accumulate, st);
  }
  return out_f32 ? linear_tma<xfb::EpiOut<128, true>>(x, m, k, ldx, w, n, bias, gate, out,
                                                      accumulate, st)
                 : linear_tma<xfb::EpiOut<128, false>>(x, m, k, ldx, w, n, bias, gate, out,
                                                       accumulate, st);
}

// ------------------------------------------------------------------ routed exchanges

// Destinations of a routed exchange as the C ABI passes them: dst[s] = rank s's
// receive buffer as mapped in this process (dst[rank] is this GPU's own).
struct Route {
  void* const* dst;
  int world, rank;
};

int check_route(void* const* dst, int world, int rank) {
  XFB_REQUIRE(world >= 1 && world <= xfb::kMaxRoute, "routed exchanges take 1..16 ranks");
  XFB_REQUIRE(rank >= 0 && rank < world, "rank out of range");
  XFB_REQUIRE(dst != nullptr, "routed destinations missing");
  for (int s = 0; s < world; ++s)
    XFB_REQUIRE(dst[s] != nullptr && aligned16(dst[s]),
                "routed destinations must be non-null and 16-byte aligned");
  return XFB_OK;
}

// ------------------------------------------------------------------ LayerNorm launcher

int run_layer_norm(const void* x, int x_dtype, int64_t rows, int64_t c, int64_t ldx,
                   const float* w, const float* b, double eps, bf16* y, int64_t ldy,
                   const bf16* mod_scale, const bf16* mod_shift, const bf16* wh, int heads,
                   bf16* head_out, int64_t head_ld, cudaStream_t st, float head_scale = 1.f,
                   const int64_t* gather_idx = nullptr, const uint8_t* gather_valid = nullptr,
                   int64_t src_rows = 0, int64_t perm_outer = 0, int64_t perm_inner = 0,
                   const Route* y_route = nullptr, int64_t route_n = 0) {
  if (rows <= 0) return XFB_OK;
  XFB_REQUIRE(x_dtype == XFB_F32 || x_dtype == XFB_BF16, "LayerNorm input must be f32 or bf16");
  XFB_REQUIRE(heads >= 0 && heads <= 16, "head projection supports at most 16 heads");
  XFB_REQUIRE(aligned16(x) && (y == nullptr || aligned16(y)), "LayerNorm buffers must be 16-byte aligned");
  xfb::LnArgs a;
  a.x = x;
  a.rows = rows;
  a.ldx = ldx;
  a.w = w;
  a.b = b;
  a.eps = static_cast<float>(eps);
  a.y = y;
  a.ldy = ldy;
  a.mod_scale = mod_scale;
  a.mod_shift = mod_shift;
  a.wh = heads > 0 ? wh : nullptr;
  a.heads = heads;
  a.head_out = head_out;
  a.head_ld = head_ld;
  a.head_scale = head_scale;
  a.gather_idx = gather_idx;
  a.gather_valid = gather_valid;
  a.src_rows = src_rows;
  a.perm_outer = perm_outer;
  a.perm_inner = perm_inner;
  XFB_REQUIRE(gather_idx == nullptr || heads == 0, "row gather excludes the head projection");
  XFB_REQUIRE(perm_outer == 0 || (heads == 0 && perm_inner > 0 && perm_outer * perm_inner == rows),
              "row permutation must cover the rows and excludes the head projection");
  if (y_route != nullptr) {
    // the row <-> column transpose of a row-sharded pair (ln_heads_tc_kernel only)
    XFB_REQUIRE(c == 128 && heads > 0 && mod_scale == nullptr && mod_shift == nullptr &&
                    ldx % 4 == 0 && ldy % 4 == 0 && y != nullptr,
                "a routed LayerNorm output needs c = 128 with a head projection");
    XFB_REQUIRE(route_n > 0 && route_n % y_route->world == 0 && rows % route_n == 0 &&
                    rows / route_n == route_n / y_route->world,
                "a routed LayerNorm takes n / world pair rows of n columns");
    a.route = 1;
    a.route_rank = y_route->rank;
    a.route_rows = static_cast<int>(route_n / y_route->world);
    a.route_n = static_cast<int>(route_n);
    for (int s = 0; s < 16; ++s)
      a.y_dst[s] = s < y_route->world ? static_cast<bf16*>(y_route->dst[s]) : nullptr;
  }
  int sms;
  XFB_TRY(sm_count(&sms));
  if (c == 128 && heads > 0 && mod_scale == nullptr && mod_shift == nullptr && ldx % 4 == 0 &&
      (y == nullptr || ldy % 4 == 0)) {
    // head projection on the tensor core, 128-row tiles; six CTAs per SM (40
    // registers x 256 threads, 36 KB shared memory and 32 TMEM columns each):
    // 184 -> 158 us for the 4-head bias at N = 1024 against four
    const int blocks = static_cast<int>(std::min<int64_t>((rows + 127) / 128, int64_t(sms) * 6));
    if (a.route) {
      if (x_dtype == XFB_F32) {
        xfb::ln_heads_tc_kernel<float, true><<<blocks, 256, 0, st>>>(a);
      } else {
        xfb::ln_heads_tc_kernel<bf16, true><<<blocks, 256, 0, st>>>(a);
      }
    } else if (x_dtype == XFB_F32) {
      xfb::ln_heads_tc_kernel<float><<<blocks, 256, 0, st>>>(a);
    } else {
      xfb::ln_heads_tc_kernel<bf16><<<blocks, 256, 0, st>>>(a);
    }
    XFB_LAUNCHED();
    return XFB_OK;
  }
  if (c == 64 && heads == 0 && ldx % 8 == 0 && (y == nullptr || ldy % 8 == 0) &&
      aligned16(mod_scale) && aligned16(mod_shift)) {
    // four rows per warp
    const int blocks = static_cast<int>(std::min<int64_t>((rows + 31) / 32, int64_t(sms) * 16));
    if (x_dtype == XFB_F32) {
      xfb::ln_rows64_kernel<float><<<blocks, 256, 0, st>>>(a);
    } else {
      xfb::ln_rows64_kernel<bf16><<<blocks, 256, 0, st>>>(a);
    }
    XFB_LAUNCHED();
    return XFB_OK;
  }
  if (c == 128 && heads == 0 && gather_idx == nullptr && perm_outer == 0 &&
      mod_scale == nullptr && mod_shift == nullptr && y != nullptr && ldx % 4 == 0 &&
      ldy % 4 == 0) {
    // four rows per warp in flight (the pair LayerNorm at N = 1024 measured
    // 154 / 121 / 141 us with 2 / 4 / 8 rows; 8 rows drop occupancy)
    constexpr int kRows = 4;
    const int blocks2 =
        static_cast<int>(std::min<int64_t>((rows + 8 * kRows - 1) / (8 * kRows), int64_t(sms) * 16));
    if (x_dtype == XFB_F32) {
      xfb::ln_rows128_multi_kernel<float, kRows><<<blocks2, 256, 0, st>>>(a);
    } else {
      xfb::ln_rows128_multi_kernel<bf16, kRows><<<blocks2, 256, 0, st>>>(a);
    }
    XFB_LAUNCHED();
    return XFB_OK;
  }
  const int64_t warps = (rows + 0);
  const int blocks = static_cast<int>(std::min<int64_t>((warps + 7) / 8, int64_t(sms) * 16));
  const dim3 block(256);
#define XFB_LN_CASE(C, T, HP)                                        \
  xfb::ln_rows_kernel<C, T, HP><<<blocks, block, 0, st>>>(a);        \
  XFB_LAUNCHED();                                                    \
  return XFB_OK;
#define XFB_LN_HEADS(C, T)                          \
  if (heads == 0) { XFB_LN_CASE(C, T, 0) }          \
  if (heads <= 4) { XFB_LN_CASE(C, T, 4) }          \
  XFB_LN_CASE(C, T, 16)
#define XFB_LN_NOHEADS(C, T) XFB_LN_CASE(C, T, 0)
#define XFB_LN_TYPES_NOHEADS(C)                                          \
  XFB_REQUIRE(heads == 0, "head projection requires C <= 128");          \
  if (x_dtype == XFB_F32) { XFB_LN_NOHEADS(C, float) }                   \
  XFB_LN_NOHEADS(C, bf16)
#define XFB_LN_TYPES(C)                                                  \
  if (x_dtype == XFB_F32) { XFB_LN_HEADS(C, float) }                     \
  XFB_LN_HEADS(C, bf16)
  switch (c) {
    case 64: { XFB_LN_TYPES(64) }
    case 128: { XFB_LN_TYPES(128) }
    case 384: { XFB_LN_TYPES_NOHEADS(384) }
    case 768: { XFB_LN_TYPES_NOHEADS(768) }
    default:
      return fail(XFB_ERR_INVALID, "LayerNorm width must be 64, 128, 384 or 768");
  }
#undef XFB_LN_TYPES
#undef XFB_LN_TYPES_NOHEADS
#undef XFB_LN_NOHEADS
#undef XFB_LN_HEADS
#undef XFB_LN_CASE
}

// ------------------------------------------------------------------ weight packing

// mode 0: triangle (proj/gate interleaved by 64 rows, then gating_linear)
// mode 1: GLU (gate/value interleaved by 64 rows)
// mode 2: concatenation of four [c][c] matrices
// mode 3: one [rows][k] matrix (a plain copy, or the transpose of [k][rows])
// transposed: the sources are the transposed nn.Linear weights [in][out] the
// reference's native extension takes; element (row, col) is read at
// col * out_features + row instead of row * k + col.
__global__ void pack_weights_kernel(const void* s0, const void* s1, const void* s2,
                                    const void* s3, int src_f32, int mode, int64_t c_or_n,
                                    int64_t k, int64_t rows, int transposed, bf16* dst) {
  const int64_t total = rows * k;
  for (int64_t idx = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; idx < total;
       idx += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t r = idx / k;
    const int64_t col = idx - r * k;
    const void* src = nullptr;
    int64_t srow = 0;
    int64_t out_features = 0;  // rows of the source matrix (its width when transposed)
    if (mode == 0) {
      const int64_t c = c_or_n;
      if (r < 4 * c) {
        const int64_t t = r / 128, w = r % 128;
        src = (w < 64) ? s0 : s1;
        srow = 64 * t + (w % 64);
        out_features = 2 * c;
      } else {
        src = s2;
        srow = r - 4 * c;
        out_features = c;
      }
    } else if (mode == 1) {
      const int64_t n = c_or_n;
      const int64_t t = r / 128, w = r % 128;
      src = s0;
      srow = (w < 64) ? 64 * t + w : n + 64 * t + (w - 64);
      out_features = 2 * n;
    } else if (mode == 2) {
      const int64_t c = c_or_n;
      const int64_t which = r / c;
      src = which == 0 ? s0 : which == 1 ? s1 : which == 2 ? s2 : s3;
      srow = r - which * c;
      out_features = c;
    } else {
      src = s0;
      srow = r;
      out_features = rows;
    }
    const int64_t off = transposed ? col * out_features + srow : srow * k + col;
    const float v = src_f32 ? reinterpret_cast<const float*>(src)[off]
                            : __bfloat162float(reinterpret_cast<const bf16*>(src)[off]);
    dst[idx] = __float2bfloat16_rn(v);
  }
}

int launch_pack(const void* s0, const void* s1, const void* s2, const void* s3, int w_dtype,
                int mode, int64_t c_or_n, int64_t k, int64_t rows, void* dst, cudaStream_t st,
                int transposed = 0) {
  XFB_REQUIRE(w_dtype == XFB_F32 || w_dtype == XFB_BF16, "weights must be f32 or bf16");
  const int64_t total = rows * k;
  const int blocks = static_cast<int>(std::min<int64_t>((total + 255) / 256, 4096));
  pack_weights_kernel<<<blocks, 256, 0, st>>>(s0, s1, s2, s3, w_dtype == XFB_F32, mode, c_or_n,
                                              k, rows, transposed, static_cast<bf16*>(dst));
  XFB_LAUNCHED();
  return XFB_OK;
}

// Head-wise repack (and optional scale) of [BH][n][d] into [BH][n][dp] with zero padding.
__global__ void repack_heads_kernel(const bf16* src, int64_t bh_n, int d, int dp, float scale,
                                    int do_scale, bf16* dst) {
  const int64_t total = bh_n * dp;
  for (int64_t idx = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; idx < total;
       idx += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t r = idx / dp;
    const int e = static_cast<int>(idx - r * dp);
    float v = 0.f;
    if (e < d) {
      v = __bfloat162float(src[r * d + e]);
      if (do_scale) v = xfb::bf16r(v * scale);
    }
    dst[idx] = __float2bfloat16_rn(v);
  }
}

// ------------------------------------------------------------------ workspace carving

struct Carver {
  uint8_t* base;
  int64_t used = 0;
  int64_t cap;
  template <typename T>
  T* take(int64_t count) {
    used = round_up(used, 256);
    T* p = reinterpret_cast<T*>(base ? base + used : nullptr);
    used += count * static_cast<int64_t>(sizeof(T));
    return p;
  }
};

int check_workspace(const Carver& cv, const void* ws, int64_t ws_bytes) {
  if (cv.used > ws_bytes) {
    char buf[160];
    snprintf(buf, sizeof(buf), "workspace too small: need %lld bytes, got %lld",
             (long long)cv.used, (long long)ws_bytes);
    return fail(XFB_ERR_INVALID, buf);
  }
  if (cv.used > 0 && (reinterpret_cast<uintptr_t>(ws) & 255) != 0)
    return fail(XFB_ERR_INVALID, "workspace must be 256-byte aligned");
  return XFB_OK;
}

// ------------------------------------------------------------------ triangle output

// W'[n][k] = bf16(gamma[k] W[n][k]), colsum[n] = sum_k W'[n][k] (the rounded
// values the GEMM multiplies), colbias[n] = sum_k beta[k] W[n][k]; one block
// of 128 threads per output channel n.
__global__ void tri_center_fold_kernel(const float* gamma, const float* beta, const bf16* w, int c,
                                       bf16* wf, float* colsum, float* colbias) {
  __shared__ float red[2][4];
  const int n = blockIdx.x;
  float s = 0.f, sb = 0.f;
  for (int k = threadIdx.x; k < c; k += blockDim.x) {
    const float wv = __bfloat162float(w[static_cast<int64_t>(n) * c + k]);
    const bf16 f = __float2bfloat16_rn((gamma ? gamma[k] : 1.f) * wv);
    wf[static_cast<int64_t>(n) * c + k] = f;
    s += __bfloat162float(f);
    sb += (beta ? beta[k] : 0.f) * wv;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    s += __shfl_xor_sync(0xffffffffu, s, o);
    sb += __shfl_xor_sync(0xffffffffu, sb, o);
  }
  if ((threadIdx.x & 31) == 0) {
    red[0][threadIdx.x >> 5] = s;
    red[1][threadIdx.x >> 5] = sb;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    colsum[n] = (red[0][0] + red[0][1]) + (red[0][2] + red[0][3]);
    colbias[n] = (red[1][0] + red[1][1]) + (red[1][2] + red[1][3]);
  }
}

struct TriCenterWs {
  float2* stats;   // [count]
  bf16* wf;        // [c][c]
  float* colsum;   // [c]
  float* colbias;  // [c]
};

void tri_center_layout(Carver& cv, int64_t count, int64_t c, TriCenterWs* w) {
  w->stats = cv.take<float2>(count);
  w->wf = cv.take<bf16>(c * c);
  w->colsum = cv.take<float>(c);
  w->colbias = cv.take<float>(c);
}

template <class EPI>
int tri_center_gemm(const bf16* z, int64_t count, int64_t c, const bf16* g, void* out,
                    int accumulate, const TriCenterWs& w, cudaStream_t st) {
  constexpr bool kF32 = EPI::kColsPerBox == 32;
  EPI epi;
  XFB_TRY(make_out_map(&epi.out_map, out, kF32, c, count, 1, c, 0));
  epi.bias = nullptr;
  epi.accumulate = accumulate;
  const uint64_t dims[3] = {static_cast<uint64_t>(c), static_cast<uint64_t>(count), 1};
  const uint64_t strides[2] = {static_cast<uint64_t>(c * 2), static_cast<uint64_t>(count * c * 2)};
  const uint32_t box[3] = {64, 128, 1};
  XFB_TRY(make_map_nd(&epi.gate_map, false, 3, g, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B));
  epi.stats = w.stats;
  epi.colsum = w.colsum;
  epi.colbias = w.colbias;
  epi.rows = static_cast<int>(count);
  // A = z read MN-major: element (position p, channel k) at z[k * count + p]
  return run_gemm<128, true, false>(z, count, 0, w.wf, c, 0, count, c, c, 1, epi, st);
}

// Centre LayerNorm + output projection + output gate of a triangle
// multiplication, for a channel-major contraction result with contiguous
// positions, z[k * count + p]:  out (=|+=) bf16(bf16(LN_c(z) W^T) * g).  The
// LayerNorm is folded into the GEMM (EpiOutLnGated): one read-only statistics
// pass over z, and the GEMM reads z itself instead of a normalised copy.
int tri_center_output(const bf16* z, int64_t count, int64_t c, const bf16* g, const float* gamma,
                      const float* beta, double eps, const bf16* w, void* out, bool out_f32,
                      int accumulate, const TriCenterWs& ws, cudaStream_t st) {
  XFB_REQUIRE(count % 8 == 0 && aligned16(z) && aligned16(g) && aligned16(out),
              "folded centre LayerNorm needs 16-byte aligned buffers and count % 8 == 0");
  int sms;
  XFB_TRY(sm_count(&sms));
  const int blocks =
      static_cast<int>(std::min<int64_t>((count / 2 + 255) / 256, int64_t(sms) * 8));
  if (c == 128) {
    xfb::ln_stats_channel_major_kernel<128><<<blocks, 256, 0, st>>>(
        z, count, count, static_cast<float>(eps), ws.stats);
  } else {
    xfb::ln_stats_channel_major_kernel<64><<<blocks, 256, 0, st>>>(
        z, count, count, static_cast<float>(eps), ws.stats);
  }
  XFB_LAUNCHED();
  tri_center_fold_kernel<<<static_cast<int>(c), 128, 0, st>>>(gamma, beta, w, static_cast<int>(c),
                                                              ws.wf, ws.colsum, ws.colbias);
  XFB_LAUNCHED();
  return out_f32 ? tri_center_gemm<xfb::EpiOutLnGated<128, true>>(z, count, c, g, out, accumulate,
                                                                  ws, st)
                 : tri_center_gemm<xfb::EpiOutLnGated<128, false>>(z, count, c, g, out,
                                                                   accumulate, ws, st);
}

// ------------------------------------------------------------------ attention launcher

template <int DP, int BMODE, bool PRE>
int launch_flash(const bf16* q, const bf16* k, const bf16* v, xfb::AttnArgs args,
                 cudaStream_t st) {
  CUtensorMap tq, tk, tv, tb;
  const CUtensorMapSwizzle swz = DP == 32 ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_128B;
  const int64_t bh = static_cast<int64_t>(args.B) * args.H;
  XFB_TRY(make_map(&tq, q, DP, args.nq, bh, DP * 2, int64_t(args.nq) * DP * 2, DP, 128, swz));
  XFB_TRY(make_map(&tk, k, DP, args.nk, bh, DP * 2, int64_t(args.nk) * DP * 2, DP,
                   xfb::kAttnBK, swz));
  XFB_TRY(make_map(&tv, v, DP, args.nk, bh, DP * 2, int64_t(args.nk) * DP * 2, DP,
                   xfb::kAttnBK, swz));
  if (BMODE == xfb::kBiasTma) {
    const int64_t z = args.bias_batched ? bh : args.H;
    XFB_TRY(make_map(&tb, args.bias, args.nk, args.nq, z, args.bias_sq * 2, args.bias_sh * 2,
                     xfb::kAttnBK, 128, CU_TENSOR_MAP_SWIZZLE_128B));
  } else {
    memset(&tb, 0, sizeof(tb));
  }
  args.q_tiles = (args.nq + 127) / 128;
  using L = xfb::AttnSmem<DP>;
  auto kernel = xfb::flash_attn_kernel<DP, BMODE, PRE>;
  XFB_TRY(set_smem(kernel, L::kLaunchBytes));
  int sms;
  XFB_TRY(sm_count(&sms));
  const int64_t items = bh * args.q_tiles;
  const int grid = static_cast<int>(std::min<int64_t>(items, int64_t(sms) * L::kCtasPerSm));
  kernel<<<grid, xfb::kAttnThreads, L::kLaunchBytes, st>>>(tq, tk, tv, tb, args);
  XFB_LAUNCHED();
  return XFB_OK;
}

// Three-query-tile triangle attention (tri_attention.cuh): head dim <= 32, one
// TMA-streamed bias shared by all batch rows.
// Triangle-attention kernel shape: XFB_TRI_CFG 0 = three slots of 64-key
// tiles, 1 = four slots of 32-key tiles (tri_attention.cuh: TriCfg).  Measured
// at N = 1024: 1.83 ms and 2.34 ms per launch -- per-tile costs (barrier
// handoffs, MMA issue, TMEM round trips) outweigh the fourth softmax warp per
// sub-partition.
#ifndef XFB_TRI_CFG
#define XFB_TRI_CFG 0
#endif
using TriShape = std::conditional_t<XFB_TRI_CFG == 0, xfb::TriCfg<3, 64>, xfb::TriCfg<4, 32>>;

template <bool PRE>
int launch_flash_tri(const bf16* q, const bf16* k, const bf16* v, xfb::AttnArgs args,
                     cudaStream_t st) {
  using C = TriShape;
  using L = xfb::TriSmem<C>;
  CUtensorMap tq, tk, tv, tb;
  const CUtensorMapSwizzle swz = CU_TENSOR_MAP_SWIZZLE_64B;
  const int64_t bh = static_cast<int64_t>(args.B) * args.H;
  XFB_TRY(make_map(&tq, q, 32, args.nq, bh, 64, int64_t(args.nq) * 64, 32, 128, swz));
  XFB_TRY(make_map(&tk, k, 32, args.nk, bh, 64, int64_t(args.nk) * 64, 32, C::kBK, swz));
  XFB_TRY(make_map(&tv, v, 32, args.nk, bh, 64, int64_t(args.nk) * 64, 32, C::kBK, swz));
  XFB_TRY(make_map(&tb, args.bias, args.nk, args.nq, args.H, args.bias_sq * 2, args.bias_sh * 2,
                   C::kBK, 128,
                   C::kBK == 64 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B));
  args.q_tiles = (args.nq + 127) / 128;
  auto kernel = xfb::flash_tri_kernel<PRE, C>;
  XFB_TRY(set_smem(kernel, L::kLaunchBytes));
  int sms;
  XFB_TRY(sm_count(&sms));
  const int64_t groups = static_cast<int64_t>((args.B + C::kSlots - 1) / C::kSlots) * args.H *
                         args.q_tiles;
  const int grid = static_cast<int>(std::min<int64_t>(groups, sms));
  kernel<<<grid, C::kThreads, L::kLaunchBytes, st>>>(tq, tk, tv, tb, args);
  XFB_LAUNCHED();
  return XFB_OK;
}

// The three-slot kernel pays off once there are enough batch rows to fill the
// slots; XFB_FLASH_TRI=0 selects the one-tile kernel for every shape.
bool use_flash_tri(const xfb::AttnArgs& args) {
  static const bool enabled = [] {
    const char* e = std::getenv("XFB_FLASH_TRI");
    return e == nullptr || std::strcmp(e, "0") != 0;
  }();
  return enabled && args.bias != nullptr && !args.bias_batched && args.B >= 48;
}

// Picks the bias path: TMA-streamed bf16 tiles when the layout allows it
// (row stride nk with nk % 8 == 0, contiguous heads, 16-byte aligned), else
// per-thread global loads.  `pre`: q and the bias already carry log2(e)
// (only the TMA bias path takes pre-scaled inputs).
//
// `exact_bias`: the bias is the caller's (any values, -inf and NaN included) and
// is added in f32 by the softmax warps.  The TMA path lets the bias enter the
// accumulator through MMAs against an identity tile, where a non-finite bias
// value times the identity's zeros would turn its 15 neighbouring scores into
// NaN; it is used for biases this library computes (finite projections).
int run_flash(int dp, int bias_dtype, bool pre, const bf16* q, const bf16* k, const bf16* v,
              const xfb::AttnArgs& args, cudaStream_t st, bool exact_bias = false) {
  XFB_REQUIRE(static_cast<int64_t>(args.B) * args.H * ((args.nq + 127) / 128) < (1ll << 31),
              "attention has too many work items");
  int mode = xfb::kBiasGlobalBf16;
  if (args.bias != nullptr) {
    if (bias_dtype == XFB_F32) {
      mode = xfb::kBiasGlobalF32;
    } else if (!exact_bias && args.bias_sq == args.nk && args.nk % 8 == 0 && aligned16(args.bias) &&
               (args.bias_sh * 2) % 16 == 0 &&
               (!args.bias_batched || args.bias_sb == args.H * args.bias_sh)) {
      mode = xfb::kBiasTma;
    }
  }
  if (pre) {
    XFB_REQUIRE(mode == xfb::kBiasTma && dp == 32, "pre-scaled attention needs the TMA bias path");
    if (use_flash_tri(args)) return launch_flash_tri<true>(q, k, v, args, st);
    return launch_flash<32, xfb::kBiasTma, true>(q, k, v, args, st);
  }
  if (dp == 32) {
    if (mode == xfb::kBiasTma && use_flash_tri(args))
      return launch_flash_tri<false>(q, k, v, args, st);
    if (mode == xfb::kBiasTma) return launch_flash<32, xfb::kBiasTma, false>(q, k, v, args, st);
    if (mode == xfb::kBiasGlobalF32)
      return launch_flash<32, xfb::kBiasGlobalF32, false>(q, k, v, args, st);
    return launch_flash<32, xfb::kBiasGlobalBf16, false>(q, k, v, args, st);
  }
  if (mode == xfb::kBiasTma) return launch_flash<64, xfb::kBiasTma, false>(q, k, v, args, st);
  if (mode == xfb::kBiasGlobalF32)
    return launch_flash<64, xfb::kBiasGlobalF32, false>(q, k, v, args, st);
  return launch_flash<64, xfb::kBiasGlobalBf16, false>(q, k, v, args, st);
}

// Key mask -> bits, one 32-bit word per 32 keys per row.
int launch_mask_bits(const void* mask, bool is_float, int64_t rows, int64_t nk, int64_t stride,
                     uint32_t* out, cudaStream_t st) {
  const int words = static_cast<int>((nk + 31) / 32);
  const int64_t total = rows * words;
  const int blocks = static_cast<int>(std::min<int64_t>((total + 255) / 256, 4096));
  xfb::pack_mask_bits_kernel<<<blocks, 256, 0, st>>>(mask, is_float ? 1 : 0, rows,
                                                     static_cast<int>(nk), stride, out, words);
  XFB_LAUNCHED();
  return XFB_OK;
}

int64_t mask_words(int64_t nk) { return (nk + 31) / 32; }

int head_pitch(int64_t d) { return d <= 32 ? 32 : 64; }

}  // namespace

// ====================================================================== C ABI

extern "C" {

XFB_API const char* xfb_last_error(void) { return g_last_error.c_str(); }

XFB_API uint64_t xfb_launch_count(void) { return g_launches.load(std::memory_order_relaxed); }

XFB_API int xfb_runtime_info(char* buf, int64_t buf_len) {
  int dev = -1, sms = 0, major = 0, minor = 0, rt = 0, drv = 0;
  cudaGetDevice(&dev);
  if (dev >= 0) {
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
    cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev);
  }
  cudaRuntimeGetVersion(&rt);
  cudaDriverGetVersion(&drv);
  cudaGetLastError();
  char tmp[1024];
  snprintf(tmp, sizeof(tmp),
           "{\"library\": \"xfold_b200\", \"target\": \"sm_100a\", \"device\": %d, "
           "\"compute_capability\": \"%d.%d\", \"sm_count\": %d, \"cuda_runtime\": %d, "
           "\"cuda_driver\": %d, \"nvcc_flags\": \"%s\"}",
           dev, major, minor, sms, rt, drv, XFB_NVCC_FLAGS);
  if (buf == nullptr || buf_len <= 0) return fail(XFB_ERR_INVALID, "buffer required");
  snprintf(buf, static_cast<size_t>(buf_len), "%s", tmp);
  return XFB_OK;
}

XFB_API int xfb_check_device(void) {
  int dev;
  XFB_TRY(current_device(&dev));
  int major = 0, minor = 0;
  XFB_CUDA(cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev));
  XFB_CUDA(cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev));
  if (major != 10 || minor != 0) {
    char buf[128];
    snprintf(buf, sizeof(buf), "device %d has compute capability %d.%d; sm_100 (B200) required",
             dev, major, minor);
    return fail(XFB_ERR_DEVICE, buf);
  }
  cudaFuncAttributes attr;
  XFB_CUDA(cudaFuncGetAttributes(&attr, xfb::flash_attn_kernel<32, xfb::kBiasTma, true>));
  XFB_TRY(get_encoder());
  return XFB_OK;
}

XFB_API int xfb_device_error(int clear, uint32_t* code) {
  unsigned int v = 0;
  XFB_CUDA(cudaMemcpyFromSymbol(&v, xfb_dev_error, sizeof(v)));
  if (code) *code = v;
  if (clear) {
    unsigned int zero = 0;
    XFB_CUDA(cudaMemcpyToSymbol(xfb_dev_error, &zero, sizeof(zero)));
  }
  return XFB_OK;
}

}  // extern "C"

namespace {
__global__ void wait_timeout_selftest_kernel(int64_t timeout_ns) {
  __shared__ uint64_t bar;
  if (threadIdx.x == 0) {
    xfb::mbar_init(&bar, 1);
    xfb::fence_mbar_init();
    const uint32_t addr = xfb::smem_u32(&bar);
    const uint64_t start = xfb::global_ns();
    // Nothing ever arrives on `bar`: the wait must give up on its own.
    while (!xfb::mbar_try_wait(addr, 0)) {
      if (xfb::global_ns() - start > static_cast<uint64_t>(timeout_ns)) {
        xfb::record_error(xfb::kErrWaitTest);
        break;
      }
    }
  }
}
}  // namespace

extern "C" {

XFB_API int xfb_selftest_wait_timeout(int64_t timeout_ns, void* stream) {
  XFB_REQUIRE(timeout_ns > 0 && timeout_ns <= 5000000000ll, "timeout must be in (0, 5 s]");
  wait_timeout_selftest_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(timeout_ns);
  XFB_LAUNCHED();
  return XFB_OK;
}

// ---------------------------------------------------------------- primitives

XFB_API int xfb_layer_norm(const void* x, int x_dtype, int64_t rows, int64_t cols,
                           const float* weight, const float* bias, double eps, void* y,
                           void* stream) {
  XFB_REQUIRE(rows >= 0, "rows must be non-negative");
  XFB_REQUIRE(std::isfinite(eps) && eps >= 0, "LayerNorm eps must be finite and non-negative");
  return run_layer_norm(x, x_dtype, rows, cols, cols, weight, bias, eps, static_cast<bf16*>(y),
                        cols, nullptr, nullptr, nullptr, 0, nullptr, 0,
                        static_cast<cudaStream_t>(stream));
}

XFB_API int xfb_linear(const void* x, int64_t m, int64_t k, const void* weight, int64_t n,
                       const float* bias, void* y, int y_dtype, int accumulate, void* stream) {
  XFB_REQUIRE(m >= 0 && k > 0 && n > 0, "linear expects m >= 0, k > 0, n > 0");
  XFB_REQUIRE(k % 8 == 0 && n % 8 == 0, "linear requires k and n to be multiples of 8");
  XFB_REQUIRE(y_dtype == XFB_F32 || y_dtype == XFB_BF16, "linear output must be f32 or bf16");
  XFB_REQUIRE(!accumulate || y_dtype == XFB_F32, "accumulate requires an f32 output");
  XFB_REQUIRE(aligned16(y), "linear output must be 16-byte aligned");
  return linear_core(static_cast<const bf16*>(x), m, k, k, static_cast<const bf16*>(weight), n,
                     bias, nullptr, 0, y, y_dtype == XFB_F32, accumulate, n,
                     static_cast<cudaStream_t>(stream));
}

XFB_API int64_t xfb_pack_glu_weight_bytes(int64_t n, int64_t k) { return 2 * n * k * 2; }

XFB_API int xfb_pack_glu_weight(const void* weight, int w_dtype, int64_t n, int64_t k,
                                void* packed, void* stream) {
  XFB_REQUIRE(n > 0 && n % 64 == 0, "GLU hidden width must be a positive multiple of 64");
  return launch_pack(weight, nullptr, nullptr, nullptr, w_dtype, 1, n, k, 2 * n, packed,
                     static_cast<cudaStream_t>(stream));
}

XFB_API int64_t xfb_gated_linear_unit_workspace(int64_t m, int64_t k, int64_t n) {
  (void)m;
  Carver cv{nullptr, 0, 0};
  cv.take<bf16>(2 * n * k);
  return cv.used;
}

XFB_API int xfb_gated_linear_unit(const void* x, int64_t m, int64_t k, const void* weight,
                                  int64_t n, int weights_packed, void* y, void* workspace,
                                  int64_t workspace_bytes, void* stream) {
  XFB_REQUIRE(m >= 0 && k > 0, "GLU expects m >= 0 and k > 0");
  XFB_REQUIRE(n > 0 && n % 64 == 0, "GLU hidden width must be a positive multiple of 64");
  XFB_REQUIRE(k % 8 == 0, "GLU input width must be a multiple of 8");
  XFB_REQUIRE(aligned16(y), "GLU output must be 16-byte aligned");
  if (m == 0) return XFB_OK;  // empty input, empty output (no tensor map of zero rows)
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const bf16* w = static_cast<const bf16*>(weight);
  if (!weights_packed) {
    Carver cv{static_cast<uint8_t*>(workspace), 0, workspace_bytes};
    bf16* pk = cv.take<bf16>(2 * n * k);
    XFB_TRY(check_workspace(cv, workspace, workspace_bytes));
    XFB_TRY(launch_pack(weight, nullptr, nullptr, nullptr, XFB_BF16, 1, n, k, 2 * n, pk, st));
    w = pk;
  }
  xfb::EpiGLU epi;
  XFB_TRY(make_out_map(&epi.out_map, y, false, n, m, 1, n, 0));
  return run_gemm<128, false, false>(x, k, 0, w, k, 0, m, 2 * n, k, 1, epi, st);
}

}  // extern "C"

namespace {

// Scratch of xfb_gated_linear_unit_noalloc: the packed weight is written here
// instead of into a caller-provided workspace.  It is part of the module, so
// every device that loads the library holds these 8 MiB until the process exits.
static __device__ __align__(256) bf16 g_glu_noalloc_scratch[XFB_GLU_NOALLOC_MAX_WEIGHT_ELEMS];

bf16* g_glu_noalloc_ptr[kMaxDevices];
std::mutex g_glu_noalloc_mutex;

// Device address of the scratch on the current device.  The host symbol is
// only a stand-in for the device array, so the address is asked for on the
// first call made with that device current and kept once the lookup has
// succeeded.  A failed lookup (for example one made while a stream was being
// captured) is not remembered: the next call asks again.
int glu_noalloc_scratch(bf16** out) {
  int dev;
  XFB_TRY(current_device(&dev));
  std::lock_guard<std::mutex> lock(g_glu_noalloc_mutex);
  if (g_glu_noalloc_ptr[dev] == nullptr) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_glu_noalloc_scratch);
    if (e != cudaSuccess || p == nullptr) {
      if (e != cudaSuccess) cudaGetLastError();  // do not leave the error for the next launch check
      return fail(XFB_ERR_CUDA, std::string("cudaGetSymbolAddress(GLU scratch): ") +
                                    cudaGetErrorString(e));
    }
    g_glu_noalloc_ptr[dev] = static_cast<bf16*>(p);
  }
  *out = g_glu_noalloc_ptr[dev];
  return XFB_OK;
}

}  // namespace

extern "C" {

XFB_API int xfb_gated_linear_unit_noalloc(const void* x, int64_t m, int64_t k, const void* weight,
                                          int64_t n, void* y, void* stream) {
  XFB_REQUIRE(m >= 0 && k > 0, "GLU expects m >= 0 and k > 0");
  XFB_REQUIRE(n > 0 && n % 64 == 0, "GLU hidden width must be a positive multiple of 64");
  XFB_REQUIRE(k % 8 == 0, "GLU input width must be a multiple of 8");
  XFB_REQUIRE(aligned16(x) && aligned16(weight) && aligned16(y),
              "GLU pointers must be 16-byte aligned");
  // Compared by division, so caller values near INT64_MAX cannot wrap 2*n*k
  // into range.
  if (k > XFB_GLU_NOALLOC_MAX_WEIGHT_ELEMS / 2 || n > XFB_GLU_NOALLOC_MAX_WEIGHT_ELEMS / (2 * k)) {
    char buf[240];
    snprintf(buf, sizeof(buf),
             "xfb_gated_linear_unit_noalloc: weight of 2n*k elements (n = %lld, k = %lld) "
             "exceeds the fixed scratch of %lld elements; use xfb_gated_linear_unit with a "
             "workspace",
             (long long)n, (long long)k, (long long)XFB_GLU_NOALLOC_MAX_WEIGHT_ELEMS);
    return fail(XFB_ERR_INVALID, buf);
  }
  if (m == 0) return XFB_OK;  // nothing to write; no tensor map of zero rows
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  bf16* packed = nullptr;
  XFB_TRY(glu_noalloc_scratch(&packed));
  // Every row of the packed weight the GEMM reads is rewritten here, so nothing
  // left from an earlier call is used.
  XFB_TRY(launch_pack(weight, nullptr, nullptr, nullptr, XFB_BF16, 1, n, k, 2 * n, packed, st));
  xfb::EpiGLU epi;
  XFB_TRY(make_out_map(&epi.out_map, y, false, n, m, 1, n, 0));
  return run_gemm<128, false, false>(x, k, 0, packed, k, 0, m, 2 * n, k, 1, epi, st);
}

XFB_API int xfb_gemm(const void* a, const void* b, void* c, int64_t batch, int64_t m, int64_t n,
                     int64_t k, int a_mn_major, int b_mn_major, int c_dtype, void* stream) {
  XFB_REQUIRE(batch >= 0 && m >= 0 && n >= 0 && k > 0, "gemm expects batch, m, n >= 0, k > 0");
  XFB_REQUIRE(c_dtype == XFB_F32 || c_dtype == XFB_BF16, "gemm output must be f32 or bf16");
  XFB_REQUIRE(aligned16(c), "gemm output must be 16-byte aligned");
  const int64_t lda = a_mn_major ? m : k;
  const int64_t ldb = b_mn_major ? n : k;
  XFB_REQUIRE(lda % 8 == 0 && ldb % 8 == 0, "gemm leading dimensions must be multiples of 8");
  XFB_REQUIRE(c_dtype == XFB_F32 ? n % 4 == 0 : n % 8 == 0, "gemm output rows must be 16-byte aligned");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  xfb::EpiDirect<256> epi;
  epi.out = c;
  epi.ld_out = n;
  epi.bstride_out = m * n;
  epi.out_f32 = c_dtype == XFB_F32;
  epi.accumulate = 0;
  epi.bias = nullptr;
  epi.gate = nullptr;
  epi.ld_gate = 0;
  epi.M = static_cast<int>(m);
  epi.N = static_cast<int>(n);
  const int64_t a_bs = m * k, b_bs = n * k;
  if (!a_mn_major && !b_mn_major)
    return run_gemm<256, false, false>(a, lda, a_bs, b, ldb, b_bs, m, n, k, batch, epi, st);
  if (a_mn_major && b_mn_major)
    return run_gemm<256, true, true>(a, lda, a_bs, b, ldb, b_bs, m, n, k, batch, epi, st);
  return fail(XFB_ERR_INVALID, "gemm supports both operands K-major or both MN-major");
}

// ---------------------------------------------------------------- triangle multiplication

XFB_API int64_t xfb_pack_triangle_weights_bytes(int64_t c) { return (5 * c) * c * 2; }

XFB_API int xfb_pack_triangle_weights(const void* projection, const void* gate,
                                      const void* gating_linear, int w_dtype, int64_t c,
                                      void* packed, void* stream) {
  XFB_REQUIRE(c == 64 || c == 128, "triangle multiplication supports c in {64, 128}");
  return launch_pack(projection, gate, gating_linear, nullptr, w_dtype, 0, c, c, 5 * c, packed,
                     static_cast<cudaStream_t>(stream));
}

namespace {
struct TriWs {
  bf16 *x, *a, *b, *g, *z, *packed;
  TriCenterWs center;  // folded centre LayerNorm (n % 8 == 0)
};
void tri_layout(Carver& cv, int64_t n, int64_t c, bool need_pack, TriWs* w) {
  const int64_t pitch = pad_pitch(n);
  w->x = cv.take<bf16>(n * n * c);
  w->a = cv.take<bf16>(c * n * pitch);
  w->b = cv.take<bf16>(c * n * pitch);
  w->z = cv.take<bf16>(c * n * pitch);
  w->g = cv.take<bf16>(n * n * c);
  w->packed = need_pack ? cv.take<bf16>(5 * c * c) : nullptr;
  tri_center_layout(cv, n * n, c, &w->center);
}
}  // namespace

XFB_API int64_t xfb_triangle_multiplication_workspace(int64_t n, int64_t c) {
  Carver cv{nullptr, 0, 0};
  TriWs w;
  tri_layout(cv, n, c, true, &w);
  return cv.used;
}

XFB_API int xfb_triangle_multiplication(
    const void* pair, int pair_dtype, int64_t n, int64_t c, const float* mask, int outgoing,
    const float* left_weight, const float* left_bias, const void* projection, const void* gate,
    const float* center_weight, const float* center_bias, const void* output_weight,
    const void* gating_weight, double left_eps, double center_eps, int weights_packed,
    const void* packed, void* out, int out_dtype, int accumulate, void* workspace,
    int64_t workspace_bytes, void* stream) {
  XFB_REQUIRE(n >= 0, "pair side must be non-negative");
  XFB_REQUIRE(c == 64 || c == 128, "triangle multiplication supports c in {64, 128}");
  XFB_REQUIRE(std::isfinite(left_eps) && left_eps >= 0 && std::isfinite(center_eps) &&
                  center_eps >= 0,
              "LayerNorm eps must be finite and non-negative");
  XFB_REQUIRE(out_dtype == XFB_F32 || out_dtype == XFB_BF16, "output must be f32 or bf16");
  XFB_REQUIRE(!accumulate || out_dtype == XFB_F32, "accumulate requires an f32 output");
  XFB_REQUIRE(output_weight != nullptr, "output_weight is required");
  XFB_REQUIRE(weights_packed ? packed != nullptr
                             : (projection && gate && gating_weight),
              "triangle weights missing");
  if (n == 0) return XFB_OK;
  XFB_REQUIRE(n * n <= (1ll << 31) - 256, "pair too large");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  Carver cv{static_cast<uint8_t*>(workspace), 0, workspace_bytes};
  TriWs w;
  tri_layout(cv, n, c, !weights_packed, &w);
  XFB_TRY(check_workspace(cv, workspace, workspace_bytes));
  const int64_t pitch = pad_pitch(n);
  const int64_t M = n * n;
  const bf16* wcat = static_cast<const bf16*>(packed);
  if (!weights_packed) {
    XFB_TRY(launch_pack(projection, gate, gating_weight, nullptr, XFB_BF16, 0, c, c, 5 * c,
                        w.packed, st));
    wcat = w.packed;
  }
  // 1. x = LN(pair)
  XFB_TRY(run_layer_norm(pair, pair_dtype, M, c, c, left_weight, left_bias, left_eps, w.x, c,
                         nullptr, nullptr, nullptr, 0, nullptr, 0, st));
  // 2. fused projection ‖ gate ‖ output gate -> a, b (channel-major), g; batched
  //    over pair rows i with the packed weight shared, tiles of 128 columns j
  {
    xfb::EpiTriProj epi;
    const uint64_t ab_dims[3] = {static_cast<uint64_t>(n), static_cast<uint64_t>(n),
                                 static_cast<uint64_t>(c)};
    const uint64_t ab_strides[2] = {static_cast<uint64_t>(pitch * 2),
                                    static_cast<uint64_t>(n * pitch * 2)};
    const uint32_t ab_box[3] = {128, 1, 32};
    XFB_TRY(make_map_nd(&epi.a_map, false, 3, w.a, ab_dims, ab_strides, ab_box,
                        CU_TENSOR_MAP_SWIZZLE_NONE));
    XFB_TRY(make_map_nd(&epi.b_map, false, 3, w.b, ab_dims, ab_strides, ab_box,
                        CU_TENSOR_MAP_SWIZZLE_NONE));
    const uint64_t g_dims[3] = {static_cast<uint64_t>(c), static_cast<uint64_t>(n),
                                static_cast<uint64_t>(n)};
    const uint64_t g_strides[2] = {static_cast<uint64_t>(c * 2), static_cast<uint64_t>(n * c * 2)};
    const uint32_t g_box[3] = {64, 128, 1};
    XFB_TRY(make_map_nd(&epi.g_map, false, 3, w.g, g_dims, g_strides, g_box,
                        CU_TENSOR_MAP_SWIZZLE_128B));
    epi.mask = mask;
    epi.n = static_cast<int>(n);
    epi.n_proj_tiles = static_cast<int>(2 * c / 64);
    epi.c = static_cast<int>(c);
    XFB_TRY((run_gemm<128, false, false>(w.x, c, n * c, wcat, c, 0, n, 5 * c, c, n, epi, st,
                                         true)));
  }
  // 3. per-channel contraction z[ch] = a[ch] b[ch]^T (outgoing) or b[ch]^T a[ch] (incoming)
  {
    xfb::EpiDirect<256> epi;
    epi.out = w.z;
    epi.ld_out = pitch;
    epi.bstride_out = n * pitch;
    epi.out_f32 = 0;
    epi.accumulate = 0;
    epi.bias = nullptr;
    epi.gate = nullptr;
    epi.ld_gate = 0;
    epi.M = static_cast<int>(n);
    epi.N = static_cast<int>(n);
    if (outgoing) {
      XFB_TRY((run_gemm<256, false, false>(w.a, pitch, n * pitch, w.b, pitch, n * pitch, n, n, n,
                                           c, epi, st)));
    } else {
      XFB_TRY((run_gemm<256, true, true>(w.b, pitch, n * pitch, w.a, pitch, n * pitch, n, n, n,
                                         c, epi, st)));
    }
  }
  // 4-5. centre LayerNorm folded into the output projection when the positions
  //      of z are contiguous (pitch == n)
  if (pitch == n) {
    return tri_center_output(w.z, M, c, w.g, center_weight, center_bias, center_eps,
                             static_cast<const bf16*>(output_weight), out, out_dtype == XFB_F32,
                             accumulate, w.center, st);
  }
  // 4. centre LayerNorm over channels (channel-major in, row-major out; x is reused)
  {
    int sms;
    XFB_TRY(sm_count(&sms));
    const int blocks = static_cast<int>(std::min<int64_t>((M + 127) / 128, int64_t(sms) * 8));
    if (c == 128) {
      xfb::ln_channel_major_kernel<128><<<blocks, 128, 0, st>>>(
          w.z, static_cast<int>(n), static_cast<int>(n), static_cast<int>(pitch), n * pitch, center_weight,
          center_bias, static_cast<float>(center_eps), w.x);
    } else {
      xfb::ln_channel_major_kernel<64><<<blocks, 128, 0, st>>>(
          w.z, static_cast<int>(n), static_cast<int>(n), static_cast<int>(pitch), n * pitch, center_weight,
          center_bias, static_cast<float>(center_eps), w.x);
    }
    XFB_LAUNCHED();
  }
  // 5. update = (LN_c(z) W_o^T) * g  -> out (or pair += update)
  XFB_REQUIRE(aligned16(out), "output must be 16-byte aligned");
  return linear_core(w.x, M, c, c, static_cast<const bf16*>(output_weight), c, nullptr, w.g, c,
                     out, out_dtype == XFB_F32, accumulate, c, st);
}

// ---------------------------------------------------------------- attention

XFB_API int64_t xfb_dot_product_attention_workspace(int64_t B, int64_t H, int64_t nq, int64_t nk,
                                                    int64_t d) {
  const int64_t dp = head_pitch(d);
  Carver cv{nullptr, 0, 0};
  cv.take<uint32_t>(B * mask_words(nk));
  cv.take<bf16>(B * H * nq * dp);
  cv.take<bf16>(B * H * nk * dp);
  cv.take<bf16>(B * H * nk * dp);
  return cv.used;
}

XFB_API int xfb_dot_product_attention(const void* q, const void* k, const void* v, int64_t B,
                                      int64_t H, int64_t nq, int64_t nk, int64_t d,
                                      const void* mask, int mask_dtype, int mask_batched,
                                      const void* bias, int bias_dtype, int bias_batched,
                                      int q_pre_scaled, void* out, void* workspace,
                                      int64_t workspace_bytes, void* stream) {
  XFB_REQUIRE(B >= 0 && H >= 0 && nq >= 0 && nk >= 0, "attention sizes must be non-negative");
  XFB_REQUIRE(d > 0 && d <= 64, "attention head dimension must be in [1, 64]");
  XFB_REQUIRE(mask == nullptr || mask_dtype == XFB_F32 || mask_dtype == XFB_U8,
              "attention mask must be f32 or uint8/bool");
  XFB_REQUIRE(bias == nullptr || bias_dtype == XFB_F32 || bias_dtype == XFB_BF16,
              "attention bias must be f32 or bf16");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (B == 0 || H == 0 || nq == 0) return XFB_OK;
  if (nk == 0) {
    // Empty key set: the reference returns zeros (dot_product_attention.cpp:263-266).
    XFB_CUDA(cudaMemsetAsync(out, 0, B * H * nq * d * sizeof(bf16), st));
    return XFB_OK;
  }
  const int dp = head_pitch(d);
  const float scale = 1.f / std::sqrt(static_cast<float>(d));
  const bf16* qq = static_cast<const bf16*>(q);
  const bf16* kk = static_cast<const bf16*>(k);
  const bf16* vv = static_cast<const bf16*>(v);
  const bool direct = (d == dp) && q_pre_scaled && aligned16(q) && aligned16(k) && aligned16(v);
  Carver cv{static_cast<uint8_t*>(workspace), 0, workspace_bytes};
  const int64_t mask_rows = mask_batched ? B : 1;
  uint32_t* bits = mask ? cv.take<uint32_t>(mask_rows * mask_words(nk)) : nullptr;
  if (direct) XFB_TRY(check_workspace(cv, workspace, workspace_bytes));
  if (mask) XFB_TRY(launch_mask_bits(mask, mask_dtype == XFB_F32, mask_rows, nk, nk, bits, st));
  if (!direct) {
    bf16* q2 = cv.take<bf16>(B * H * nq * dp);
    bf16* k2 = cv.take<bf16>(B * H * nk * dp);
    bf16* v2 = cv.take<bf16>(B * H * nk * dp);
    XFB_TRY(check_workspace(cv, workspace, workspace_bytes));
    const int blocks = 2048;
    repack_heads_kernel<<<blocks, 256, 0, st>>>(qq, B * H * nq, static_cast<int>(d), dp, scale,
                                                q_pre_scaled ? 0 : 1, q2);
    repack_heads_kernel<<<blocks, 256, 0, st>>>(kk, B * H * nk, static_cast<int>(d), dp, 1.f, 0,
                                                k2);
    repack_heads_kernel<<<blocks, 256, 0, st>>>(vv, B * H * nk, static_cast<int>(d), dp, 1.f, 0,
                                                v2);
    g_launches.fetch_add(2, std::memory_order_relaxed);  // q and k repacks
    XFB_LAUNCHED();
    qq = q2;
    kk = k2;
    vv = v2;
  }
  xfb::AttnArgs a;
  a.B = static_cast<int>(B);
  a.H = static_cast<int>(H);
  a.nq = static_cast<int>(nq);
  a.nk = static_cast<int>(nk);
  a.d = static_cast<int>(d);
  a.mask_bits = bits;
  a.mask_sb = mask_batched ? mask_words(nk) : 0;
  a.bias = bias;
  a.bias_sb = bias_batched ? H * nq * nk : 0;
  a.bias_sh = nq * nk;
  a.bias_sq = nk;
  a.out = static_cast<bf16*>(out);
  a.out_sb = H * nq * d;
  a.out_sh = nq * d;
  a.out_sq = d;
  a.gate = nullptr;
  a.gate_sb = a.gate_sh = a.gate_sq = 0;
  a.bias_batched = bias_batched;
  return run_flash(dp, bias_dtype, false, qq, kk, vv, a, st, /*exact_bias=*/true);
}

XFB_API int64_t xfb_pack_attention_weights_bytes(int64_t c) { return 4 * c * c * 2; }

XFB_API int xfb_pack_attention_weights(const void* q_w, const void* k_w, const void* v_w,
                                       const void* gate_w, int w_dtype, int64_t c,
                                       void* packed, void* stream) {
  XFB_REQUIRE(c > 0 && c % 8 == 0, "attention width must be a positive multiple of 8");
  return launch_pack(q_w, k_w, v_w, gate_w, w_dtype, 2, c, c, 4 * c, packed,
                     static_cast<cudaStream_t>(stream));
}

namespace {
struct GsaWs {
  bf16 *x, *bias, *q, *k, *v, *g, *packed;
  uint32_t* bits;
};
void gsa_layout(Carver& cv, int64_t n, int64_t c, int64_t heads, bool need_pack, GsaWs* w) {
  const int64_t dp = head_pitch(c / heads);
  w->x = cv.take<bf16>(n * n * c);
  w->bias = cv.take<bf16>(heads * n * n);
  w->q = cv.take<bf16>(n * heads * n * dp);
  w->k = cv.take<bf16>(n * heads * n * dp);
  w->v = cv.take<bf16>(n * heads * n * dp);
  w->g = cv.take<bf16>(n * n * c);
  w->packed = need_pack ? cv.take<bf16>(4 * c * c) : nullptr;
  w->bits = cv.take<uint32_t>(n * mask_words(n));
}
}  // namespace

XFB_API int64_t xfb_grid_self_attention_workspace(int64_t n, int64_t c, int64_t heads) {
  if (heads <= 0) return 0;
  Carver cv{nullptr, 0, 0};
  GsaWs w;
  gsa_layout(cv, n, c, heads, true, &w);
  return cv.used;
}

XFB_API int xfb_grid_self_attention(
    const void* pair, int pair_dtype, int64_t n, int64_t c, int64_t heads, const float* mask,
    int transpose, const float* norm_weight, const float* norm_bias, double eps,
    const void* bias_weight, const void* q_w, const void* k_w, const void* v_w,
    const void* gate_w, const void* output_w, int weights_packed, const void* packed,
    void* out, int out_dtype, int accumulate, void* workspace, int64_t workspace_bytes,
    void* stream) {
  XFB_REQUIRE(n >= 0, "pair side must be non-negative");
  XFB_REQUIRE(c == 64 || c == 128, "grid self-attention supports c in {64, 128}");
  XFB_REQUIRE(heads > 0 && heads <= 16 && c % heads == 0, "heads must divide c (<= 16)");
  const int64_t d = c / heads;
  XFB_REQUIRE(d == 16 || d == 32, "grid self-attention head dim must be 16 or 32");
  XFB_REQUIRE(out_dtype == XFB_F32 || out_dtype == XFB_BF16, "output must be f32 or bf16");
  XFB_REQUIRE(!accumulate || out_dtype == XFB_F32, "accumulate requires an f32 output");
  XFB_REQUIRE(bias_weight != nullptr && output_w != nullptr, "attention weights missing");
  XFB_REQUIRE(weights_packed ? packed != nullptr : (q_w && k_w && v_w && gate_w),
              "attention weights missing");
  XFB_REQUIRE(std::isfinite(eps) && eps >= 0, "LayerNorm eps must be finite and non-negative");
  if (n == 0) return XFB_OK;
  XFB_REQUIRE(n <= 16384 && n * n <= (1ll << 31) - 256, "pair too large");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  Carver cv{static_cast<uint8_t*>(workspace), 0, workspace_bytes};
  GsaWs w;
  gsa_layout(cv, n, c, heads, !weights_packed, &w);
  XFB_TRY(check_workspace(cv, workspace, workspace_bytes));
  const int dp = head_pitch(d);
  const int64_t M = n * n;
  const bf16* wcat = static_cast<const bf16*>(packed);
  if (!weights_packed) {
    XFB_TRY(launch_pack(q_w, k_w, v_w, gate_w, XFB_BF16, 2, c, c, 4 * c, w.packed, st));
    wcat = w.packed;
  }
  // Scores in log2 units from the producers (q and bias carry log2(e)) when the
  // bias can stream through TMA; otherwise the attention kernel scales them.
  const bool pre = dp == 32 && n % 8 == 0;
  const float log2e = 1.4426950408889634f;
  // 1. x = LN(pair) and the pair bias (projected before any transpose)
  XFB_TRY(run_layer_norm(pair, pair_dtype, M, c, c, norm_weight, norm_bias, eps, w.x, c, nullptr,
                         nullptr, static_cast<const bf16*>(bias_weight),
                         static_cast<int>(heads), w.bias, M, st, pre ? log2e : 1.f));
  // 2. q, k, v (head-major per batch row) and the squashed gate
  if (d != dp) {
    const int64_t bytes = n * heads * n * dp * 2;
    XFB_CUDA(cudaMemsetAsync(w.q, 0, bytes, st));
    XFB_CUDA(cudaMemsetAsync(w.k, 0, bytes, st));
    XFB_CUDA(cudaMemsetAsync(w.v, 0, bytes, st));
  }
  if (c == 128 && heads == 4) {
    // batched over pair rows i (weight shared), TMA stores of 128-token tiles
    xfb::EpiAttProjTma epi;
    bf16* bufs[3] = {w.q, w.k, w.v};
    for (int t = 0; t < 3; ++t) {
      if (!transpose) {
        const uint64_t dims[3] = {32, static_cast<uint64_t>(n), static_cast<uint64_t>(n * 4)};
        const uint64_t strides[2] = {64, static_cast<uint64_t>(n * 64)};
        const uint32_t box[3] = {32, 128, 1};
        XFB_TRY(make_map_nd(&epi.qkv_map[t], false, 3, bufs[t], dims, strides, box,
                            CU_TENSOR_MAP_SWIZZLE_64B));
      } else {
        const uint64_t dims[4] = {32, static_cast<uint64_t>(n), 4, static_cast<uint64_t>(n)};
        const uint64_t strides[3] = {64, static_cast<uint64_t>(n * 64),
                                     static_cast<uint64_t>(4 * n * 64)};
        const uint32_t box[4] = {32, 1, 1, 128};
        XFB_TRY(make_map_nd(&epi.qkv_map[t], false, 4, bufs[t], dims, strides, box,
                            CU_TENSOR_MAP_SWIZZLE_64B));
      }
    }
    const uint64_t g_dims[3] = {static_cast<uint64_t>(c), static_cast<uint64_t>(n),
                                static_cast<uint64_t>(n)};
    const uint64_t g_strides[2] = {static_cast<uint64_t>(c * 2), static_cast<uint64_t>(n * c * 2)};
    const uint32_t g_box[3] = {64, 128, 1};
    XFB_TRY(make_map_nd(&epi.g_map, false, 3, w.g, g_dims, g_strides, g_box,
                        CU_TENSOR_MAP_SWIZZLE_128B));
    epi.q_scale = (pre ? log2e : 1.f) / std::sqrt(static_cast<float>(d));
    epi.transpose = transpose;
    XFB_TRY((run_gemm<128, false, false>(w.x, c, n * c, wcat, c, 0, n, 4 * c, c, n, epi, st,
                                         true)));
  } else {
    xfb::EpiAttProjDirect epi;
    epi.q = w.q;
    epi.k = w.k;
    epi.v = w.v;
    epi.g = w.g;
    epi.n = static_cast<int>(n);
    epi.c = static_cast<int>(c);
    epi.heads = static_cast<int>(heads);
    epi.d = static_cast<int>(d);
    epi.dp = dp;
    epi.transpose = transpose;
    epi.M = static_cast<int>(M);
    epi.q_scale = (pre ? log2e : 1.f) / std::sqrt(static_cast<float>(d));
    epi.q_bias = nullptr;
    XFB_TRY((run_gemm<128, false, false>(w.x, c, 0, wcat, c, 0, M, 4 * c, c, 1, epi, st)));
  }
  // 3. attention per batch row; output written back in pair order, gated (x reused)
  {
    xfb::AttnArgs a;
    a.B = static_cast<int>(n);
    a.H = static_cast<int>(heads);
    a.nq = static_cast<int>(n);
    a.nk = static_cast<int>(n);
    a.d = static_cast<int>(d);
    if (mask != nullptr) XFB_TRY(launch_mask_bits(mask, true, n, n, n, w.bits, st));
    a.mask_bits = mask ? w.bits : nullptr;
    a.mask_sb = mask_words(n);
    a.bias = w.bias;
    a.bias_sb = 0;
    a.bias_sh = M;
    a.bias_sq = n;
    a.bias_batched = 0;
    a.out = w.x;
    a.gate = w.g;
    if (!transpose) {  // batch row r = pair row i, token = column j
      a.out_sb = n * c;
      a.out_sq = c;
    } else {  // batch row r = pair column j, token = row i
      a.out_sb = c;
      a.out_sq = n * c;
    }
    a.out_sh = d;
    a.gate_sb = a.out_sb;
    a.gate_sh = a.out_sh;
    a.gate_sq = a.out_sq;
    XFB_TRY(run_flash(dp, XFB_BF16, pre, w.q, w.k, w.v, a, st));
  }
  // 4. output projection (+ residual)
  XFB_REQUIRE(aligned16(out), "output must be 16-byte aligned");
  return linear_core(w.x, M, c, c, static_cast<const bf16*>(output_w), c, nullptr, nullptr, 0,
                     out, out_dtype == XFB_F32, accumulate, c, st);
}

// ---------------------------------------------------------------- transition

namespace {
struct TrWs {
  bf16 *x, *h, *packed;
};
void tr_layout(Carver& cv, int64_t rows, int64_t c, int64_t f, bool need_pack, TrWs* w) {
  w->x = cv.take<bf16>(rows * c);
  w->h = cv.take<bf16>(rows * f * c);
  w->packed = need_pack ? cv.take<bf16>(2 * f * c * c) : nullptr;
}
}  // namespace

XFB_API int64_t xfb_transition_workspace(int64_t rows, int64_t c, int64_t factor) {
  Carver cv{nullptr, 0, 0};
  TrWs w;
  tr_layout(cv, rows, c, factor, true, &w);
  return cv.used;
}

namespace {
// The fused GLU transition (transition.cuh) for c = 128 with an f32 output and
// no output gate; XFB_FUSED_TRANSITION=0 selects the two-GEMM form.
bool use_fused_transition() {
  static const bool enabled = [] {
    const char* e = std::getenv("XFB_FUSED_TRANSITION");
    return e == nullptr || std::strcmp(e, "0") != 0;
  }();
  return enabled;
}

int launch_fused_transition(const bf16* x, int64_t rows, int64_t hid, const bf16* w1p,
                            const bf16* w2, void* out, int accumulate, cudaStream_t st) {
  XFB_REQUIRE(rows <= (1ll << 31) - 256, "transition has too many rows");
  XFB_REQUIRE(aligned16(x) && aligned16(w1p) && aligned16(w2),
              "transition buffers must be 16-byte aligned");
  CUtensorMap tx, tw1, tw2, to;
  XFB_TRY(make_map(&tx, x, 128, rows, 1, 256, 0, 64, 128, CU_TENSOR_MAP_SWIZZLE_128B));
  XFB_TRY(make_map(&tw1, w1p, 128, 2 * hid, 1, 256, 0, 64, 128, CU_TENSOR_MAP_SWIZZLE_128B));
  XFB_TRY(make_map(&tw2, w2, hid, 128, 1, hid * 2, 0, 64, 128, CU_TENSOR_MAP_SWIZZLE_128B));
  XFB_TRY(make_out_map(&to, out, true, 128, rows, 1, 128, 0));
  int sms;
  XFB_TRY(sm_count(&sms));
  const int64_t m_tiles = (rows + 127) / 128;
  const int grid = static_cast<int>(std::min<int64_t>(m_tiles, sms));
  XFB_TRY(set_smem(xfb::fused_transition_kernel, xfb::FtSmem::kLaunchBytes));
  xfb::fused_transition_kernel<<<grid, xfb::kFtThreads, xfb::FtSmem::kLaunchBytes, st>>>(
      tx, tw1, tw2, to, static_cast<int>(rows), static_cast<int>(hid / 64), accumulate);
  XFB_LAUNCHED();
  return XFB_OK;
}
}  // namespace

XFB_API int xfb_transition(const void* x, int x_dtype, int64_t rows, int64_t c,
                           int64_t factor, const float* norm_weight, const float* norm_bias,
                           double eps, const void* mod_scale, const void* mod_shift,
                           const void* w1, int weights_packed, const void* w2,
                           const void* out_gate, void* out, int out_dtype, int accumulate,
                           void* workspace, int64_t workspace_bytes, void* stream) {
  XFB_REQUIRE(rows >= 0 && factor > 0, "transition expects rows >= 0 and factor > 0");
  XFB_REQUIRE(c == 64 || c == 128 || c == 384 || c == 768, "transition width must be 64/128/384/768");
  XFB_REQUIRE((factor * c) % 64 == 0, "transition hidden width must be a multiple of 64");
  XFB_REQUIRE(out_dtype == XFB_F32 || out_dtype == XFB_BF16, "output must be f32 or bf16");
  XFB_REQUIRE(!accumulate || out_dtype == XFB_F32, "accumulate requires an f32 output");
  XFB_REQUIRE(w1 != nullptr && w2 != nullptr, "transition weights missing");
  XFB_REQUIRE(std::isfinite(eps) && eps >= 0, "LayerNorm eps must be finite and non-negative");
  XFB_REQUIRE(aligned16(out), "output must be 16-byte aligned");
  if (rows == 0) return XFB_OK;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  Carver cv{static_cast<uint8_t*>(workspace), 0, workspace_bytes};
  TrWs w;
  tr_layout(cv, rows, c, factor, !weights_packed, &w);
  XFB_TRY(check_workspace(cv, workspace, workspace_bytes));
  const int64_t hid = factor * c;
  const bf16* w1p = static_cast<const bf16*>(w1);
  if (!weights_packed) {
    XFB_TRY(launch_pack(w1, nullptr, nullptr, nullptr, XFB_BF16, 1, hid, c, 2 * hid, w.packed, st));
    w1p = w.packed;
  }
  XFB_TRY(run_layer_norm(x, x_dtype, rows, c, c, norm_weight, norm_bias, eps, w.x, c,
                         static_cast<const bf16*>(mod_scale), static_cast<const bf16*>(mod_shift),
                         nullptr, 0, nullptr, 0, st));
  if (c == 128 && out_gate == nullptr && out_dtype == XFB_F32 && use_fused_transition()) {
    return launch_fused_transition(w.x, rows, hid, w1p, static_cast<const bf16*>(w2), out,
                                   accumulate, st);
  }
  {
    xfb::EpiGLU epi;
    XFB_TRY(make_out_map(&epi.out_map, w.h, false, hid, rows, 1, hid, 0));
    XFB_TRY((run_gemm<128, false, false>(w.x, c, 0, w1p, c, 0, rows, 2 * hid, c, 1, epi, st)));
  }
  return linear_core(w.h, rows, hid, hid, static_cast<const bf16*>(w2), c, nullptr,
                     static_cast<const bf16*>(out_gate), c, out, out_dtype == XFB_F32,
                     accumulate, c, st);
}

// ---------------------------------------------------------------- single attention

namespace {
struct SaWs {
  bf16 *x, *q, *k, *v, *g, *packed;
  uint32_t* bits;
};
void sa_layout(Carver& cv, int64_t n, int64_t c, int64_t heads, bool need_pack, SaWs* w) {
  const int64_t dp = head_pitch(c / heads);
  w->x = cv.take<bf16>(n * c);
  w->q = cv.take<bf16>(heads * n * dp);
  w->k = cv.take<bf16>(heads * n * dp);
  w->v = cv.take<bf16>(heads * n * dp);
  w->g = cv.take<bf16>(n * c);
  w->packed = need_pack ? cv.take<bf16>(4 * c * c) : nullptr;
  w->bits = cv.take<uint32_t>(mask_words(n));
}
}  // namespace

XFB_API int64_t xfb_self_attention_workspace(int64_t n, int64_t c, int64_t heads) {
  if (heads <= 0) return 0;
  Carver cv{nullptr, 0, 0};
  SaWs w;
  sa_layout(cv, n, c, heads, true, &w);
  return cv.used;
}

namespace {
// Self-attention of the query rows [row0, row0 + q_rows) against all n keys;
// LayerNorm and projections run on all n tokens (the keys need them), the
// attention, output projection and update only on the query rows, whose pair
// logits are `pair_logits` [heads][q_rows][n].
int self_attention_impl(const void* x, int x_dtype, int64_t n, int64_t c, int64_t heads,
                        int64_t row0, int64_t q_rows, const float* mask, const void* pair_logits,
                        const float* norm_weight, const float* norm_bias, double eps,
                        const void* mod_scale, const void* mod_shift, const void* q_w,
                        const float* q_bias, const void* k_w, const void* v_w, const void* gate_w,
                        int weights_packed, const void* packed, const void* wo,
                        const void* out_gate, void* out, int out_dtype, int accumulate,
                        void* workspace, int64_t workspace_bytes, void* stream) {
  XFB_REQUIRE(n >= 0, "token count must be non-negative");
  XFB_REQUIRE(c == 128 || c == 384 || c == 768, "self-attention width must be 128, 384 or 768");
  XFB_REQUIRE(heads > 0 && c % heads == 0 && c / heads <= 64, "heads must divide c, d <= 64");
  XFB_REQUIRE(out_dtype == XFB_F32 || out_dtype == XFB_BF16, "output must be f32 or bf16");
  XFB_REQUIRE(!accumulate || out_dtype == XFB_F32, "accumulate requires an f32 output");
  XFB_REQUIRE(wo != nullptr, "output projection weight missing");
  XFB_REQUIRE(weights_packed ? packed != nullptr : (q_w && k_w && v_w && gate_w),
              "attention weights missing");
  XFB_REQUIRE(std::isfinite(eps) && eps >= 0, "LayerNorm eps must be finite and non-negative");
  XFB_REQUIRE(aligned16(out), "output must be 16-byte aligned");
  XFB_REQUIRE(row0 >= 0 && q_rows >= 0 && row0 + q_rows <= n, "query rows out of range");
  if (n == 0 || q_rows == 0) return XFB_OK;
  XFB_REQUIRE(n <= 16384, "self-attention supports at most 16384 tokens");
  const bool subset = q_rows != n;
  XFB_REQUIRE(!subset || (row0 * c) % 8 == 0, "query rows must start on a 16-byte boundary");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  Carver cv{static_cast<uint8_t*>(workspace), 0, workspace_bytes};
  SaWs w;
  sa_layout(cv, n, c, heads, !weights_packed, &w);
  const int64_t d = c / heads;
  const int dp = head_pitch(d);
  bf16* q_sub = subset ? cv.take<bf16>(heads * q_rows * dp) : nullptr;
  XFB_TRY(check_workspace(cv, workspace, workspace_bytes));
  const bf16* wcat = static_cast<const bf16*>(packed);
  if (!weights_packed) {
    XFB_TRY(launch_pack(q_w, k_w, v_w, gate_w, XFB_BF16, 2, c, c, 4 * c, w.packed, st));
    wcat = w.packed;
  }
  XFB_TRY(run_layer_norm(x, x_dtype, n, c, c, norm_weight, norm_bias, eps, w.x, c,
                         static_cast<const bf16*>(mod_scale), static_cast<const bf16*>(mod_shift),
                         nullptr, 0, nullptr, 0, st));
  if (d != dp) {
    const int64_t bytes = heads * n * dp * 2;
    XFB_CUDA(cudaMemsetAsync(w.q, 0, bytes, st));
    XFB_CUDA(cudaMemsetAsync(w.k, 0, bytes, st));
    XFB_CUDA(cudaMemsetAsync(w.v, 0, bytes, st));
  }
  {
    xfb::EpiAttProjDirect epi;
    epi.q = w.q;
    epi.k = w.k;
    epi.v = w.v;
    epi.g = w.g;
    epi.n = static_cast<int>(n);
    epi.c = static_cast<int>(c);
    epi.heads = static_cast<int>(heads);
    epi.d = static_cast<int>(d);
    epi.dp = dp;
    epi.transpose = 0;
    epi.M = static_cast<int>(n);
    epi.q_scale = 1.f / std::sqrt(static_cast<float>(d));
    epi.q_bias = q_bias;
    XFB_TRY((run_gemm<128, false, false>(w.x, c, 0, wcat, c, 0, n, 4 * c, c, 1, epi, st)));
  }
  const bf16* q = w.q;
  if (subset) {
    // the query rows of every head, [heads][q_rows][dp]
    XFB_CUDA(cudaMemcpy2DAsync(q_sub, q_rows * dp * 2, w.q + row0 * dp, n * dp * 2,
                               q_rows * dp * 2, heads, cudaMemcpyDeviceToDevice, st));
    q = q_sub;
  }
  bf16* o = w.x + row0 * c;  // the LayerNorm'd tokens are no longer needed
  {
    xfb::AttnArgs a;
    a.B = 1;
    a.H = static_cast<int>(heads);
    a.nq = static_cast<int>(q_rows);
    a.nk = static_cast<int>(n);
    a.d = static_cast<int>(d);
    if (mask != nullptr) XFB_TRY(launch_mask_bits(mask, true, 1, n, n, w.bits, st));
    a.mask_bits = mask ? w.bits : nullptr;
    a.mask_sb = 0;
    a.bias = pair_logits;
    a.bias_sb = 0;
    a.bias_sh = q_rows * n;
    a.bias_sq = n;
    a.bias_batched = 0;
    a.out = o;
    a.out_sb = 0;
    a.out_sh = d;
    a.out_sq = c;
    a.gate = w.g + row0 * c;
    a.gate_sb = 0;
    a.gate_sh = d;
    a.gate_sq = c;
    XFB_TRY(run_flash(dp, XFB_BF16, false, q, w.k, w.v, a, st));
  }
  const bf16* og = out_gate ? static_cast<const bf16*>(out_gate) + row0 * c : nullptr;
  void* out_rows = static_cast<uint8_t*>(out) + row0 * c * (out_dtype == XFB_F32 ? 4 : 2);
  return linear_core(o, q_rows, c, c, static_cast<const bf16*>(wo), c, nullptr, og, c, out_rows,
                     out_dtype == XFB_F32, accumulate, c, st);
}
}  // namespace

XFB_API int xfb_self_attention(const void* x, int x_dtype, int64_t n, int64_t c, int64_t heads,
                               const float* mask, const void* pair_logits,
                               const float* norm_weight, const float* norm_bias, double eps,
                               const void* mod_scale, const void* mod_shift, const void* q_w,
                               const float* q_bias, const void* k_w, const void* v_w,
                               const void* gate_w, int weights_packed, const void* packed,
                               const void* wo, const void* out_gate, void* out, int out_dtype,
                               int accumulate, void* workspace, int64_t workspace_bytes,
                               void* stream) {
  return self_attention_impl(x, x_dtype, n, c, heads, 0, n, mask, pair_logits, norm_weight,
                             norm_bias, eps, mod_scale, mod_shift, q_w, q_bias, k_w, v_w, gate_w,
                             weights_packed, packed, wo, out_gate, out, out_dtype, accumulate,
                             workspace, workspace_bytes, stream);
}

XFB_API int64_t xfb_self_attention_rows_workspace(int64_t n, int64_t c, int64_t heads,
                                                  int64_t q_rows) {
  if (heads <= 0) return 0;
  Carver cv{nullptr, 0, 0};
  SaWs w;
  sa_layout(cv, n, c, heads, false, &w);
  cv.take<bf16>(heads * q_rows * head_pitch(c / heads));
  return cv.used;
}

XFB_API int xfb_self_attention_rows(const void* x, int x_dtype, int64_t n, int64_t c,
                                    int64_t heads, int64_t row0, int64_t q_rows,
                                    const float* mask, const void* pair_logits,
                                    const float* norm_weight, const float* norm_bias, double eps,
                                    const void* packed, const float* q_bias, const void* wo,
                                    const void* out_gate, void* out, int out_dtype,
                                    int accumulate, void* workspace, int64_t workspace_bytes,
                                    void* stream) {
  XFB_REQUIRE(packed != nullptr, "packed attention weights are required");
  return self_attention_impl(x, x_dtype, n, c, heads, row0, q_rows, mask, pair_logits,
                             norm_weight, norm_bias, eps, nullptr, nullptr, nullptr, q_bias,
                             nullptr, nullptr, nullptr, 1, packed, wo, out_gate, out, out_dtype,
                             accumulate, workspace, workspace_bytes, stream);
}

XFB_API int xfb_pair_logits(const void* pair, int pair_dtype, int64_t n, int64_t c,
                            int64_t heads, const float* norm_weight, const float* norm_bias,
                            double eps, const void* w, void* logits, void* stream) {
  XFB_REQUIRE(n >= 0 && heads > 0 && heads <= 16, "pair logits expect 1..16 heads");
  XFB_REQUIRE(c == 64 || c == 128, "pair width must be 64 or 128");
  if (n == 0) return XFB_OK;
  return run_layer_norm(pair, pair_dtype, n * n, c, c, norm_weight, norm_bias, eps, nullptr, 0,
                        nullptr, nullptr, static_cast<const bf16*>(w), static_cast<int>(heads),
                        static_cast<bf16*>(logits), n * n, static_cast<cudaStream_t>(stream));
}


// ---------------------------------------------------------------- row-block stages
// The operators above take the whole N x N pair.  The entry points below run the
// same arithmetic on a block of pair rows and stop where a row-sharded pair needs
// an exchange between GPUs: TriMul projection | rows -> channels | contraction
// (xfb_gemm) | channels -> rows | TriMul output; grid-attention prepare (LN and
// the bias rows) | bias all-gather (and, for the ending node, a row <-> column
// transpose of the LN'd pair) | grid attention on rows.  Every tensor here has
// n % 8 == 0 columns so rows can be exchanged without padding.

namespace {
// Scores in log2 units (q and bias pre-multiplied by log2(e)) exactly when the
// attention kernel streams the bias by TMA with 32-wide heads.
bool grid_pre_scaled(int64_t c, int64_t heads, int64_t n) {
  return head_pitch(static_cast<int>(c / heads)) == 32 && n % 8 == 0;
}

struct RowAttWs {
  bf16 *q, *k, *v, *g, *o;
  uint32_t* bits;
};
void row_att_layout(Carver& cv, int64_t rows, int64_t n, int64_t c, int64_t heads, RowAttWs* w) {
  const int64_t dp = head_pitch(static_cast<int>(c / heads));
  w->q = cv.take<bf16>(rows * heads * n * dp);
  w->k = cv.take<bf16>(rows * heads * n * dp);
  w->v = cv.take<bf16>(rows * heads * n * dp);
  w->g = cv.take<bf16>(rows * n * c);
  w->o = cv.take<bf16>(rows * n * c);
  w->bits = cv.take<uint32_t>(rows * mask_words(n));
}
}  // namespace

XFB_API int64_t xfb_triangle_projection_workspace(int64_t rows, int64_t n, int64_t c) {
  Carver cv{nullptr, 0, 0};
  cv.take<bf16>(rows * n * c);
  return cv.used;
}

namespace {
int triangle_projection_impl(const void* pair, int pair_dtype, int64_t rows, int64_t n, int64_t c,
                             const float* mask, const float* left_weight, const float* left_bias,
                             double left_eps, const void* packed, void* a, void* b,
                             const Route* ra, const Route* rb, void* g, void* workspace,
                             int64_t workspace_bytes, cudaStream_t st) {
  XFB_REQUIRE(rows >= 0 && n >= 0 && n % 8 == 0, "row blocks need n % 8 == 0 columns");
  XFB_REQUIRE(c == 64 || c == 128, "triangle multiplication supports c in {64, 128}");
  XFB_REQUIRE(packed != nullptr, "packed triangle weights are required");
  XFB_REQUIRE(std::isfinite(left_eps) && left_eps >= 0, "LayerNorm eps must be finite and non-negative");
  XFB_REQUIRE(aligned16(a) && aligned16(b) && aligned16(g), "a, b, g must be 16-byte aligned");
  if (rows == 0 || n == 0) return XFB_OK;
  XFB_REQUIRE(rows * n <= (1ll << 31) - 256, "row block too large");
  Carver cv{static_cast<uint8_t*>(workspace), 0, workspace_bytes};
  bf16* x = cv.take<bf16>(rows * n * c);
  XFB_TRY(check_workspace(cv, workspace, workspace_bytes));
  XFB_TRY(run_layer_norm(pair, pair_dtype, rows * n, c, c, left_weight, left_bias, left_eps, x, c,
                         nullptr, nullptr, nullptr, 0, nullptr, 0, st));
  xfb::EpiTriProj epi;
  if (ra != nullptr) {
    // rows -> channels by the producer: rank s receives channels [s cs, (s+1) cs)
    // of every row block as [cs][n][n]
    XFB_REQUIRE(rows * ra->world == n && c % ra->world == 0,
                "a routed row block holds n / world rows and c / world channels per rank");
    std::memset(&epi.a_map, 0, sizeof(epi.a_map));
    std::memset(&epi.b_map, 0, sizeof(epi.b_map));
    epi.route = 1;
    epi.rank = ra->rank;
    epi.route_rows = static_cast<int>(rows);
    epi.route_cs = static_cast<int>(c / ra->world);
    for (int s = 0; s < xfb::kMaxRoute; ++s) {
      epi.a_dst[s] = s < ra->world ? ra->dst[s] : nullptr;
      epi.b_dst[s] = s < rb->world ? rb->dst[s] : nullptr;
    }
  } else {
    const uint64_t ab_dims[3] = {static_cast<uint64_t>(n), static_cast<uint64_t>(rows),
                                 static_cast<uint64_t>(c)};
    const uint64_t ab_strides[2] = {static_cast<uint64_t>(n * 2),
                                    static_cast<uint64_t>(rows * n * 2)};
    const uint32_t ab_box[3] = {128, 1, 32};
    XFB_TRY(make_map_nd(&epi.a_map, false, 3, a, ab_dims, ab_strides, ab_box,
                        CU_TENSOR_MAP_SWIZZLE_NONE));
    XFB_TRY(make_map_nd(&epi.b_map, false, 3, b, ab_dims, ab_strides, ab_box,
                        CU_TENSOR_MAP_SWIZZLE_NONE));
  }
  const uint64_t g_dims[3] = {static_cast<uint64_t>(c), static_cast<uint64_t>(n),
                              static_cast<uint64_t>(rows)};
  const uint64_t g_strides[2] = {static_cast<uint64_t>(c * 2), static_cast<uint64_t>(n * c * 2)};
  const uint32_t g_box[3] = {64, 128, 1};
  XFB_TRY(make_map_nd(&epi.g_map, false, 3, g, g_dims, g_strides, g_box,
                      CU_TENSOR_MAP_SWIZZLE_128B));
  epi.mask = mask;
  epi.n = static_cast<int>(n);
  epi.n_proj_tiles = static_cast<int>(2 * c / 64);
  epi.c = static_cast<int>(c);
  return run_gemm<128, false, false>(x, c, n * c, packed, c, 0, n, 5 * c, c, rows, epi, st, true);
}
}  // namespace

XFB_API int xfb_triangle_projection(const void* pair, int pair_dtype, int64_t rows, int64_t n,
                                    int64_t c, const float* mask, const float* left_weight,
                                    const float* left_bias, double left_eps, const void* packed,
                                    void* a, void* b, void* g, void* workspace,
                                    int64_t workspace_bytes, void* stream) {
  return triangle_projection_impl(pair, pair_dtype, rows, n, c, mask, left_weight, left_bias,
                                  left_eps, packed, a, b, nullptr, nullptr, g, workspace,
                                  workspace_bytes, static_cast<cudaStream_t>(stream));
}

XFB_API int xfb_triangle_projection_routed(const void* pair, int pair_dtype, int64_t rows,
                                           int64_t n, int64_t c, const float* mask,
                                           const float* left_weight, const float* left_bias,
                                           double left_eps, const void* packed,
                                           void* const* a_dst, void* const* b_dst, int world,
                                           int rank, void* g, void* workspace,
                                           int64_t workspace_bytes, void* stream) {
  XFB_TRY(check_route(a_dst, world, rank));
  XFB_TRY(check_route(b_dst, world, rank));
  const Route ra{a_dst, world, rank}, rb{b_dst, world, rank};
  return triangle_projection_impl(pair, pair_dtype, rows, n, c, mask, left_weight, left_bias,
                                  left_eps, packed, a_dst[rank], b_dst[rank], &ra, &rb, g,
                                  workspace, workspace_bytes, static_cast<cudaStream_t>(stream));
}

XFB_API int xfb_triangle_contraction_routed(const void* a, const void* b, int64_t cs, int64_t n,
                                            int outgoing, void* const* z_dst, int world, int rank,
                                            void* stream) {
  XFB_TRY(check_route(z_dst, world, rank));
  XFB_REQUIRE(cs >= 0 && n >= 0 && n % 8 == 0, "the contraction needs n % 8 == 0");
  XFB_REQUIRE(n % world == 0, "a routed contraction splits n rows evenly over the ranks");
  XFB_REQUIRE(aligned16(a) && aligned16(b), "a and b must be 16-byte aligned");
  if (cs == 0 || n == 0) return XFB_OK;
  xfb::EpiRowsRouted<128> epi;
  epi.ld_out = n;
  epi.M = static_cast<int>(n);
  epi.N = static_cast<int>(n);
  epi.route = 1;
  epi.rank = rank;
  epi.route_rows = static_cast<int>(n / world);
  epi.route_batch = static_cast<int>(cs);
  epi.route_n = static_cast<int>(n);
  for (int s = 0; s < xfb::kMaxRoute; ++s) epi.dst[s] = s < world ? z_dst[s] : nullptr;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int64_t bs = n * n;
  // outgoing z[c,i,j] = sum_k a[c,i,k] b[c,j,k]; incoming sum_k a[c,k,j] b[c,k,i]
  if (outgoing) return run_gemm<128, false, false>(a, n, bs, b, n, bs, n, n, n, cs, epi, st);
  return run_gemm<128, true, true>(b, n, bs, a, n, bs, n, n, n, cs, epi, st);
}

XFB_API int64_t xfb_triangle_output_workspace(int64_t rows, int64_t n, int64_t c) {
  Carver cv{nullptr, 0, 0};
  TriCenterWs w;
  tri_center_layout(cv, rows * n, c, &w);
  return cv.used;
}

XFB_API int xfb_triangle_output(const void* z, int64_t rows, int64_t n, int64_t c, const void* g,
                                const float* center_weight, const float* center_bias,
                                double center_eps, const void* output_weight, void* out,
                                int out_dtype, int accumulate, void* workspace,
                                int64_t workspace_bytes, void* stream) {
  XFB_REQUIRE(rows >= 0 && n >= 0 && n % 8 == 0, "row blocks need n % 8 == 0 columns");
  XFB_REQUIRE(c == 64 || c == 128, "triangle multiplication supports c in {64, 128}");
  XFB_REQUIRE(out_dtype == XFB_F32 || out_dtype == XFB_BF16, "output must be f32 or bf16");
  XFB_REQUIRE(!accumulate || out_dtype == XFB_F32, "accumulate requires an f32 output");
  XFB_REQUIRE(std::isfinite(center_eps) && center_eps >= 0,
              "LayerNorm eps must be finite and non-negative");
  XFB_REQUIRE(output_weight != nullptr && g != nullptr, "output weight and gate are required");
  if (rows == 0 || n == 0) return XFB_OK;
  XFB_REQUIRE(rows * n <= (1ll << 31) - 256, "row block too large");
  XFB_REQUIRE(aligned16(out), "output must be 16-byte aligned");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  Carver cv{static_cast<uint8_t*>(workspace), 0, workspace_bytes};
  TriCenterWs w;
  tri_center_layout(cv, rows * n, c, &w);
  XFB_TRY(check_workspace(cv, workspace, workspace_bytes));
  return tri_center_output(static_cast<const bf16*>(z), rows * n, c, static_cast<const bf16*>(g),
                           center_weight, center_bias, center_eps,
                           static_cast<const bf16*>(output_weight), out, out_dtype == XFB_F32,
                           accumulate, w, st);
}

namespace {
int grid_attention_prepare_impl(const void* pair, int pair_dtype, int64_t rows, int64_t n,
                                int64_t c, int64_t heads, const float* norm_weight,
                                const float* norm_bias, double eps, const void* bias_weight,
                                void* x, const Route* x_route, void* bias, void* stream) {
  XFB_REQUIRE(rows >= 0 && n >= 0 && n % 8 == 0, "row blocks need n % 8 == 0 columns");
  XFB_REQUIRE(c == 64 || c == 128, "grid self-attention supports c in {64, 128}");
  XFB_REQUIRE(heads > 0 && heads <= 16 && c % heads == 0, "heads must divide c (<= 16)");
  XFB_REQUIRE(bias_weight != nullptr && x != nullptr && bias != nullptr,
              "bias weight and outputs are required");
  XFB_REQUIRE(std::isfinite(eps) && eps >= 0, "LayerNorm eps must be finite and non-negative");
  if (rows == 0 || n == 0) return XFB_OK;
  const float scale = grid_pre_scaled(c, heads, n) ? 1.4426950408889634f : 1.f;
  return run_layer_norm(pair, pair_dtype, rows * n, c, c, norm_weight, norm_bias, eps,
                        static_cast<bf16*>(x), c, nullptr, nullptr,
                        static_cast<const bf16*>(bias_weight), static_cast<int>(heads),
                        static_cast<bf16*>(bias), rows * n, static_cast<cudaStream_t>(stream),
                        scale, nullptr, nullptr, 0, 0, 0, x_route, n);
}
}  // namespace

XFB_API int xfb_grid_attention_prepare(const void* pair, int pair_dtype, int64_t rows, int64_t n,
                                       int64_t c, int64_t heads, const float* norm_weight,
                                       const float* norm_bias, double eps, const void* bias_weight,
                                       void* x, void* bias, void* stream) {
  return grid_attention_prepare_impl(pair, pair_dtype, rows, n, c, heads, norm_weight, norm_bias,
                                     eps, bias_weight, x, nullptr, bias, stream);
}

XFB_API int xfb_grid_attention_prepare_routed(const void* pair, int pair_dtype, int64_t rows,
                                              int64_t n, int64_t c, int64_t heads,
                                              const float* norm_weight, const float* norm_bias,
                                              double eps, const void* bias_weight,
                                              void* const* x_dst, int world, int rank, void* bias,
                                              void* stream) {
  XFB_TRY(check_route(x_dst, world, rank));
  XFB_REQUIRE(rows * world == n, "a routed row block holds n / world rows");
  const Route r{x_dst, world, rank};
  return grid_attention_prepare_impl(pair, pair_dtype, rows, n, c, heads, norm_weight, norm_bias,
                                     eps, bias_weight, x_dst[rank], &r, bias, stream);
}

XFB_API int64_t xfb_grid_attention_rows_workspace(int64_t rows, int64_t n, int64_t c,
                                                  int64_t heads) {
  if (heads <= 0) return 0;
  Carver cv{nullptr, 0, 0};
  RowAttWs w;
  row_att_layout(cv, rows, n, c, heads, &w);
  return cv.used;
}

namespace {
int grid_attention_rows_impl(const void* x, int64_t rows, int64_t n, int64_t c, int64_t heads,
                             const float* mask, const void* bias, const void* packed,
                             const void* output_w, void* out, int out_dtype, int accumulate,
                             const Route* out_route, void* workspace, int64_t workspace_bytes,
                             void* stream) {
  XFB_REQUIRE(rows >= 0 && n >= 0 && n % 8 == 0, "row blocks need n % 8 == 0 columns");
  XFB_REQUIRE(c == 64 || c == 128, "grid self-attention supports c in {64, 128}");
  XFB_REQUIRE(heads > 0 && heads <= 16 && c % heads == 0, "heads must divide c (<= 16)");
  const int64_t d = c / heads;
  XFB_REQUIRE(d == 16 || d == 32, "grid self-attention head dim must be 16 or 32");
  XFB_REQUIRE(out_dtype == XFB_F32 || out_dtype == XFB_BF16, "output must be f32 or bf16");
  XFB_REQUIRE(!accumulate || out_dtype == XFB_F32, "accumulate requires an f32 output");
  XFB_REQUIRE(packed != nullptr && output_w != nullptr && bias != nullptr,
              "packed weights, output weight and bias are required");
  if (rows == 0 || n == 0) return XFB_OK;
  XFB_REQUIRE(n <= 16384 && rows * n <= (1ll << 31) - 256, "row block too large");
  XFB_REQUIRE(aligned16(out) && aligned16(bias), "output and bias must be 16-byte aligned");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  Carver cv{static_cast<uint8_t*>(workspace), 0, workspace_bytes};
  RowAttWs w;
  row_att_layout(cv, rows, n, c, heads, &w);
  XFB_TRY(check_workspace(cv, workspace, workspace_bytes));
  const int dp = head_pitch(static_cast<int>(d));
  const bool pre = grid_pre_scaled(c, heads, n);
  const float log2e = 1.4426950408889634f;
  const bf16* xx = static_cast<const bf16*>(x);
  const bf16* wcat = static_cast<const bf16*>(packed);
  if (d != dp) {
    const int64_t bytes = rows * heads * n * dp * 2;
    XFB_CUDA(cudaMemsetAsync(w.q, 0, bytes, st));
    XFB_CUDA(cudaMemsetAsync(w.k, 0, bytes, st));
    XFB_CUDA(cudaMemsetAsync(w.v, 0, bytes, st));
  }
  if (c == 128 && heads == 4) {
    xfb::EpiAttProjTma epi;
    bf16* bufs[3] = {w.q, w.k, w.v};
    for (int t = 0; t < 3; ++t) {
      const uint64_t dims[3] = {32, static_cast<uint64_t>(n), static_cast<uint64_t>(rows * 4)};
      const uint64_t strides[2] = {64, static_cast<uint64_t>(n * 64)};
      const uint32_t box[3] = {32, 128, 1};
      XFB_TRY(make_map_nd(&epi.qkv_map[t], false, 3, bufs[t], dims, strides, box,
                          CU_TENSOR_MAP_SWIZZLE_64B));
    }
    const uint64_t g_dims[3] = {static_cast<uint64_t>(c), static_cast<uint64_t>(n),
                                static_cast<uint64_t>(rows)};
    const uint64_t g_strides[2] = {static_cast<uint64_t>(c * 2), static_cast<uint64_t>(n * c * 2)};
    const uint32_t g_box[3] = {64, 128, 1};
    XFB_TRY(make_map_nd(&epi.g_map, false, 3, w.g, g_dims, g_strides, g_box,
                        CU_TENSOR_MAP_SWIZZLE_128B));
    epi.q_scale = (pre ? log2e : 1.f) / std::sqrt(static_cast<float>(d));
    epi.transpose = 0;
    XFB_TRY((run_gemm<128, false, false>(xx, c, n * c, wcat, c, 0, n, 4 * c, c, rows, epi, st,
                                         true)));
  } else {
    xfb::EpiAttProjDirect epi;
    epi.q = w.q;
    epi.k = w.k;
    epi.v = w.v;
    epi.g = w.g;
    epi.n = static_cast<int>(n);
    epi.c = static_cast<int>(c);
    epi.heads = static_cast<int>(heads);
    epi.d = static_cast<int>(d);
    epi.dp = dp;
    epi.transpose = 0;
    epi.M = static_cast<int>(rows * n);
    epi.q_scale = (pre ? log2e : 1.f) / std::sqrt(static_cast<float>(d));
    epi.q_bias = nullptr;
    XFB_TRY((run_gemm<128, false, false>(xx, c, 0, wcat, c, 0, rows * n, 4 * c, c, 1, epi, st)));
  }
  xfb::AttnArgs a;
  a.B = static_cast<int>(rows);
  a.H = static_cast<int>(heads);
  a.nq = static_cast<int>(n);
  a.nk = static_cast<int>(n);
  a.d = static_cast<int>(d);
  if (mask != nullptr) XFB_TRY(launch_mask_bits(mask, true, rows, n, n, w.bits, st));
  a.mask_bits = mask ? w.bits : nullptr;
  a.mask_sb = mask_words(n);
  a.bias = bias;
  a.bias_sb = 0;
  a.bias_sh = n * n;
  a.bias_sq = n;
  a.bias_batched = 0;
  a.out = w.o;
  a.out_sb = n * c;
  a.out_sh = d;
  a.out_sq = c;
  a.gate = w.g;
  a.gate_sb = a.out_sb;
  a.gate_sh = a.out_sh;
  a.gate_sq = a.out_sq;
  XFB_TRY(run_flash(dp, XFB_BF16, pre, w.q, w.k, w.v, a, st));
  if (out_route != nullptr) {
    // the update of column block jj, pair row i, goes back to the owner of row i
    xfb::EpiRowsRouted<128> epi;
    epi.ld_out = c;
    epi.M = static_cast<int>(rows * n);
    epi.N = static_cast<int>(c);
    epi.route = 2;
    epi.rank = out_route->rank;
    epi.route_rows = static_cast<int>(rows);
    epi.route_batch = 0;
    epi.route_n = static_cast<int>(n);
    for (int s = 0; s < xfb::kMaxRoute; ++s)
      epi.dst[s] = s < out_route->world ? out_route->dst[s] : nullptr;
    return run_gemm<128, false, false>(w.o, c, 0, output_w, c, 0, rows * n, c, c, 1, epi, st);
  }
  return linear_core(w.o, rows * n, c, c, static_cast<const bf16*>(output_w), c, nullptr, nullptr,
                     0, out, out_dtype == XFB_F32, accumulate, c, st);
}
}  // namespace

XFB_API int xfb_grid_attention_rows(const void* x, int64_t rows, int64_t n, int64_t c,
                                    int64_t heads, const float* mask, const void* bias,
                                    const void* packed, const void* output_w, void* out,
                                    int out_dtype, int accumulate, void* workspace,
                                    int64_t workspace_bytes, void* stream) {
  return grid_attention_rows_impl(x, rows, n, c, heads, mask, bias, packed, output_w, out,
                                  out_dtype, accumulate, nullptr, workspace, workspace_bytes,
                                  stream);
}

XFB_API int xfb_grid_attention_rows_routed(const void* x, int64_t rows, int64_t n, int64_t c,
                                           int64_t heads, const float* mask, const void* bias,
                                           const void* packed, const void* output_w,
                                           void* const* out_dst, int world, int rank,
                                           void* workspace, int64_t workspace_bytes,
                                           void* stream) {
  XFB_TRY(check_route(out_dst, world, rank));
  XFB_REQUIRE(rows * world == n, "a routed row block holds n / world rows");
  const Route r{out_dst, world, rank};
  return grid_attention_rows_impl(x, rows, n, c, heads, mask, bias, packed, output_w,
                                  out_dst[rank], XFB_BF16, 0, &r, workspace, workspace_bytes,
                                  stream);
}

XFB_API int64_t xfb_grid_attention_core_workspace(int64_t rows, int64_t n) {
  Carver cv{nullptr, 0, 0};
  cv.take<uint32_t>(rows * mask_words(n));
  return cv.used;
}

XFB_API int xfb_grid_attention_core(const void* q, const void* k, const void* v, int64_t rows,
                                    int64_t heads, int64_t n, const float* mask, const void* bias,
                                    const void* gate, void* out, void* workspace,
                                    int64_t workspace_bytes, void* stream) {
  XFB_REQUIRE(rows >= 0 && n >= 0 && n % 8 == 0, "the attention core needs n % 8 == 0 tokens");
  XFB_REQUIRE(heads > 0 && heads <= 16, "heads must be in 1..16");
  XFB_REQUIRE(q && k && v && bias && out, "q, k, v, bias and out are required");
  if (rows == 0 || n == 0) return XFB_OK;
  XFB_REQUIRE(n <= 16384 && rows * n <= (1ll << 31) - 256, "row block too large");
  XFB_REQUIRE(aligned16(q) && aligned16(k) && aligned16(v) && aligned16(bias) && aligned16(out) &&
                  aligned16(gate),
              "attention core tensors must be 16-byte aligned");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  Carver cv{static_cast<uint8_t*>(workspace), 0, workspace_bytes};
  uint32_t* bits = mask ? cv.take<uint32_t>(rows * mask_words(n)) : nullptr;
  XFB_TRY(check_workspace(cv, workspace, workspace_bytes));
  const int64_t c = heads * 32;
  xfb::AttnArgs a;
  a.B = static_cast<int>(rows);
  a.H = static_cast<int>(heads);
  a.nq = static_cast<int>(n);
  a.nk = static_cast<int>(n);
  a.d = 32;
  if (mask != nullptr) XFB_TRY(launch_mask_bits(mask, true, rows, n, n, bits, st));
  a.mask_bits = bits;
  a.mask_sb = mask_words(n);
  a.bias = bias;
  a.bias_sb = 0;
  a.bias_sh = n * n;
  a.bias_sq = n;
  a.bias_batched = 0;
  a.out = static_cast<bf16*>(out);
  a.out_sb = n * c;
  a.out_sh = 32;
  a.out_sq = c;
  a.gate = static_cast<const bf16*>(gate);
  a.gate_sb = a.out_sb;
  a.gate_sh = a.out_sh;
  a.gate_sq = a.out_sq;
  return run_flash(32, XFB_BF16, true, static_cast<const bf16*>(q), static_cast<const bf16*>(k),
                   static_cast<const bf16*>(v), a, st);
}

XFB_API int xfb_pair_logits_rows(const void* pair, int pair_dtype, int64_t rows, int64_t n,
                                 int64_t c, int64_t heads, const float* norm_weight,
                                 const float* norm_bias, double eps, const void* w, void* logits,
                                 void* stream) {
  XFB_REQUIRE(rows >= 0 && n >= 0 && heads > 0 && heads <= 16, "pair logits expect 1..16 heads");
  XFB_REQUIRE(c == 64 || c == 128, "pair width must be 64 or 128");
  if (rows == 0 || n == 0) return XFB_OK;
  return run_layer_norm(pair, pair_dtype, rows * n, c, c, norm_weight, norm_bias, eps, nullptr, 0,
                        nullptr, nullptr, static_cast<const bf16*>(w), static_cast<int>(heads),
                        static_cast<bf16*>(logits), rows * n, static_cast<cudaStream_t>(stream));
}


XFB_API int xfb_exchange_copy(const xfb_copy_box* boxes, int count, void* stream) {
  XFB_REQUIRE(count >= 0 && count <= xfb::kMaxCopyBoxes, "exchange copy takes at most 16 boxes");
  XFB_REQUIRE(count == 0 || boxes != nullptr, "exchange copy boxes missing");
  xfb::CopyBoxes kb;
  memset(&kb, 0, sizeof(kb));
  kb.count = count;
  uint64_t largest = 0;
  for (int i = 0; i < count; ++i) {
    const xfb_copy_box& b = boxes[i];
    XFB_REQUIRE(b.d0 >= 0 && b.d1 >= 0 && b.d2_bytes >= 0, "exchange copy extents must be >= 0");
    XFB_REQUIRE(b.d2_bytes % 16 == 0 && b.src_stride0 % 16 == 0 && b.src_stride1 % 16 == 0 &&
                    b.dst_stride0 % 16 == 0 && b.dst_stride1 % 16 == 0,
                "exchange copy runs and strides must be multiples of 16 bytes");
    XFB_REQUIRE(b.src_stride0 >= 0 && b.src_stride1 >= 0 && b.dst_stride0 >= 0 && b.dst_stride1 >= 0,
                "exchange copy strides must be non-negative");
    const uint64_t vecs = static_cast<uint64_t>(b.d0) * b.d1 * (b.d2_bytes / 16);
    XFB_REQUIRE(vecs == 0 || (aligned16(b.src) && aligned16(b.dst)),
                "exchange copy pointers must be 16-byte aligned");
    XFB_REQUIRE(static_cast<uint64_t>(b.d0) * b.d1 * (b.d2_bytes / 16) < (1ull << 32) - (1ull << 28),
                "exchange copy box too large (at most 2^32 - 2^28 vectors of 16 bytes)");
    xfb::CopyBox& k = kb.box[i];
    k.src = static_cast<const uint4*>(b.src);
    k.dst = static_cast<uint4*>(b.dst);
    k.d0 = static_cast<uint32_t>(b.d0);
    k.d1 = static_cast<uint32_t>(b.d1);
    k.d2 = static_cast<uint32_t>(b.d2_bytes / 16);
    k.s0 = b.src_stride0 / 16;
    k.s1 = b.src_stride1 / 16;
    k.t0 = b.dst_stride0 / 16;
    k.t1 = b.dst_stride1 / 16;
    largest = std::max(largest, vecs);
  }
  if (largest == 0) return XFB_OK;
  int sms;
  XFB_TRY(sm_count(&sms));
  const uint64_t want = (largest + 1023) / 1024;  // four vectors per thread
  const uint64_t cap = std::max<uint64_t>(1, static_cast<uint64_t>(sms) * 8 / count);
  dim3 grid(static_cast<unsigned>(std::min(want, cap)), count);
  xfb::exchange_copy_kernel<<<grid, 256, 0, static_cast<cudaStream_t>(stream)>>>(kb);
  XFB_LAUNCHED();
  return XFB_OK;
}


// ---------------------------------------------------------------- CUDA IPC for exchanges

XFB_API int64_t xfb_ipc_handle_bytes(void) { return sizeof(cudaIpcMemHandle_t); }

XFB_API int xfb_ipc_handle(const void* ptr, void* handle, int64_t* offset) {
  XFB_REQUIRE(ptr != nullptr && handle != nullptr && offset != nullptr, "ipc handle arguments missing");
  static PFN_cuMemGetAddressRange_v3020 range_fn = nullptr;
  static std::once_flag once;
  std::call_once(once, []() {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &fn, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      range_fn = reinterpret_cast<PFN_cuMemGetAddressRange_v3020>(fn);
  });
  XFB_REQUIRE(range_fn != nullptr, "cuMemGetAddressRange is unavailable");
  CUdeviceptr base = 0;
  size_t size = 0;
  if (range_fn(&base, &size, reinterpret_cast<CUdeviceptr>(ptr)) != CUDA_SUCCESS)
    return fail(XFB_ERR_CUDA, "cuMemGetAddressRange failed for the exchange buffer");
  cudaIpcMemHandle_t h;
  XFB_CUDA(cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(base)));
  memcpy(handle, &h, sizeof(h));
  *offset = static_cast<int64_t>(reinterpret_cast<uintptr_t>(ptr) - static_cast<uintptr_t>(base));
  return XFB_OK;
}

XFB_API int xfb_ipc_open(const void* handle, int64_t offset, void** peer_ptr) {
  XFB_REQUIRE(handle != nullptr && peer_ptr != nullptr && offset >= 0, "ipc open arguments missing");
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  void* base = nullptr;
  XFB_CUDA(cudaIpcOpenMemHandle(&base, h, cudaIpcMemLazyEnablePeerAccess));
  *peer_ptr = static_cast<uint8_t*>(base) + offset;
  return XFB_OK;
}

XFB_API int xfb_ipc_close(void* peer_ptr, int64_t offset) {
  XFB_REQUIRE(peer_ptr != nullptr && offset >= 0, "ipc close arguments missing");
  XFB_CUDA(cudaIpcCloseMemHandle(static_cast<uint8_t*>(peer_ptr) - offset));
  return XFB_OK;
}


// ---------------------------------------------------------------- diffusion conditioning

XFB_API int xfb_conditioning(const void* x, int64_t m, int64_t k, const void* weight, int64_t n,
                             const float* bias, int64_t chunk, int sig_mode, void* out,
                             void* stream) {
  XFB_REQUIRE(m >= 0 && k > 0 && n >= 0, "conditioning expects m, n >= 0 and k > 0");
  XFB_REQUIRE(k % 8 == 0, "conditioning input width must be a multiple of 8");
  XFB_REQUIRE(chunk > 0 && chunk % 64 == 0 && n % chunk == 0,
              "conditioning chunks must be multiples of 64 columns that divide n");
  XFB_REQUIRE(sig_mode >= 0 && sig_mode <= 2, "sig_mode must be 0, 1 or 2");
  XFB_REQUIRE(aligned16(x) && aligned16(weight) && aligned16(out) &&
                  (bias == nullptr || aligned16(bias)),
              "conditioning buffers must be 16-byte aligned");
  XFB_REQUIRE(m * n < (1ll << 40) && m < (1 << 30) && n < (1 << 30), "conditioning too large");
  if (m == 0 || n == 0) return XFB_OK;
  xfb::EpiCondTma<128> epi;
  XFB_TRY(make_out_map(&epi.out_map, out, false, chunk, m, n / chunk, chunk, m * chunk));
  epi.bias = bias;
  epi.accumulate = 0;
  epi.chunk = static_cast<int>(chunk);
  epi.sig_mode = sig_mode;
  return run_gemm<128, false, false>(x, k, 0, weight, k, 0, m, n, k, 1, epi,
                                     static_cast<cudaStream_t>(stream));
}

// ---------------------------------------------------------------- atom cross-attention

XFB_API int xfb_cross_pair_logits(const void* pair_cond, int pair_dtype, int64_t subsets,
                                  int64_t nq, int64_t nk, int64_t c, int64_t blocks,
                                  int64_t heads, const float* norm_weight, const float* norm_bias,
                                  double eps, const void* w, void* logits, void* stream) {
  XFB_REQUIRE(pair_dtype == XFB_F32 || pair_dtype == XFB_BF16, "pair conditioning must be f32 or bf16");
  XFB_REQUIRE(subsets >= 0 && nq > 0 && nk > 0, "cross pair logits expect subsets >= 0, nq, nk > 0");
  XFB_REQUIRE(c == 16, "cross pair logits take 16 pair-conditioning channels");
  XFB_REQUIRE(blocks > 0 && heads > 0 && blocks * heads <= 16, "blocks * heads must be 1..16");
  XFB_REQUIRE(std::isfinite(eps) && eps >= 0, "LayerNorm eps must be finite and non-negative");
  XFB_REQUIRE(w != nullptr && logits != nullptr, "projection weight and output required");
  XFB_REQUIRE(aligned16(pair_cond), "pair conditioning must be 16-byte aligned");
  const int64_t pairs = nq * nk;
  XFB_REQUIRE(pairs < (1 << 30), "window too large");
  if (subsets == 0) return XFB_OK;
  int sms;
  XFB_TRY(sm_count(&sms));
  const int64_t total = subsets * pairs;
  const int grid = static_cast<int>(std::min<int64_t>((total + 255) / 256, int64_t(sms) * 8));
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (pair_dtype == XFB_F32) {
    xfb::cross_pair_logits_kernel<float><<<grid, 256, 0, st>>>(
        static_cast<const float*>(pair_cond), subsets, static_cast<int>(pairs),
        static_cast<int>(heads), static_cast<int>(blocks * heads), norm_weight, norm_bias,
        static_cast<float>(eps), static_cast<const bf16*>(w), static_cast<bf16*>(logits));
  } else {
    xfb::cross_pair_logits_kernel<bf16><<<grid, 256, 0, st>>>(
        static_cast<const bf16*>(pair_cond), subsets, static_cast<int>(pairs),
        static_cast<int>(heads), static_cast<int>(blocks * heads), norm_weight, norm_bias,
        static_cast<float>(eps), static_cast<const bf16*>(w), static_cast<bf16*>(logits));
  }
  XFB_LAUNCHED();
  return XFB_OK;
}

namespace {
struct CaWs {
  bf16 *xq, *xk, *qg, *kv, *o;
  float* bias;
};
void ca_layout(Carver& cv, int64_t subsets, CaWs* w) {
  const int64_t mq = subsets * xfb::kWinQ, mk = subsets * xfb::kWinK;
  w->xq = cv.take<bf16>(mq * xfb::kWinC);
  w->xk = cv.take<bf16>(mk * xfb::kWinC);
  w->qg = cv.take<bf16>(mq * 2 * xfb::kWinC);
  w->kv = cv.take<bf16>(mk * 2 * xfb::kWinC);
  w->o = cv.take<bf16>(mq * xfb::kWinC);
  w->bias = cv.take<float>(2 * xfb::kWinC);
}
}  // namespace

XFB_API int64_t xfb_cross_attention_workspace(int64_t subsets) {
  if (subsets <= 0) return 0;
  Carver cv{nullptr, 0, 0};
  CaWs w;
  ca_layout(cv, subsets, &w);
  return cv.used;
}

XFB_API int xfb_cross_attention(
    const void* x_q, int x_dtype, int64_t subsets, int64_t nq, int64_t nk, int64_t c,
    int64_t heads, const void* x_k, const int64_t* key_index, const uint8_t* key_valid,
    int64_t source_rows, const float* mask_q, const float* mask_k, const void* pair_logits,
    double eps, const void* q_mod_scale, const void* q_mod_shift, const void* k_mod_scale,
    const void* k_mod_shift, const void* packed, const float* q_bias, const void* wo,
    const void* out_gate, void* out, int out_dtype, int accumulate, void* workspace,
    int64_t workspace_bytes, void* stream) {
  XFB_REQUIRE(x_dtype == XFB_F32 || x_dtype == XFB_BF16, "activations must be f32 or bf16");
  XFB_REQUIRE(subsets >= 0, "subset count must be non-negative");
  XFB_REQUIRE(nq == xfb::kWinQ && nk == xfb::kWinK && c == xfb::kWinC && heads == xfb::kWinH,
              "cross-attention windows are 32 queries x 128 keys, c = 128, 4 heads");
  XFB_REQUIRE(out_dtype == XFB_F32 || out_dtype == XFB_BF16, "output must be f32 or bf16");
  XFB_REQUIRE(!accumulate || out_dtype == XFB_F32, "accumulate requires an f32 output");
  XFB_REQUIRE(packed != nullptr && wo != nullptr, "attention weights missing");
  XFB_REQUIRE(key_index != nullptr ? source_rows >= 0 : x_k != nullptr,
              "keys need either x_k or a gather index");
  XFB_REQUIRE((q_mod_scale == nullptr) == (q_mod_shift == nullptr) &&
                  (k_mod_scale == nullptr) == (k_mod_shift == nullptr),
              "modulation needs both scale and shift");
  XFB_REQUIRE(std::isfinite(eps) && eps >= 0, "LayerNorm eps must be finite and non-negative");
  XFB_REQUIRE(aligned16(x_q) && (x_k == nullptr || aligned16(x_k)) && aligned16(packed) &&
                  aligned16(wo) && aligned16(out) &&
                  (pair_logits == nullptr || aligned16(pair_logits)) &&
                  (out_gate == nullptr || aligned16(out_gate)),
              "cross-attention buffers must be 16-byte aligned");
  if (subsets == 0) return XFB_OK;
  XFB_REQUIRE(subsets < (1 << 24), "too many subsets");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  Carver cv{static_cast<uint8_t*>(workspace), 0, workspace_bytes};
  CaWs w;
  ca_layout(cv, subsets, &w);
  XFB_TRY(check_workspace(cv, workspace, workspace_bytes));
  const int64_t mq = subsets * nq, mk = subsets * nk;
  const bf16* wcat = static_cast<const bf16*>(packed);  // rows: q | gate | k | v
  // AdaLN of the queries and of the keys (gathered from the queries' rows)
  XFB_TRY(run_layer_norm(x_q, x_dtype, mq, c, c, nullptr, nullptr, eps, w.xq, c,
                         static_cast<const bf16*>(q_mod_scale), static_cast<const bf16*>(q_mod_shift),
                         nullptr, 0, nullptr, 0, st));
  if (key_index != nullptr) {
    XFB_TRY(run_layer_norm(x_q, x_dtype, mk, c, c, nullptr, nullptr, eps, w.xk, c,
                           static_cast<const bf16*>(k_mod_scale),
                           static_cast<const bf16*>(k_mod_shift), nullptr, 0, nullptr, 0, st, 1.f,
                           key_index, key_valid, source_rows));
  } else {
    XFB_TRY(run_layer_norm(x_k, x_dtype, mk, c, c, nullptr, nullptr, eps, w.xk, c,
                           static_cast<const bf16*>(k_mod_scale),
                           static_cast<const bf16*>(k_mod_shift), nullptr, 0, nullptr, 0, st));
  }
  // [q + q_bias | gate] and [k | v]
  XFB_CUDA(cudaMemsetAsync(w.bias, 0, 2 * c * sizeof(float), st));
  if (q_bias != nullptr)
    XFB_CUDA(cudaMemcpyAsync(w.bias, q_bias, c * sizeof(float), cudaMemcpyDeviceToDevice, st));
  XFB_TRY(linear_core(w.xq, mq, c, c, wcat, 2 * c, w.bias, nullptr, 0, w.qg, 0, 0, 2 * c, st));
  XFB_TRY(linear_core(w.xk, mk, c, c, wcat + 2 * c * c, 2 * c, nullptr, nullptr, 0, w.kv, 0, 0,
                      2 * c, st));
  {
    XFB_TRY(set_smem(xfb::window_attention_kernel, xfb::WinSmem::kLaunchBytes));
    xfb::WindowAttnArgs a;
    const uint64_t kv_dims[2] = {static_cast<uint64_t>(2 * c), static_cast<uint64_t>(mk)};
    const uint64_t kv_strides[1] = {static_cast<uint64_t>(2 * c * sizeof(bf16))};
    const uint32_t kv_box[2] = {64u, static_cast<uint32_t>(nk)};
    XFB_TRY(make_map_nd(&a.kv_map, false, 2, w.kv, kv_dims, kv_strides, kv_box,
                        CU_TENSOR_MAP_SWIZZLE_128B));
    a.qg = w.qg;
    a.bias = static_cast<const bf16*>(pair_logits);
    a.mask_q = mask_q;
    a.mask_k = mask_k;
    a.out = w.o;
    a.q_scale = 1.f / std::sqrt(static_cast<float>(c / heads));
    xfb::window_attention_kernel<<<static_cast<unsigned>(subsets), xfb::kWinThreads,
                                   xfb::WinSmem::kLaunchBytes, st>>>(a);
    XFB_LAUNCHED();
  }
  return linear_core(w.o, mq, c, c, static_cast<const bf16*>(wo), c, nullptr,
                     static_cast<const bf16*>(out_gate), c, out, out_dtype == XFB_F32, accumulate,
                     c, st);
}

// ---------------------------------------------------------------- MSA attention

namespace {
struct MsaWs {
  bf16 *x, *vt, *gt, *logits, *weights, *ot, *o, *wvg;
  float* kmask;
};
void msa_layout(Carver& cv, int64_t s, int64_t n, MsaWs* w) {
  const int64_t rows = s * n;
  w->x = cv.take<bf16>(rows * 64);
  w->vt = cv.take<bf16>(rows * 64);
  w->gt = cv.take<bf16>(rows * 64);
  w->logits = cv.take<bf16>(8 * n * n);
  w->weights = cv.take<bf16>(8 * n * n);
  w->ot = cv.take<bf16>(rows * 64);
  w->o = cv.take<bf16>(rows * 64);
  w->wvg = cv.take<bf16>(128 * 64);
  w->kmask = cv.take<float>(n);
}
}  // namespace

XFB_API int64_t xfb_msa_attention_workspace(int64_t s, int64_t n) {
  if (s <= 0 || n <= 0) return 0;
  Carver cv{nullptr, 0, 0};
  MsaWs w;
  msa_layout(cv, s, n, &w);
  return cv.used;
}

XFB_API int xfb_msa_attention(const void* msa, int msa_dtype, int64_t s, int64_t n,
                              int64_t c_msa, const float* msa_mask, const void* pair,
                              int pair_dtype, int64_t c_pair, int64_t heads,
                              const float* act_norm_w, const float* act_norm_b,
                              const float* pair_norm_w, const float* pair_norm_b, double eps,
                              const void* pair_logits_w, const void* v_w, const void* gate_w,
                              const void* out_w, void* out, int out_dtype, int accumulate,
                              void* workspace, int64_t workspace_bytes, void* stream) {
  XFB_REQUIRE(msa_dtype == XFB_F32 || msa_dtype == XFB_BF16, "msa must be f32 or bf16");
  XFB_REQUIRE(pair_dtype == XFB_F32 || pair_dtype == XFB_BF16, "pair must be f32 or bf16");
  XFB_REQUIRE(s >= 0 && n >= 0, "sizes must be non-negative");
  XFB_REQUIRE(c_msa == 64 && heads == 8 && c_pair == 128,
              "MSA attention takes c_msa = 64, 8 heads of 8, c_pair = 128");
  XFB_REQUIRE(n % 8 == 0, "the token count must be a multiple of 8");
  XFB_REQUIRE(out_dtype == XFB_F32 || out_dtype == XFB_BF16, "output must be f32 or bf16");
  XFB_REQUIRE(!accumulate || out_dtype == XFB_F32, "accumulate requires an f32 output");
  XFB_REQUIRE(pair_logits_w && v_w && gate_w && out_w, "MSA attention weights missing");
  XFB_REQUIRE(std::isfinite(eps) && eps >= 0, "LayerNorm eps must be finite and non-negative");
  XFB_REQUIRE(aligned16(msa) && aligned16(pair) && aligned16(out) && aligned16(v_w) &&
                  aligned16(gate_w) && aligned16(out_w),
              "MSA attention buffers must be 16-byte aligned");
  if (s == 0 || n == 0) return XFB_OK;
  XFB_REQUIRE(s * n < (1ll << 31) - 256 && n <= 16384, "MSA too large");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  Carver cv{static_cast<uint8_t*>(workspace), 0, workspace_bytes};
  MsaWs w;
  msa_layout(cv, s, n, &w);
  XFB_TRY(check_workspace(cv, workspace, workspace_bytes));
  const int64_t rows = s * n;
  int sms;
  XFB_TRY(sm_count(&sms));
  // normalised MSA, rows reordered (token, sequence)
  XFB_TRY(run_layer_norm(msa, msa_dtype, rows, 64, 64, act_norm_w, act_norm_b, eps, w.x, 64,
                         nullptr, nullptr, nullptr, 0, nullptr, 0, st, 1.f, nullptr, nullptr, 0,
                         s, n));
  // v | gate projection, head-major outputs
  XFB_CUDA(cudaMemcpyAsync(w.wvg, v_w, 64 * 64 * sizeof(bf16), cudaMemcpyDeviceToDevice, st));
  XFB_CUDA(cudaMemcpyAsync(w.wvg + 64 * 64, gate_w, 64 * 64 * sizeof(bf16),
                           cudaMemcpyDeviceToDevice, st));
  {
    xfb::EpiMsaVG epi;
    epi.vt = w.vt;
    epi.gt = w.gt;
    epi.M = rows;
    XFB_TRY((run_gemm<128, false, false>(w.x, 64, 0, w.wvg, 64, 0, rows, 128, 64, 1, epi, st)));
  }
  // pair logits [8][n][n] (LayerNorm of the pair and the head projection)
  XFB_TRY(run_layer_norm(pair, pair_dtype, n * n, 128, 128, pair_norm_w, pair_norm_b, eps,
                         nullptr, 0, nullptr, nullptr, static_cast<const bf16*>(pair_logits_w), 8,
                         w.logits, n * n, st));
  // key mask and the shared softmax weights
  const float* kmask = nullptr;
  if (msa_mask != nullptr) {
    xfb::msa_key_mask_kernel<<<static_cast<unsigned>((n + 31) / 32), 1024, 0, st>>>(msa_mask, s, n,
                                                                                  w.kmask);
    XFB_LAUNCHED();
    kmask = w.kmask;
  }
  {
    const int grid = static_cast<int>(std::min<int64_t>((8 * n + 7) / 8, sms * 8));
    xfb::msa_softmax_kernel<<<grid, 256, 0, st>>>(w.logits, kmask, 8 * n, n, w.weights);
    XFB_LAUNCHED();
  }
  // weighted average per head: ot[h] = (weights[h] @ vt[h]) * gt[h], [n][s*8]
  {
    xfb::EpiOutGated<128, false> epi;
    XFB_TRY(make_out_map(&epi.out_map, w.ot, false, s * 8, n, 8, s * 8, n * s * 8));
    const uint64_t dims[3] = {static_cast<uint64_t>(s * 8), static_cast<uint64_t>(n), 8};
    const uint64_t strides[2] = {static_cast<uint64_t>(s * 16), static_cast<uint64_t>(n * s * 16)};
    const uint32_t box[3] = {64, 128, 1};
    XFB_TRY(make_map_nd(&epi.gate_map, false, 3, w.gt, dims, strides, box,
                        CU_TENSOR_MAP_SWIZZLE_128B));
    epi.bias = nullptr;
    epi.accumulate = 0;
    XFB_TRY((run_gemm<128, false, true>(w.weights, n, n * n, w.vt, s * 8, n * s * 8, n, s * 8, n,
                                        8, epi, st)));
  }
  {
    const int grid = static_cast<int>(std::min<int64_t>((rows + 255) / 256, sms * 8));
    xfb::msa_merge_heads_kernel<<<grid, 256, 0, st>>>(w.ot, s, n, w.o);
    XFB_LAUNCHED();
  }
  return linear_core(w.o, rows, 64, 64, static_cast<const bf16*>(out_w), 64, nullptr, nullptr, 0,
                     out, out_dtype == XFB_F32, accumulate, 64, st);
}

// ---------------------------------------------------------------- OuterProductMean

namespace {
constexpr int64_t kOpmChunkBytes = 64ll << 20;  // outer products of one chunk of rows i

int64_t opm_chunk_rows(int64_t n) {
  const int64_t r = kOpmChunkBytes / (n * 1024 * 2);
  return std::max<int64_t>(1, std::min<int64_t>(n, r));
}

struct OpmWs {
  bf16 *x, *wlr, *left, *right, *maskb, *outer;
  float* norm;
};
void opm_layout(Carver& cv, int64_t s, int64_t n, OpmWs* w) {
  const int64_t rows = s * n;
  w->x = cv.take<bf16>(rows * 64);
  w->wlr = cv.take<bf16>(64 * 64);
  w->left = cv.take<bf16>(rows * 32);
  w->right = cv.take<bf16>(rows * 32);
  w->maskb = cv.take<bf16>(rows);
  w->norm = cv.take<float>(n * n);
  w->outer = cv.take<bf16>(opm_chunk_rows(n) * n * 1024);
}
}  // namespace

XFB_API int64_t xfb_pack_outer_product_weight_bytes(int64_t c_out) { return c_out * 1024 * 2; }

XFB_API int xfb_pack_outer_product_weight(const void* output_w, int w_dtype, int64_t c_out,
                                          void* packed, void* stream) {
  XFB_REQUIRE(w_dtype == XFB_F32 || w_dtype == XFB_BF16, "output_w must be f32 or bf16");
  XFB_REQUIRE(c_out > 0 && output_w != nullptr && packed != nullptr, "bad outer-product weight");
  int sms;
  XFB_TRY(sm_count(&sms));
  const int grid = static_cast<int>(std::min<int64_t>((c_out * 1024 + 255) / 256, sms * 8));
  xfb::pack_opm_weight_kernel<<<grid, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      output_w, w_dtype == XFB_F32, c_out, static_cast<bf16*>(packed));
  XFB_LAUNCHED();
  return XFB_OK;
}

XFB_API int64_t xfb_outer_product_mean_workspace(int64_t s, int64_t n) {
  if (s <= 0 || n <= 0) return 0;
  Carver cv{nullptr, 0, 0};
  OpmWs w;
  opm_layout(cv, s, n, &w);
  return cv.used;
}

XFB_API int xfb_outer_product_mean(const void* msa, int msa_dtype, int64_t s, int64_t n,
                                   int64_t c_msa, const float* mask, const float* norm_w,
                                   const float* norm_b, double eps, const void* left_w,
                                   const void* right_w, const void* packed_output_w,
                                   const float* output_b, int64_t c_out, void* out,
                                   int accumulate, void* workspace, int64_t workspace_bytes,
                                   void* stream) {
  XFB_REQUIRE(msa_dtype == XFB_F32 || msa_dtype == XFB_BF16, "msa must be f32 or bf16");
  XFB_REQUIRE(s >= 0 && n >= 0, "sizes must be non-negative");
  XFB_REQUIRE(c_msa == 64 && c_out == 128, "outer product mean takes c_msa = 64, 32 outer "
                                           "channels and 128 outputs");
  XFB_REQUIRE(n % 8 == 0, "the token count must be a multiple of 8");
  XFB_REQUIRE(mask != nullptr && left_w && right_w && packed_output_w && output_b,
              "outer product mean needs the mask and every weight");
  XFB_REQUIRE(std::isfinite(eps) && eps >= 0, "LayerNorm eps must be finite and non-negative");
  XFB_REQUIRE(aligned16(msa) && aligned16(out) && aligned16(packed_output_w) &&
                  aligned16(left_w) && aligned16(right_w),
              "outer product mean buffers must be 16-byte aligned");
  if (s == 0 || n == 0) return XFB_OK;
  XFB_REQUIRE(s * n < (1ll << 31) - 256 && n * 32 < (1 << 30), "MSA too large");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  Carver cv{static_cast<uint8_t*>(workspace), 0, workspace_bytes};
  OpmWs w;
  opm_layout(cv, s, n, &w);
  XFB_TRY(check_workspace(cv, workspace, workspace_bytes));
  const int64_t rows = s * n;
  int sms;
  XFB_TRY(sm_count(&sms));
  XFB_TRY(run_layer_norm(msa, msa_dtype, rows, 64, 64, norm_w, norm_b, eps, w.x, 64, nullptr,
                         nullptr, nullptr, 0, nullptr, 0, st));
  XFB_CUDA(cudaMemcpyAsync(w.wlr, left_w, 32 * 64 * sizeof(bf16), cudaMemcpyDeviceToDevice, st));
  XFB_CUDA(cudaMemcpyAsync(w.wlr + 32 * 64, right_w, 32 * 64 * sizeof(bf16),
                           cudaMemcpyDeviceToDevice, st));
  {
    xfb::EpiOpmLR epi;
    epi.left = w.left;
    epi.right = w.right;
    epi.mask = mask;
    epi.M = rows;
    XFB_TRY((run_gemm<128, false, false>(w.x, 64, 0, w.wlr, 64, 0, rows, 64, 64, 1, epi, st)));
  }
  // overlap counts norm[i][j] = sum_a mask[a][i] mask[a][j] (exact in f32)
  {
    const int grid = static_cast<int>(std::min<int64_t>((rows + 255) / 256, sms * 8));
    xfb::f32_to_bf16_kernel<<<grid, 256, 0, st>>>(mask, rows, w.maskb);
    XFB_LAUNCHED();
    xfb::EpiOut<128, true> epi;
    XFB_TRY(make_out_map(&epi.out_map, w.norm, true, n, n, 1, n, 0));
    epi.bias = nullptr;
    epi.accumulate = 0;
    XFB_TRY((run_gemm<128, true, true>(w.maskb, n, 0, w.maskb, n, 0, n, n, s, 1, epi, st)));
  }
  const int64_t chunk = opm_chunk_rows(n);
  for (int64_t i0 = 0; i0 < n; i0 += chunk) {
    const int64_t ci = std::min(chunk, n - i0);
    {
      xfb::EpiOpmOuter epi;
      epi.outer = w.outer;
      epi.M = static_cast<int>(ci * 32);
      epi.N = static_cast<int>(n);
      XFB_TRY((run_gemm<256, true, true>(w.left + i0 * 32, n * 32, 0, w.right, n * 32, 0, ci * 32,
                                         n * 32, s, 1, epi, st)));
    }
    {
      xfb::EpiOpmOut epi;
      float* dst = static_cast<float*>(out) + i0 * n * c_out;
      XFB_TRY(make_out_map(&epi.out_map, dst, true, c_out, ci * n, 1, c_out, 0));
      epi.bias = output_b;
      epi.accumulate = accumulate;
      epi.norm = w.norm + i0 * n;
      epi.eps = 1e-3f;
      epi.M = static_cast<int>(ci * n);
      XFB_TRY((run_gemm<128, false, false>(w.outer, 1024, 0, packed_output_w, 1024, 0, ci * n,
                                           c_out, 1024, 1, epi, st)));
    }
  }
  return XFB_OK;
}

namespace {
int exchange_signal(void* const* peer_flags, int world, int rank, uint32_t epoch,
                    uint32_t* counter, void* stream) {
  XFB_REQUIRE(world > 0 && world <= xfb::kMaxPeers && rank >= 0 && rank < world,
              "exchange barrier takes 1..16 GPUs");
  XFB_REQUIRE(peer_flags != nullptr, "peer flag pointers missing");
  xfb::PeerFlags p;
  memset(&p, 0, sizeof(p));
  for (int s = 0; s < world; ++s) {
    XFB_REQUIRE(peer_flags[s] != nullptr && (reinterpret_cast<uintptr_t>(peer_flags[s]) & 3) == 0,
                "peer flag arrays must be 4-byte aligned device pointers");
    p.flags[s] = static_cast<uint32_t*>(peer_flags[s]);
  }
  p.world = world;
  p.rank = rank;
  p.epoch = epoch;
  p.counter = counter;
  xfb::exchange_signal_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(p);
  XFB_LAUNCHED();
  return XFB_OK;
}

int exchange_wait(const void* flags, int world, uint32_t epoch, const uint32_t* counter,
                  void* stream) {
  XFB_REQUIRE(world > 0 && world <= xfb::kMaxPeers, "exchange barrier takes 1..16 GPUs");
  XFB_REQUIRE(flags != nullptr && (reinterpret_cast<uintptr_t>(flags) & 3) == 0,
              "flag array must be a 4-byte aligned device pointer");
  xfb::exchange_wait_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint32_t*>(flags), world, epoch, counter);
  XFB_LAUNCHED();
  return XFB_OK;
}
}  // namespace

XFB_API int xfb_exchange_signal(void* const* peer_flags, int world, int rank, uint32_t epoch,
                                void* stream) {
  return exchange_signal(peer_flags, world, rank, epoch, nullptr, stream);
}

XFB_API int xfb_exchange_wait(const void* flags, int world, uint32_t epoch, void* stream) {
  return exchange_wait(flags, world, epoch, nullptr, stream);
}

XFB_API int xfb_exchange_signal_counted(void* const* peer_flags, int world, int rank,
                                        uint32_t* counter, void* stream) {
  XFB_REQUIRE(counter != nullptr && (reinterpret_cast<uintptr_t>(counter) & 3) == 0,
              "the epoch counter must be a 4-byte aligned device pointer");
  return exchange_signal(peer_flags, world, rank, 0, counter, stream);
}

XFB_API int xfb_exchange_wait_counted(const void* flags, int world, const uint32_t* counter,
                                      void* stream) {
  XFB_REQUIRE(counter != nullptr && (reinterpret_cast<uintptr_t>(counter) & 3) == 0,
              "the epoch counter must be a 4-byte aligned device pointer");
  return exchange_wait(flags, world, 0, counter, stream);
}

}  // extern "C"

// ====================================================================== af3_kernels-compatible ABI

namespace {

// The CPU tile sizes of the reference's native extension (block_size, M_BLK,
// N_BLK, query_block): validated like xsmm_size (positive, 32-bit), otherwise
// without effect -- the tile shapes of these kernels are fixed.
int check_cpu_block(int64_t b, const char* name) {
  if (b <= 0 || b > 0x7fffffff)
    return fail(XFB_ERR_INVALID, std::string(name) + " must be a positive 32-bit size");
  return XFB_OK;
}

int reject_vnni(int packed) {
  if (packed)
    return fail(XFB_ERR_INVALID,
                "VNNI2-packed weights are a CPU layout; pass the [in, out] weights "
                "(weights_packed = false)");
  return XFB_OK;
}

}  // namespace

extern "C" {

XFB_API int64_t xfb_af3_linear_workspace(int64_t k, int64_t n) {
  Carver cv{nullptr, 0, 0};
  cv.take<bf16>(n * k);
  return cv.used;
}

XFB_API int xfb_af3_linear(const void* x, int64_t m, int64_t k, const void* weight, int w_dtype,
                           int64_t n, const float* bias, int weight_packed, void* y, int y_dtype,
                           void* workspace, int64_t workspace_bytes, void* stream) {
  XFB_TRY(reject_vnni(weight_packed));
  XFB_REQUIRE(m >= 0 && k > 0 && n > 0, "linear expects m >= 0, k > 0, n > 0");
  XFB_REQUIRE(k % 8 == 0 && n % 8 == 0, "linear requires k and n to be multiples of 8");
  XFB_REQUIRE(y_dtype == XFB_F32 || y_dtype == XFB_BF16, "linear output must be f32 or bf16");
  XFB_REQUIRE(aligned16(x) && aligned16(y), "linear input and output must be 16-byte aligned");
  if (m == 0) return XFB_OK;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  Carver cv{static_cast<uint8_t*>(workspace), 0, workspace_bytes};
  bf16* w = cv.take<bf16>(n * k);
  XFB_TRY(check_workspace(cv, workspace, workspace_bytes));
  XFB_TRY(launch_pack(weight, nullptr, nullptr, nullptr, w_dtype, 3, n, k, n, w, st, 1));
  return linear_core(static_cast<const bf16*>(x), m, k, k, w, n, bias, nullptr, 0, y,
                     y_dtype == XFB_F32, 0, n, st);
}

XFB_API int64_t xfb_af3_gated_linear_unit_workspace(int64_t k, int64_t n) {
  Carver cv{nullptr, 0, 0};
  cv.take<bf16>(2 * n * k);
  return cv.used;
}

XFB_API int xfb_af3_gated_linear_unit(const void* x, int64_t m, int64_t k, const void* weight,
                                      int w_dtype, int64_t n, int64_t m_block, int64_t n_block,
                                      int weight_packed, void* y, void* workspace,
                                      int64_t workspace_bytes, void* stream) {
  XFB_TRY(reject_vnni(weight_packed));
  XFB_TRY(check_cpu_block(m_block, "M_BLK"));
  XFB_TRY(check_cpu_block(n_block, "N_BLK"));
  XFB_REQUIRE(m >= 0 && k > 0, "GLU expects m >= 0 and k > 0");
  XFB_REQUIRE(n > 0 && n % 64 == 0, "GLU hidden width must be a positive multiple of 64");
  XFB_REQUIRE(k % 8 == 0, "GLU input width must be a multiple of 8");
  XFB_REQUIRE(aligned16(x) && aligned16(y), "GLU input and output must be 16-byte aligned");
  if (m == 0) return XFB_OK;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  Carver cv{static_cast<uint8_t*>(workspace), 0, workspace_bytes};
  bf16* pk = cv.take<bf16>(2 * n * k);
  XFB_TRY(check_workspace(cv, workspace, workspace_bytes));
  XFB_TRY(launch_pack(weight, nullptr, nullptr, nullptr, w_dtype, 1, n, k, 2 * n, pk, st, 1));
  xfb::EpiGLU epi;
  XFB_TRY(make_out_map(&epi.out_map, y, false, n, m, 1, n, 0));
  return run_gemm<128, false, false>(x, k, 0, pk, k, 0, m, 2 * n, k, 1, epi, st);
}

XFB_API int64_t xfb_af3_triangle_multiplication_workspace(int64_t n, int64_t c) {
  Carver cv{nullptr, 0, 0};
  cv.take<bf16>(5 * c * c);  // packed projection | gate | gating_linear
  cv.take<bf16>(c * c);      // output_projection in [out][in]
  cv.take<uint8_t>(xfb_triangle_multiplication_workspace(n, c));
  return cv.used;
}

XFB_API int xfb_af3_triangle_multiplication(
    const void* pair, int pair_dtype, int64_t n, int64_t c, const float* mask, int outgoing,
    const float* left_weight, const float* left_bias, const void* projection, const void* gate,
    const float* center_weight, const float* center_bias, const void* output_weight,
    const void* gating_weight, int w_dtype, double left_eps, double center_eps,
    int64_t block_size, int weights_packed, void* out, int out_dtype, void* workspace,
    int64_t workspace_bytes, void* stream) {
  XFB_TRY(reject_vnni(weights_packed));
  XFB_TRY(check_cpu_block(block_size, "block_size"));
  XFB_REQUIRE(c == 64 || c == 128, "triangle multiplication supports c in {64, 128}");
  XFB_REQUIRE(projection && gate && output_weight && gating_weight, "triangle weights missing");
  XFB_REQUIRE(n >= 0, "pair side must be non-negative");
  if (n == 0) return XFB_OK;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  Carver cv{static_cast<uint8_t*>(workspace), 0, workspace_bytes};
  bf16* packed = cv.take<bf16>(5 * c * c);
  bf16* wo = cv.take<bf16>(c * c);
  const int64_t inner = xfb_triangle_multiplication_workspace(n, c);
  uint8_t* ws = cv.take<uint8_t>(inner);
  XFB_TRY(check_workspace(cv, workspace, workspace_bytes));
  XFB_TRY(launch_pack(projection, gate, gating_weight, nullptr, w_dtype, 0, c, c, 5 * c, packed,
                      st, 1));
  XFB_TRY(launch_pack(output_weight, nullptr, nullptr, nullptr, w_dtype, 3, c, c, c, wo, st, 1));
  return xfb_triangle_multiplication(pair, pair_dtype, n, c, mask, outgoing, left_weight,
                                     left_bias, nullptr, nullptr, center_weight, center_bias, wo,
                                     nullptr, left_eps, center_eps, 1, packed, out, out_dtype, 0,
                                     ws, inner, stream);
}

XFB_API int64_t xfb_af3_dot_product_attention_workspace(int64_t B, int64_t H, int64_t nq,
                                                        int64_t nk, int64_t d) {
  return xfb_dot_product_attention_workspace(B, H, nq, nk, d);
}

XFB_API int xfb_af3_dot_product_attention(const void* q, const void* k, const void* v, int64_t B,
                                          int64_t H, int64_t nq, int64_t nk, int64_t d,
                                          const void* mask, int mask_dtype, int mask_batched,
                                          const void* bias, int bias_dtype, int bias_batched,
                                          int64_t query_block, int q_pre_scaled, void* out,
                                          void* workspace, int64_t workspace_bytes,
                                          void* stream) {
  XFB_TRY(check_cpu_block(query_block, "query_block"));
  return xfb_dot_product_attention(q, k, v, B, H, nq, nk, d, mask, mask_dtype, mask_batched,
                                   bias, bias_dtype, bias_batched, q_pre_scaled, out, workspace,
                                   workspace_bytes, stream);
}

}  // extern "C"

// ---------------------------------------------------------------- float32 path

extern "C" {

XFB_API int xfb_f32_gemm(const xfb_f32_gemm_args* g, void* stream) {
  XFB_REQUIRE(g != nullptr, "gemm arguments missing");
  XFB_REQUIRE(g->m >= 0 && g->n >= 0 && g->k >= 0 && g->batch >= 0, "negative gemm extent");
  XFB_REQUIRE(g->act == 0 || g->act == 1, "act must be 0 (none) or 1 (sigmoid)");
  if (g->m == 0 || g->n == 0 || g->batch == 0) return XFB_OK;
  XFB_REQUIRE(g->a && g->b && g->c, "gemm operands missing");
  XFB_REQUIRE(g->m < (1ll << 31) && g->n < (1ll << 31) && g->k < (1ll << 31) &&
                  (g->m + 63) / 64 <= 65535 && g->batch <= 65535,
              "fp32 gemm too large");
  xfb::F32Gemm k;
  k.A = g->a;
  k.a_sb = g->a_sb;
  k.a_si = g->a_si;
  k.a_sk = g->a_sk;
  k.B = g->b;
  k.b_sb = g->b_sb;
  k.b_sj = g->b_sj;
  k.b_sk = g->b_sk;
  k.C = g->c;
  k.c_sb = g->c_sb;
  k.c_si = g->c_si;
  k.c_sj = g->c_sj;
  k.M = static_cast<int>(g->m);
  k.N = static_cast<int>(g->n);
  k.K = static_cast<int>(g->k);
  k.batch = static_cast<int>(g->batch);
  k.bias = g->bias;
  k.act = g->act;
  k.row_scale = g->row_scale;
  k.rs_sb = g->rs_sb;
  k.rs_si = g->rs_si;
  k.mul = g->mul;
  k.m_sb = g->mul_sb;
  k.m_si = g->mul_si;
  k.m_sj = g->mul_sj;
  k.accumulate = g->accumulate;
  const dim3 grid(static_cast<unsigned>((g->n + 63) / 64), static_cast<unsigned>((g->m + 63) / 64),
                  static_cast<unsigned>(g->batch));
  xfb::f32_gemm_kernel<<<grid, 256, 0, static_cast<cudaStream_t>(stream)>>>(k);
  XFB_LAUNCHED();
  return XFB_OK;
}

XFB_API int xfb_f32_layer_norm(const float* x, int64_t rows, int64_t cols, int64_t ldx,
                               const float* weight, const float* bias, double eps, float* y,
                               int64_t ldy, void* stream) {
  XFB_REQUIRE(rows >= 0 && cols > 0 && cols <= 1024, "fp32 LayerNorm takes 1..1024 columns");
  XFB_REQUIRE(std::isfinite(eps) && eps >= 0, "LayerNorm eps must be finite and non-negative");
  if (rows == 0) return XFB_OK;
  XFB_REQUIRE(x != nullptr && y != nullptr, "LayerNorm tensors missing");
  int sms;
  XFB_TRY(sm_count(&sms));
  const int blocks = static_cast<int>(std::min<int64_t>((rows + 7) / 8, int64_t(sms) * 8));
  xfb::f32_layer_norm_kernel<<<blocks, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      x, rows, static_cast<int>(cols), ldx, weight, bias, static_cast<float>(eps), y, ldy);
  XFB_LAUNCHED();
  return XFB_OK;
}

XFB_API int xfb_f32_attention(const xfb_f32_attention_args* a, void* stream) {
  XFB_REQUIRE(a != nullptr, "attention arguments missing");
  XFB_REQUIRE(a->batch >= 0 && a->heads >= 0 && a->nq >= 0 && a->nk >= 0, "negative extent");
  XFB_REQUIRE(a->d > 0 && a->d <= 64 && a->dv > 0 && a->dv <= 64, "head dims must be 1..64");
  if (a->batch == 0 || a->heads == 0 || a->nq == 0) return XFB_OK;
  XFB_REQUIRE(a->q && a->k && a->v && a->out, "attention tensors missing");
  XFB_REQUIRE(a->nk > 0, "attention over no keys");
  XFB_REQUIRE(a->batch * a->heads <= 65535 && a->nq < (1ll << 31) && a->nk < (1ll << 31),
              "fp32 attention too large");
  xfb::F32Attn k;
  k.q = a->q;
  k.q_sb = a->q_sb;
  k.q_sh = a->q_sh;
  k.q_si = a->q_si;
  k.k = a->k;
  k.k_sb = a->k_sb;
  k.k_sh = a->k_sh;
  k.k_si = a->k_si;
  k.v = a->v;
  k.v_sb = a->v_sb;
  k.v_sh = a->v_sh;
  k.v_si = a->v_si;
  k.bias = a->bias;
  k.bias_sb = a->bias_sb;
  k.bias_sh = a->bias_sh;
  k.bias_si = a->bias_si;
  k.mask = a->mask;
  k.mask_sb = a->mask_sb;
  k.out = a->out;
  k.o_sb = a->out_sb;
  k.o_sh = a->out_sh;
  k.o_si = a->out_si;
  k.gate = a->gate;
  k.g_sb = a->gate_sb;
  k.g_sh = a->gate_sh;
  k.g_si = a->gate_si;
  k.B = static_cast<int>(a->batch);
  k.H = static_cast<int>(a->heads);
  k.Q = static_cast<int>(a->nq);
  k.K = static_cast<int>(a->nk);
  k.d = static_cast<int>(a->d);
  k.dv = static_cast<int>(a->dv);
  k.scale = static_cast<float>(a->scale);
  const dim3 grid(static_cast<unsigned>((a->nq + xfb::kF32AttnWarps - 1) / xfb::kF32AttnWarps),
                  static_cast<unsigned>(a->batch * a->heads));
  xfb::f32_attention_kernel<<<grid, 32 * xfb::kF32AttnWarps, 0,
                              static_cast<cudaStream_t>(stream)>>>(k);
  XFB_LAUNCHED();
  return XFB_OK;
}

XFB_API int xfb_f32_silu_mul(const float* h, int64_t rows, int64_t f, float* y, void* stream) {
  XFB_REQUIRE(rows >= 0 && f > 0 && f < (1ll << 30), "silu_mul extents out of range");
  if (rows == 0) return XFB_OK;
  XFB_REQUIRE(h != nullptr && y != nullptr, "silu_mul tensors missing");
  int sms;
  XFB_TRY(sm_count(&sms));
  const int blocks = static_cast<int>(std::min<int64_t>((rows * f + 255) / 256, int64_t(sms) * 16));
  xfb::f32_silu_mul_kernel<<<blocks, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      h, rows, static_cast<int>(f), y);
  XFB_LAUNCHED();
  return XFB_OK;
}

XFB_API int xfb_f32_scale_shift(float* y, const float* scale, const float* shift, int64_t n,
                                void* stream) {
  XFB_REQUIRE(n >= 0, "negative length");
  if (n == 0) return XFB_OK;
  XFB_REQUIRE(y && scale && shift, "scale_shift tensors missing");
  int sms;
  XFB_TRY(sm_count(&sms));
  const int blocks = static_cast<int>(std::min<int64_t>((n + 255) / 256, int64_t(sms) * 16));
  xfb::f32_scale_shift_kernel<<<blocks, 256, 0, static_cast<cudaStream_t>(stream)>>>(y, scale,
                                                                                     shift, n);
  XFB_LAUNCHED();
  return XFB_OK;
}

}  // extern "C"

// ---------------------------------------------------------------- checkpoint upload

extern "C" {

XFB_API int xfb_gather_bytes(const void* src, int64_t src_bytes, void* dst, int64_t dst_bytes,
                             const int64_t* spans, const int64_t* host_spans, int64_t count,
                             void* stream) {
  XFB_REQUIRE(count >= 0, "negative record count");
  if (count == 0) return XFB_OK;
  XFB_REQUIRE(src && dst && spans && host_spans, "gather_bytes pointers missing");
  // the spans are checked on the host copy the caller also uploaded
  for (int64_t r = 0; r < count; ++r) {
    const int64_t so = host_spans[3 * r], dof = host_spans[3 * r + 1], nb = host_spans[3 * r + 2];
    XFB_REQUIRE(so >= 0 && nb >= 0 && so <= src_bytes - nb, "record outside the source blob");
    XFB_REQUIRE(dof >= 0 && dof % 4 == 0 && dof <= dst_bytes - nb,
                "record outside the arena or not 4-byte aligned");
  }
  int sms;
  XFB_TRY(sm_count(&sms));
  const int blocks = static_cast<int>(std::min<int64_t>(count, int64_t(sms) * 4));
  xfb::gather_bytes_kernel<<<blocks, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint8_t*>(src), static_cast<uint8_t*>(dst), spans, count);
  XFB_LAUNCHED();
  return XFB_OK;
}

}  // extern "C"
