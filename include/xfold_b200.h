/*
 * xfold_b200 — C ABI of the B200 (sm_100a) Pairformer / diffusion hot path.
 *
 * This is the drop-in boundary for xfold's `cuda` operator backend.  It
 * exposes the operators of the reference's native extension `af3_kernels._C`
 * (af3_kernels/src/csrc/bindings.cpp:10-49) with plain pointers, sizes and a
 * CUDA stream instead of ATen tensors, plus fused module-level entry points
 * (grid self-attention, transition, single/diffusion self-attention) that the
 * reference composes in Python.
 *
 * Conventions
 *   - All pointers are device pointers on the current CUDA device; `stream` is
 *     a cudaStream_t (NULL = legacy default stream).  Nothing synchronises.
 *   - Dtype codes: XFB_F32 = 0, XFB_BF16 = 1.
 *   - Weights are bf16 in nn.Linear layout [out_features][in_features]
 *     (K-major: what the tensor cores read).  The reference's bridge passes
 *     weight.T instead (xfold/fastnn/native.py:61); this ABI does not need the
 *     transposed copy.  LayerNorm weights/biases are f32 [C]; NULL bias = none,
 *     NULL weight = no affine.
 *   - `weights_packed` mirrors the reference's `weights_packed` /
 *     `weight_packed` flags: 0 = the separate nn.Linear weights are passed and
 *     packed into the workspace on every call; 1 = `packed` points to the
 *     buffer made once by the matching xfb_pack_* call (separate pointers
 *     ignored, may be NULL).
 *   - Scratch: each operator needs `xfb_*_workspace(...)` bytes of device
 *     memory passed as (workspace, workspace_bytes); it is not retained.
 *   - Outputs: `out` receives the update (accumulate = 0, the reference's
 *     "return the update only" contract, triangle_multiplication.cpp:71) or
 *     adds it into an f32 residual stream in place (accumulate = 1, the
 *     `pair += op(pair)` of xfold/nn/pairformer.py:96-100).
 *   - Return value: XFB_OK or an error code; xfb_last_error() describes the
 *     last failure of the calling thread.  XFB_ERR_INVALID is a shape / dtype /
 *     alignment error (the reference raises RuntimeError from TORCH_CHECK).
 */
#ifndef XFOLD_B200_H_
#define XFOLD_B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define XFB_API __attribute__((visibility("default")))

enum {
  XFB_OK = 0,
  XFB_ERR_INVALID = 1,   /* bad argument (shape, dtype, alignment, workspace too small) */
  XFB_ERR_CUDA = 2,      /* CUDA runtime / driver error (launch, tensor map) */
  XFB_ERR_DEVICE = 3,    /* device is not sm_100 */
  XFB_ERR_TIMEOUT = 4    /* a device-side bounded wait expired (see xfb_device_error) */
};

enum { XFB_F32 = 0, XFB_BF16 = 1, XFB_U8 = 2 };

/* Message for the last error returned on this thread ("" if none). */
XFB_API const char* xfb_last_error(void);

/* Number of kernels launched by this library so far (process-wide). */
XFB_API uint64_t xfb_launch_count(void);

/* JSON description of the build and device (arch, SM count, nvcc flags).
 * Counterpart of af3_kernels runtime_info() (bindings.cpp:13-20). */
XFB_API int xfb_runtime_info(char* buf, int64_t buf_len);

/* Preflight: the current device must be compute capability 10.0 and the
 * kernels must load.  Mirrors the native-backend checks of
 * run_alphafold.py:401-427 / xfold/fastnn/native.py:7-18. */
XFB_API int xfb_check_device(void);

/* Reads (and with clear != 0 resets) the device error word written by kernels
 * whose bounded waits expired.  Synchronises the device. */
XFB_API int xfb_device_error(int clear, uint32_t* code);

/* Self-test of the bounded-wait path: one thread waits on an mbarrier nothing
 * arrives on, gives up after `timeout_ns` and records code 0x1ff. */
XFB_API int xfb_selftest_wait_timeout(int64_t timeout_ns, void* stream);

/* ---------------------------------------------------------------- primitives */

/* y[rows][cols] (bf16) = LayerNorm(x) * weight + bias over the last dim.
 * cols in {64, 128, 384, 768}.  Replaces fastnn.LayerNorm
 * (xfold/fastnn/layer_norm.py:55-80).  x: f32 or bf16. */
XFB_API int xfb_layer_norm(const void* x, int x_dtype, int64_t rows, int64_t cols,
                           const float* weight, const float* bias, double eps, void* y,
                           void* stream);

/* y[m][n] = x[m][k] @ weight[n][k]^T (+ bias), bf16 in, f32 accumulate, output
 * rounded like an autocast linear.  y_dtype f32 or bf16; accumulate = 1 adds into
 * an f32 y.  Replaces af3_kernels linear (matrix.cpp:119-129).
 * Requires k % 8 == 0 and n % 8 == 0. */
XFB_API int xfb_linear(const void* x, int64_t m, int64_t k, const void* weight, int64_t n,
                       const float* bias, void* y, int y_dtype, int accumulate, void* stream);

/* Allocation-free variant of xfb_gated_linear_unit for callers that cannot
 * hand this library device memory: code that runs where cudaMalloc is not
 * allowed or not wanted (a host runtime that owns every device allocation
 * through its own pool and budget, or a service that must keep its footprint
 * fixed after start-up).  It has no counterpart in the reference.
 * `weight` is the unpacked transition1.weight [2n][k] (bf16); the packed copy
 * goes to a fixed scratch array built into the library (8 MiB per device,
 * held from load until exit), so 2*n*k must not exceed
 * XFB_GLU_NOALLOC_MAX_WEIGHT_ELEMS (larger weights are rejected with
 * XFB_ERR_INVALID).  No cudaMalloc / cudaFree happens.  The first call on a
 * device looks up the scratch's device address; make that first call before
 * any stream capture.  All calls share the one scratch array, so calls that
 * overlap on the GPU (other streams, other threads) race; each call rewrites
 * every scratch element it reads. */
#define XFB_GLU_NOALLOC_MAX_WEIGHT_ELEMS (4ll * 1024 * 1024)
XFB_API int xfb_gated_linear_unit_noalloc(const void* x, int64_t m, int64_t k, const void* weight,
                                          int64_t n, void* y, void* stream);

/* Batched GEMM, bf16 in, f32 accumulate: c[b][i][j] = sum_k A_b(i, k) B_b(j, k).
 * K-major operands: a [batch][m][k], b [batch][n][k]; MN-major (a_mn_major =
 * b_mn_major = 1): a [batch][k][m], b [batch][k][n].  c [batch][m][n], f32 or bf16.
 * Counterpart of af3_kernels gemm (bindings.cpp:26, tools.cpp); it is the
 * triangle contraction kernel on its own. */
XFB_API int xfb_gemm(const void* a, const void* b, void* c, int64_t batch, int64_t m, int64_t n,
                     int64_t k, int a_mn_major, int b_mn_major, int c_dtype, void* stream);

/* Packs transition1.weight [2n][k] (first n rows: SiLU gate) for the GLU kernel. */
XFB_API int64_t xfb_pack_glu_weight_bytes(int64_t n, int64_t k);
XFB_API int xfb_pack_glu_weight(const void* weight, int w_dtype, int64_t n, int64_t k,
                                void* packed, void* stream);

/* y[m][n] = silu(x @ W[:n]^T) * (x @ W[n:]^T), bf16.  weight = transition1.weight
 * [2n][k] (unpacked) or the packed buffer.  Replaces af3_kernels
 * gated_linear_unit (gated_linear_unit.cpp:78-121), whose weight is W^T [k][2n].
 * Requires n % 64 == 0, k % 8 == 0. */
XFB_API int64_t xfb_gated_linear_unit_workspace(int64_t m, int64_t k, int64_t n);
XFB_API int xfb_gated_linear_unit(const void* x, int64_t m, int64_t k, const void* weight,
                                  int64_t n, int weights_packed, void* y, void* workspace,
                                  int64_t workspace_bytes, void* stream);

/* ---------------------------------------------------------------- triangle multiplication */

/* Packed projection ‖ gate ‖ gating_linear weights for the fused input projection. */
XFB_API int64_t xfb_pack_triangle_weights_bytes(int64_t c);
XFB_API int xfb_pack_triangle_weights(const void* projection, const void* gate,
                                      const void* gating_linear, int w_dtype, int64_t c,
                                      void* packed, void* stream);

/* TriangleMultiplication update for pair [n][n][c] (f32 or bf16, contiguous):
 *   x = LN(pair); p = (x W_p^T) * mask * sigmoid(x W_g^T); a = p[..., 0::2], b = p[..., 1::2]
 *   z[c][i][j] = sum_k a[c][i][k] b[c][j][k]   (outgoing)
 *              = sum_k a[c][k][j] b[c][k][i]   (incoming)
 *   update = (LN_center(z) W_o^T) * sigmoid(x W_gl^T)
 * mask: f32 [n][n] or NULL.  Weights: projection, gate [2c][c]; output_weight,
 * gating_weight [c][c].  out: update (out_dtype f32/bf16, accumulate 0) or
 * pair += update (f32, accumulate 1).  c in {64, 128}.
 * Replaces af3_kernels triangle_multiplication (triangle_multiplication.cpp:6-73,
 * signature bindings.cpp:35-43) and TriangleMultiplication._forward_torch
 * (xfold/nn/triangle_multiplication.py:71-105). */
XFB_API int64_t xfb_triangle_multiplication_workspace(int64_t n, int64_t c);
XFB_API int xfb_triangle_multiplication(
    const void* pair, int pair_dtype, int64_t n, int64_t c, const float* mask, int outgoing,
    const float* left_weight, const float* left_bias, const void* projection, const void* gate,
    const float* center_weight, const float* center_bias, const void* output_weight,
    const void* gating_weight, double left_eps, double center_eps, int weights_packed,
    const void* packed, void* out, int out_dtype, int accumulate, void* workspace,
    int64_t workspace_bytes, void* stream);

/* ---------------------------------------------------------------- attention */

/* out[B][H][nq][dv] (bf16) = softmax(q k^T * d^-0.5 + bias, mask) v.
 * q [B][H][nq][d], k [B][H][nk][d], v [B][H][nk][d] bf16 contiguous, d = dv <= 64.
 * mask: key mask [B or 1][nk] (mask_dtype XFB_F32 or XFB_U8, nonzero = keep),
 *   mask_batched = 0 for a shared [nk] mask, or NULL; masked keys get logit -1e9.
 * bias: [B or 1][H][nq][nk] (bias_dtype f32 or bf16), bias_batched = 0 when shared
 *   across B, or NULL.
 * q_pre_scaled = 1 when q already carries the d^-0.5 factor (reference bridge,
 * xfold/fastnn/attention.py:21-29).  Replaces af3_kernels dot_product_attention
 * (dot_product_attention.cpp:110-174) and fastnn.dot_product_attention_torch
 * (xfold/fastnn/attention.py:45-66). */
XFB_API int64_t xfb_dot_product_attention_workspace(int64_t B, int64_t H, int64_t nq,
                                                    int64_t nk, int64_t d);
XFB_API int xfb_dot_product_attention(const void* q, const void* k, const void* v, int64_t B,
                                      int64_t H, int64_t nq, int64_t nk, int64_t d,
                                      const void* mask, int mask_dtype, int mask_batched,
                                      const void* bias, int bias_dtype, int bias_batched,
                                      int q_pre_scaled, void* out, void* workspace,
                                      int64_t workspace_bytes, void* stream);

/* Packed q ‖ k ‖ v ‖ gating_query weights [4c][c]. */
XFB_API int64_t xfb_pack_attention_weights_bytes(int64_t c);
XFB_API int xfb_pack_attention_weights(const void* q_w, const void* k_w, const void* v_w,
                                       const void* gate_w, int w_dtype, int64_t c,
                                       void* packed, void* stream);

/* GridSelfAttention update for pair [n][n][c] (triangle attention around the
 * starting node, transpose = 0, or the ending node, transpose = 1):
 *   x = LN(pair); bias[h][i][j] = x[i][j] . w_b[h]  (before any transpose)
 *   per batch row r: softmax(q k^T / sqrt(d) + bias, pair_mask[r][:]) v, gated by
 *   sigmoid(x W_gate^T), then output_projection.
 * mask: f32 [n][n] or NULL (row r is the key mask of batch row r in both
 * directions, as xfold/nn/attention.py:100).  bias_weight [heads][c].
 * c in {64, 128}, c / heads in {16, 32}.  Replaces GridSelfAttention.forward
 * (xfold/nn/attention.py:80-105). */
XFB_API int64_t xfb_grid_self_attention_workspace(int64_t n, int64_t c, int64_t heads);
XFB_API int xfb_grid_self_attention(
    const void* pair, int pair_dtype, int64_t n, int64_t c, int64_t heads, const float* mask,
    int transpose, const float* norm_weight, const float* norm_bias, double eps,
    const void* bias_weight, const void* q_w, const void* k_w, const void* v_w,
    const void* gate_w, const void* output_w, int weights_packed, const void* packed,
    void* out, int out_dtype, int accumulate, void* workspace, int64_t workspace_bytes,
    void* stream);

/* ---------------------------------------------------------------- transitions */

/* GLU transition x[rows][c] -> update (Transition, xfold/nn/primitives.py:33-37;
 * DiffusionTransition, xfold/nn/diffusion_transformer.py:124-128):
 *   y = LN(x) [* mod_scale + mod_shift]; h = silu(y W1[:fc]^T) * (y W1[fc:]^T);
 *   update = (h W2^T) [* out_gate]
 * w1 = transition1.weight [2fc][c] (or packed), w2 = transition2.weight [c][fc].
 * mod_scale / mod_shift / out_gate: bf16 [rows][c] or NULL (adaptive
 * conditioning, already passed through sigmoid where the reference does).
 * c in {64, 128, 384, 768}; f*c % 64 == 0. */
XFB_API int64_t xfb_transition_workspace(int64_t rows, int64_t c, int64_t factor);
XFB_API int xfb_transition(const void* x, int x_dtype, int64_t rows, int64_t c,
                           int64_t factor, const float* norm_weight, const float* norm_bias,
                           double eps, const void* mod_scale, const void* mod_shift,
                           const void* w1, int weights_packed, const void* w2,
                           const void* out_gate, void* out, int out_dtype, int accumulate,
                           void* workspace, int64_t workspace_bytes, void* stream);

/* ---------------------------------------------------------------- single attention */

/* SelfAttention with pair bias for x [n][c] (xfold/nn/diffusion_transformer.py:184-217):
 *   y = LN(x) [* mod_scale + mod_shift]; q = y Wq^T + q_bias, k, v, gate;
 *   o = softmax(q k^T / sqrt(d) + pair_logits, seq_mask) v * sigmoid(gate);
 *   update = (o Wo^T) [* out_gate]
 * pair_logits: bf16 [heads][n][n] or NULL; mask: f32 [n] or NULL;
 * packed = xfb_pack_attention_weights of (q, k, v, gating_query) when
 * weights_packed; wo = adaptive_zero_init.transition2.weight [c][c].
 * c in {128, 384, 768}, c / heads <= 64. */
XFB_API int64_t xfb_self_attention_workspace(int64_t n, int64_t c, int64_t heads);
XFB_API int xfb_self_attention(const void* x, int x_dtype, int64_t n, int64_t c, int64_t heads,
                               const float* mask, const void* pair_logits,
                               const float* norm_weight, const float* norm_bias, double eps,
                               const void* mod_scale, const void* mod_shift, const void* q_w,
                               const float* q_bias, const void* k_w, const void* v_w,
                               const void* gate_w, int weights_packed, const void* packed,
                               const void* wo, const void* out_gate, void* out, int out_dtype,
                               int accumulate, void* workspace, int64_t workspace_bytes,
                               void* stream);

/* Pair-logit projection for the single track (xfold/nn/pairformer.py:103-106):
 * logits[h][i][j] = LN(pair)[i][j] . w[h], bf16 [heads][n][n], heads <= 16. */
XFB_API int xfb_pair_logits(const void* pair, int pair_dtype, int64_t n, int64_t c,
                            int64_t heads, const float* norm_weight, const float* norm_bias,
                            double eps, const void* w, void* logits, void* stream);

/* ---- Row-block stages.  No counterpart in the reference, which runs every
 * operator on the whole pair inside one process.  These run the operators above
 * on a block of pair rows [rows][n][c] (n % 8 == 0) and stop exactly where a
 * row-sharded pair must exchange data between GPUs; xfold_cpu_b200/sharded.py
 * chains them with NCCL all-to-all / all-gather steps. */

/* TriMul stage 1 (xfold/nn/triangle_multiplication.py:71-95 on a row block):
 * x = LN(pair rows); a, b = channel-major [c][rows][n] bf16 (a = projection
 * channel 2k, b = 2k+1, masked and multiplied by the sigmoid gate); g = [rows][n][c]
 * bf16 output gate.  mask = [rows][n] f32 rows of the pair mask, or null; packed =
 * xfb_pack_triangle_weights.  Between stages 1 and 3 the contraction of a channel
 * shard is xfb_gemm: outgoing (a, b, both K-major), incoming (b, a, both MN-major). */
XFB_API int64_t xfb_triangle_projection_workspace(int64_t rows, int64_t n, int64_t c);
XFB_API int xfb_triangle_projection(const void* pair, int pair_dtype, int64_t rows, int64_t n,
                                    int64_t c, const float* mask, const float* left_weight,
                                    const float* left_bias, double left_eps, const void* packed,
                                    void* a, void* b, void* g, void* workspace,
                                    int64_t workspace_bytes, void* stream);

/* TriMul stage 3 (triangle_multiplication.py:96-105 on a row block): z = the
 * contraction for these rows, channel-major [c][rows][n] bf16; update =
 * (LN_c(z) W_o^T) * g -> out [rows][n][c] (accumulate: out f32 += update).  The
 * centre LayerNorm is folded into the projection GEMM (per-position statistics,
 * weights scaled by the LayerNorm weight); the workspace holds those statistics. */
XFB_API int64_t xfb_triangle_output_workspace(int64_t rows, int64_t n, int64_t c);
XFB_API int xfb_triangle_output(const void* z, int64_t rows, int64_t n, int64_t c, const void* g,
                                const float* center_weight, const float* center_bias,
                                double center_eps, const void* output_weight, void* out,
                                int out_dtype, int accumulate, void* workspace,
                                int64_t workspace_bytes, void* stream);

/* Grid attention stage 1 (xfold/nn/attention.py:86-98 on a row block):
 * x = LN(pair rows) bf16 [rows][n][c]; bias rows [heads][rows][n] bf16, multiplied
 * by log2(e) when c / heads == 32 and n % 8 == 0 (the units stage 2 expects). */
XFB_API int xfb_grid_attention_prepare(const void* pair, int pair_dtype, int64_t rows, int64_t n,
                                       int64_t c, int64_t heads, const float* norm_weight,
                                       const float* norm_bias, double eps, const void* bias_weight,
                                       void* x, void* bias, void* stream);

/* Grid attention stage 2 (attention.py:61-78 and 99-105 on a row block): q, k, v
 * and the gate from x rows; each row attends over its n tokens with bias
 * [heads][n][n] (stage 1 of every row block, assembled) and key mask [rows][n] f32
 * (or null); gated output projection -> out [rows][n][c].  packed =
 * xfb_pack_attention_weights.  For the ending node the caller passes the
 * transposed rows (columns of the pair) and the mask rows of those columns. */
XFB_API int64_t xfb_grid_attention_rows_workspace(int64_t rows, int64_t n, int64_t c,
                                                  int64_t heads);
XFB_API int xfb_grid_attention_rows(const void* x, int64_t rows, int64_t n, int64_t c,
                                    int64_t heads, const float* mask, const void* bias,
                                    const void* packed, const void* output_w, void* out,
                                    int out_dtype, int accumulate, void* workspace,
                                    int64_t workspace_bytes, void* stream);

/* Grid attention core (the softmax(q k^T + bias, mask) v, gated, of
 * xfold/nn/attention.py:61-78 for head dim 32), the kernel between the input
 * projections and the output projection of stage 2, for callers that hold the
 * projected operands:
 *   q, k, v [rows][heads][n][32] bf16, q already multiplied by
 *     log2(e) / sqrt(32) (scores in base-2 units); bias [heads][n][n] bf16 in
 *     base-2 units (multiplied by log2(e)), shared by every row;
 *   mask [rows][n] f32 key mask (0 = masked: logit -1e9) or null;
 *   gate [rows][n][heads*32] bf16 (already passed through sigmoid) or null;
 *   out [rows][n][heads*32] bf16 = gate * attention output.
 * n % 8 == 0.  No counterpart in the reference (it is one of this library's
 * row-block stages). */
XFB_API int64_t xfb_grid_attention_core_workspace(int64_t rows, int64_t n);
XFB_API int xfb_grid_attention_core(const void* q, const void* k, const void* v, int64_t rows,
                                    int64_t heads, int64_t n, const float* mask, const void* bias,
                                    const void* gate, void* out, void* workspace,
                                    int64_t workspace_bytes, void* stream);

/* Pair-logit projection (pairformer.py:103-106) of a row block:
 * logits [heads][rows][n] bf16. */
XFB_API int xfb_pair_logits_rows(const void* pair, int pair_dtype, int64_t rows, int64_t n,
                                 int64_t c, int64_t heads, const float* norm_weight,
                                 const float* norm_bias, double eps, const void* w, void* logits,
                                 void* stream);

/* Routed stages: the same arithmetic as the stages above, with the exchange
 * that follows each one done by the producer.  Instead of a local output the
 * kernel stores every row straight into the receive buffer of the rank that
 * needs it: dst[s] is rank s's buffer as mapped into this process (dst[rank]
 * is this GPU's own; a CUDA IPC mapping for the others), world <= 16 ranks,
 * this block = pair rows [rank * rows, (rank + 1) * rows) with rows * world =
 * n.  Stores are plain 16-byte stores (no TMA, no multicast) and the kernel
 * ends with a system-scope fence, so the caller's exchange barrier after it
 * (xfb_exchange_signal / xfb_exchange_wait) publishes them.  No counterpart in
 * the reference (it has no multi-GPU pair).
 *
 * xfb_triangle_projection_routed: as xfb_triangle_projection, but a and b
 * channel ch of pair row i go to rank s = ch / (c / world) as
 * a_dst[s] / b_dst[s] [c / world][n][n] at [ch % (c / world)][i][j] (the rows
 * -> channels exchange); g stays local. */
XFB_API int xfb_triangle_projection_routed(const void* pair, int pair_dtype, int64_t rows,
                                           int64_t n, int64_t c, const float* mask,
                                           const float* left_weight, const float* left_bias,
                                           double left_eps, const void* packed,
                                           void* const* a_dst, void* const* b_dst, int world,
                                           int rank, void* g, void* workspace,
                                           int64_t workspace_bytes, void* stream);

/* The TriMul contraction of this rank's channel shard a, b [cs][n][n] bf16
 * (outgoing z[c,i,j] = sum_k a[c,i,k] b[c,j,k]; incoming sum_k a[c,k,j]
 * b[c,k,i]; triangle_multiplication.py:34-36), row i of channel ch stored as
 * bf16 into rank s = i / (n / world) as z_dst[s] [world * cs][n / world][n] at
 * [rank * cs + ch][i % (n / world)] (the channels -> rows exchange). */
XFB_API int xfb_triangle_contraction_routed(const void* a, const void* b, int64_t cs, int64_t n,
                                            int outgoing, void* const* z_dst, int world, int rank,
                                            void* stream);

/* xfb_grid_attention_prepare with the ending node's transpose: the LayerNorm'd
 * row (i, j) goes to rank s = j / rows as x_dst[s] [rows][n][c] at
 * [j % rows][rank * rows + i] (attention.py:97-98); the bias rows stay local.
 * c = 128. */
XFB_API int xfb_grid_attention_prepare_routed(const void* pair, int pair_dtype, int64_t rows,
                                              int64_t n, int64_t c, int64_t heads,
                                              const float* norm_weight, const float* norm_bias,
                                              double eps, const void* bias_weight,
                                              void* const* x_dst, int world, int rank, void* bias,
                                              void* stream);

/* xfb_grid_attention_rows for the ending node with the transpose back: the bf16
 * update of column jj (this rank's rows of the transposed pair), pair row i,
 * goes to rank s = i / rows as out_dst[s] [rows][n][c] at [i % rows][rank *
 * rows + jj]; the owner adds it to its pair rows.  Workspace as
 * xfb_grid_attention_rows_workspace. */
XFB_API int xfb_grid_attention_rows_routed(const void* x, int64_t rows, int64_t n, int64_t c,
                                           int64_t heads, const float* mask, const void* bias,
                                           const void* packed, const void* output_w,
                                           void* const* out_dst, int world, int rank,
                                           void* workspace, int64_t workspace_bytes,
                                           void* stream);

/* Single-track attention of the query rows [row0, row0 + q_rows) of a
 * row-sharded Pairformer (pairformer.py:102-108 for those rows): LayerNorm and
 * the q / k / v / gate projections over all n tokens, attention of the query
 * rows against every key with their pair logits [heads][q_rows][n] bf16 (the
 * rows xfb_pair_logits_rows gives this rank, so the logits need no exchange),
 * gated output projection into out rows [row0, row0 + q_rows) (f32 with
 * accumulate = 1 adds into them).  packed as xfb_pack_attention_weights. */
XFB_API int64_t xfb_self_attention_rows_workspace(int64_t n, int64_t c, int64_t heads,
                                                  int64_t q_rows);
XFB_API int xfb_self_attention_rows(const void* x, int x_dtype, int64_t n, int64_t c,
                                    int64_t heads, int64_t row0, int64_t q_rows,
                                    const float* mask, const void* pair_logits,
                                    const float* norm_weight, const float* norm_bias, double eps,
                                    const void* packed, const float* q_bias, const void* wo,
                                    const void* out_gate, void* out, int out_dtype,
                                    int accumulate, void* workspace, int64_t workspace_bytes,
                                    void* stream);

/* One block of an exchange between GPUs of a row-sharded pair: copy
 * [d0][d1][d2_bytes] from src to dst with byte strides (runs of d2_bytes are
 * contiguous on both sides).  dst may be another GPU's receive buffer mapped
 * into this process by CUDA IPC; the copy uses plain 16-byte loads and stores
 * (every size, stride and pointer a multiple of 16 bytes). */
typedef struct {
  const void* src;
  void* dst;
  int64_t d0, d1, d2_bytes;
  int64_t src_stride0, src_stride1;
  int64_t dst_stride0, dst_stride1;
} xfb_copy_box;

/* Copies up to 16 boxes in one launch, ending with a system-scope fence so a
 * peer that synchronises with this stream afterwards (the caller's barrier)
 * sees every store.  No counterpart in the reference (it has no multi-GPU pair). */
XFB_API int xfb_exchange_copy(const xfb_copy_box* boxes, int count, void* stream);

/* Barrier after an exchange copy, without a collective call (no counterpart in
 * the reference).  xfb_exchange_signal writes `epoch` into slot `rank` of every
 * GPU's uint32 flag array (peer_flags[s]: GPU s's array as mapped here, world
 * <= 16) with system-scope release stores, ordered after the work already on
 * `stream`; xfb_exchange_wait makes `stream` wait until every slot of this
 * GPU's own array holds at least `epoch` (giving up after 2 s, with the
 * device error code 0x105).  Epochs increase by one per exchange. */
XFB_API int xfb_exchange_signal(void* const* peer_flags, int world, int rank, uint32_t epoch,
                                void* stream);
XFB_API int xfb_exchange_wait(const void* flags, int world, uint32_t epoch, void* stream);

/* The same barrier with the epoch kept on the device: `counter` is a uint32 in
 * this GPU's memory, zero before the first barrier; xfb_exchange_signal_counted
 * advances it and signals its new value, xfb_exchange_wait_counted waits for
 * that value.  Nothing of the barrier is a launch argument that changes from
 * one exchange to the next, so a stream segment of exchanges can be captured
 * into a CUDA graph and replayed (every rank must replay the same segments). */
XFB_API int xfb_exchange_signal_counted(void* const* peer_flags, int world, int rank,
                                        uint32_t* counter, void* stream);
XFB_API int xfb_exchange_wait_counted(const void* flags, int world, const uint32_t* counter,
                                      void* stream);

/* CUDA IPC for the exchange receive buffers (no counterpart in the reference).
 * xfb_ipc_handle: the IPC handle (xfb_ipc_handle_bytes() bytes) of the device
 * allocation holding ptr, and ptr's byte offset in it.  xfb_ipc_open: maps a
 * peer process's allocation on the current device with lazy peer access and
 * returns the address of the peer's ptr; xfb_ipc_close unmaps it. */
XFB_API int64_t xfb_ipc_handle_bytes(void);
XFB_API int xfb_ipc_handle(const void* ptr, void* handle, int64_t* offset);
XFB_API int xfb_ipc_open(const void* handle, int64_t offset, void** peer_ptr);
XFB_API int xfb_ipc_close(void* peer_ptr, int64_t offset);

/* Conditioning projections of one diffusion step, for every block at once:
 * out = act(x W^T + bias) bf16, where x [m][k] bf16 is the (LayerNorm'd) single
 * conditioning and W [n][k] bf16 stacks the blocks' AdaLN scale / shift weights
 * (LayerNorm weight folded in) or AdaLNZero gate weights.  The n columns are
 * written as n / chunk contiguous [m][chunk] tensors (chunk a multiple of 64
 * that divides n); act = sigmoid on every
 * chunk (sig_mode 2), on the even chunks (1) or none (0).  Replaces, per block,
 * AdaptiveLayerNorm's conditioning (xfold/nn/diffusion_transformer.py:51-62) and
 * AdaLNZero's gate (:85-94), which the reference recomputes for each block. */
XFB_API int xfb_conditioning(const void* x, int64_t m, int64_t k, const void* weight, int64_t n,
                             const float* bias, int64_t chunk, int sig_mode, void* out,
                             void* stream);

/* ---- Atom transformer: windowed cross-attention (DiffusionCrossAttTransformer,
 * xfold/nn/diffusion_transformer.py:275-411).  The reference computes these
 * with torch einsum; its native extension has no counterpart.
 *
 * xfb_cross_pair_logits: the transformer's cached pair logits (:376-380):
 * LayerNorm over the c = 16 channels of pair_cond [subsets][nq][nk][16]
 * (norm_bias may be null: the reference's LayerNorm has none), projection by
 * w [blocks*heads][16] bf16 (pair_logits_projection.weight, rows ordered
 * (block, head)), written bf16 as logits [blocks][subsets][heads][nq][nk]
 * (the reference's rearrange 'n q k (b h) -> b n h q k'). */
XFB_API int xfb_cross_pair_logits(const void* pair_cond, int pair_dtype, int64_t subsets,
                                  int64_t nq, int64_t nk, int64_t c, int64_t blocks,
                                  int64_t heads, const float* norm_weight, const float* norm_bias,
                                  double eps, const void* w, void* logits, void* stream);

/* xfb_cross_attention: CrossAttention.forward (:307-350) for subsets windows of
 * nq = 32 queries and nk = 128 keys, c = 128, 4 heads (the sizes the
 * reference's DiffusionCrossAttTransformer builds).
 *   x_q      [subsets*32][128] queries_act (f32 or bf16)
 *   keys     key_index != null: keys are rows of x_q (flattened, source_rows
 *            rows): key row r = x_q[key_index[r]] where key_valid[r] != 0 (or
 *            key_valid null), zeros elsewhere -- atom_layout.convert with the
 *            queries_to_keys GatherInfo (xfold/nn/atom_layout.py:88-160), fused
 *            into the keys' LayerNorm; an index outside [0, source_rows) reads
 *            zeros and sets the device error 0x106.  key_index == null: x_k
 *            [subsets*128][128] holds the keys.
 *   mask_q [subsets*32], mask_k [subsets*128] f32 (0 = masked) or null: the
 *            reference's bias 1e9 * !mask_q[q] * !mask_k[k] (:318-322) enters the
 *            logits before the pair logits.
 *   pair_logits [subsets][4][32][128] bf16 or null.
 *   q_mod_* / k_mod_* [rows][128] bf16: AdaLN sigmoid(scale) and shift of the
 *            q / k adaptive LayerNorms (no-affine LayerNorm, eps); null = plain.
 *   packed   [512][128] bf16: q_projection | gating_query | k_projection |
 *            v_projection weights (nn.Linear layout); q_bias [128] f32 or null.
 *   wo       [128][128] bf16 adaptive_zero_init.transition2.weight; out_gate
 *            [subsets*32][128] bf16 sigmoid(adaptive_zero_cond(single_cond_q))
 *            or null.
 *   out      [subsets*32][128]: the update (accumulate = 0) or added into an f32
 *            residual (accumulate = 1, the caller's queries_act += ...). */
XFB_API int64_t xfb_cross_attention_workspace(int64_t subsets);
XFB_API int xfb_cross_attention(
    const void* x_q, int x_dtype, int64_t subsets, int64_t nq, int64_t nk, int64_t c,
    int64_t heads, const void* x_k, const int64_t* key_index, const uint8_t* key_valid,
    int64_t source_rows, const float* mask_q, const float* mask_k, const void* pair_logits,
    double eps, const void* q_mod_scale, const void* q_mod_shift, const void* k_mod_scale,
    const void* k_mod_shift, const void* packed, const float* q_bias, const void* wo,
    const void* out_gate, void* out, int out_dtype, int accumulate, void* workspace,
    int64_t workspace_bytes, void* stream);

/* ---- Evoformer MSA stack (xfold/nn/pairformer.py:117-156).  The reference
 * runs these in torch (einsum); its native extension has no counterpart.
 *
 * xfb_msa_attention: MSAAttention.forward (xfold/nn/attention.py:125-144) for
 * msa [s][n][64] (f32 or bf16), msa_mask [s][n] f32 (null = all ones), pair
 * [n][n][128]: LayerNorms act_norm (64) and pair_norm (128) with eps,
 * pair_logits_w [8][128], v_w / gate_w / out_w [64][64] bf16 (nn.Linear
 * layout), 8 heads of 8.  The [8][n][n] softmax weights over keys (pair
 * logits + 1e9 (max_s mask - 1)) are shared by all s rows; out [s][n][64] is
 * the update (accumulate = 0) or added into an f32 msa (accumulate = 1).
 * n must be a multiple of 8. */
XFB_API int64_t xfb_msa_attention_workspace(int64_t s, int64_t n);
XFB_API int xfb_msa_attention(const void* msa, int msa_dtype, int64_t s, int64_t n,
                              int64_t c_msa, const float* msa_mask, const void* pair,
                              int pair_dtype, int64_t c_pair, int64_t heads,
                              const float* act_norm_w, const float* act_norm_b,
                              const float* pair_norm_w, const float* pair_norm_b, double eps,
                              const void* pair_logits_w, const void* v_w, const void* gate_w,
                              const void* out_w, void* out, int out_dtype, int accumulate,
                              void* workspace, int64_t workspace_bytes, void* stream);

/* xfb_outer_product_mean: OuterProductMean.forward (xfold/nn/primitives.py:62-75)
 * for msa [s][n][64], mask [s][n] f32: LayerNorm (norm_w, norm_b, eps),
 * left_w / right_w [32][64] bf16, output_w packed by
 * xfb_pack_outer_product_weight (from the [32][32][c_out] parameter), output_b
 * [c_out] f32, c_out = 128.  out [n][n][128] f32 receives the update
 * (accumulate = 0) or has it added (accumulate = 1, the caller's
 * pair += ...).  The outer products are formed one chunk of rows at a time
 * (64 MiB of workspace per chunk). */
XFB_API int64_t xfb_pack_outer_product_weight_bytes(int64_t c_out);
XFB_API int xfb_pack_outer_product_weight(const void* output_w, int w_dtype, int64_t c_out,
                                          void* packed, void* stream);
XFB_API int64_t xfb_outer_product_mean_workspace(int64_t s, int64_t n);
XFB_API int xfb_outer_product_mean(const void* msa, int msa_dtype, int64_t s, int64_t n,
                                   int64_t c_msa, const float* mask, const float* norm_w,
                                   const float* norm_b, double eps, const void* left_w,
                                   const void* right_w, const void* packed_output_w,
                                   const float* output_b, int64_t c_out, void* out,
                                   int accumulate, void* workspace, int64_t workspace_bytes,
                                   void* stream);

/* ---- af3_kernels-compatible entry points.  The argument lists of the
 * reference's native extension (af3_kernels/src/csrc/bindings.cpp:26-49) with
 * plain pointers: weights are the transposed nn.Linear weights [in][out] that
 * its bridges pass (xfold/fastnn/native.py:61, xfold/nn/triangle_multiplication.py:58-60),
 * f32 or bf16 (w_dtype); the CPU tile sizes (block_size, M_BLK, N_BLK,
 * query_block) must be positive 32-bit sizes, as xsmm_size requires
 * (af3_kernels/src/csrc/tools.cpp:30-34), and do not change results;
 * weights_packed = 1 (the CPU's VNNI2 layout) is rejected with
 * XFB_ERR_INVALID.  Computation is bf16 with f32 accumulation, as the other
 * entry points; each call packs its weights into the workspace. */

/* linear (matrix.cpp:119-129): y[m][n] = x[m][k] (bf16) @ weight[k][n] + bias,
 * bias f32 [n] or NULL, y f32 or bf16.  k, n multiples of 8. */
XFB_API int64_t xfb_af3_linear_workspace(int64_t k, int64_t n);
XFB_API int xfb_af3_linear(const void* x, int64_t m, int64_t k, const void* weight, int w_dtype,
                           int64_t n, const float* bias, int weight_packed, void* y, int y_dtype,
                           void* workspace, int64_t workspace_bytes, void* stream);

/* gated_linear_unit (gated_linear_unit.cpp:78-121): y[m][n] (bf16) =
 * silu(x @ weight[:, :n]) * (x @ weight[:, n:]) for x [m][k] bf16 and weight
 * [k][2n].  n a multiple of 64, k a multiple of 8. */
XFB_API int64_t xfb_af3_gated_linear_unit_workspace(int64_t k, int64_t n);
XFB_API int xfb_af3_gated_linear_unit(const void* x, int64_t m, int64_t k, const void* weight,
                                      int w_dtype, int64_t n, int64_t m_block, int64_t n_block,
                                      int weight_packed, void* y, void* workspace,
                                      int64_t workspace_bytes, void* stream);

/* triangle_multiplication (triangle_multiplication.cpp:6-73): the update for
 * pair [n][n][c] (f32 or bf16) with projection, gate [c][2c] and
 * output_weight, gating_weight [c][c]; mask f32 [n][n] (the reference's
 * broadcast to [N, N] done by the caller) or NULL.  out [n][n][c], f32 or bf16. */
XFB_API int64_t xfb_af3_triangle_multiplication_workspace(int64_t n, int64_t c);
XFB_API int xfb_af3_triangle_multiplication(
    const void* pair, int pair_dtype, int64_t n, int64_t c, const float* mask, int outgoing,
    const float* left_weight, const float* left_bias, const void* projection, const void* gate,
    const float* center_weight, const float* center_bias, const void* output_weight,
    const void* gating_weight, int w_dtype, double left_eps, double center_eps,
    int64_t block_size, int weights_packed, void* out, int out_dtype, void* workspace,
    int64_t workspace_bytes, void* stream);

/* dot_product_attention (dot_product_attention.cpp:110-174): xfb_dot_product_attention
 * with the reference's query_block argument. */
XFB_API int64_t xfb_af3_dot_product_attention_workspace(int64_t B, int64_t H, int64_t nq,
                                                        int64_t nk, int64_t d);
XFB_API int xfb_af3_dot_product_attention(const void* q, const void* k, const void* v, int64_t B,
                                          int64_t H, int64_t nq, int64_t nk, int64_t d,
                                          const void* mask, int mask_dtype, int mask_batched,
                                          const void* bias, int bias_dtype, int bias_batched,
                                          int64_t query_block, int q_pre_scaled, void* out,
                                          void* workspace, int64_t workspace_bytes,
                                          void* stream);

/* ------------------------------------------------------------------ float32 path
 * The reference's float32 route (no autocast: xfold/fastnn/native.py:31-43 keeps
 * fp32; torch matmul, LayerNorm and softmax in fp32) on the CUDA cores, for the
 * 1e-4 precision contract.  All tensors are float32; every operand is given by
 * strides in elements, so transposes, head splits and the triangle
 * multiplication's channel interleave need no copies. */

/* C[b](i, j) (=, or += with accumulate) ((act(sum_k A[b](i,k) B[b](j,k) + bias[j]))
 * * row_scale[b](i)) * mul[b](i, j); act 0 = none, 1 = sigmoid; null pointers
 * skip their step.  Replaces the fp32 matmuls / einsums of
 * triangle_multiplication.py:71-105, attention.py:61-105, primitives.py:33-37,
 * diffusion_transformer.py:51-217. */
typedef struct xfb_f32_gemm_args {
  const float* a;
  int64_t a_sb, a_si, a_sk;
  const float* b;
  int64_t b_sb, b_sj, b_sk;
  float* c;
  int64_t c_sb, c_si, c_sj;
  int64_t m, n, k, batch;
  const float* bias;
  int act;
  const float* row_scale;
  int64_t rs_sb, rs_si;
  const float* mul;
  int64_t mul_sb, mul_si, mul_sj;
  int accumulate;
} xfb_f32_gemm_args;
XFB_API int xfb_f32_gemm(const xfb_f32_gemm_args* args, void* stream);

/* LayerNorm over rows of cols <= 1024 fp32 values (fastnn/layer_norm.py:14-80,
 * F.layer_norm): weight / bias optional. */
XFB_API int xfb_f32_layer_norm(const float* x, int64_t rows, int64_t cols, int64_t ldx,
                               const float* weight, const float* bias, double eps, float* y,
                               int64_t ldy, void* stream);

/* out[b][h][i][:] = gate * softmax_k(q[b][h][i] . k[b][h][k] * scale + bias[b][h][i][k],
 * mask[b][k]) v[b][h][k][:] in fp32 (fastnn/attention.py:45-66): masked keys
 * (mask value 0) get -1e9 after the bias; rows of each tensor contiguous in the
 * head dimension (d, dv <= 64); strides of 0 broadcast. */
typedef struct xfb_f32_attention_args {
  const float* q;
  int64_t q_sb, q_sh, q_si;
  const float* k;
  int64_t k_sb, k_sh, k_si;
  const float* v;
  int64_t v_sb, v_sh, v_si;
  const float* bias;
  int64_t bias_sb, bias_sh, bias_si;
  const float* mask;
  int64_t mask_sb;
  float* out;
  int64_t out_sb, out_sh, out_si;
  const float* gate;
  int64_t gate_sb, gate_sh, gate_si;
  int64_t batch, heads, nq, nk, d, dv;
  double scale;
} xfb_f32_attention_args;
XFB_API int xfb_f32_attention(const xfb_f32_attention_args* args, void* stream);

/* y[r][c] = silu(h[r][c]) * h[r][f + c] for h [rows][2f] (gated_linear_unit_torch,
 * fastnn/gated_linear_unit.py:103-107). */
XFB_API int xfb_f32_silu_mul(const float* h, int64_t rows, int64_t f, float* y, void* stream);

/* y[t] = y[t] * scale[t] + shift[t] over n values (AdaptiveLayerNorm modulation,
 * diffusion_transformer.py:57-62). */
XFB_API int xfb_f32_scale_shift(float* y, const float* scale, const float* shift, int64_t n,
                                void* stream);

/* ------------------------------------------------------------------ checkpoint upload
 * Scatter of a parameter record stream (xfold/params.py:39-95, read by
 * get_alphafold3_params :245-256) already on the device as one blob: record r's
 * array bytes [spans[3r], + spans[3r+2]) of src go to dst + spans[3r+1] (4-byte
 * aligned; the caller picks 256-byte aligned slots so every array is a typed
 * view).  `spans` is the device copy of `host_spans`; the host copy is used to
 * check every span against src_bytes / dst_bytes before the launch. */
XFB_API int xfb_gather_bytes(const void* src, int64_t src_bytes, void* dst, int64_t dst_bytes,
                             const int64_t* spans, const int64_t* host_spans, int64_t count,
                             void* stream);

#ifdef __cplusplus
}
#endif

#endif /* XFOLD_B200_H_ */
