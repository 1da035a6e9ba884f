/*
 * libqmtp -- C ABI of the B200 (sm_100a) decode hot path for Qwen3.5 MTP speculative decoding.
 *
 * Conventions for every entry point:
 *   - pointers are DEVICE pointers of the current CUDA device; `stream` is a cudaStream_t (may be 0);
 *   - bf16 tensors are passed as uint16 bit patterns, row-major and contiguous unless a leading
 *     dimension is given;
 *   - the caller allocates every output and workspace; the library never allocates, frees or
 *     synchronises inside an entry point, so calls can be captured in a CUDA graph;
 *   - the return value is QMTP_OK or a negative QMTP_ERR_* code (host-side validation or launch
 *     failure); kernels that can time out on a bounded wait record it in the device error word
 *     read by qmtp_device_error().
 * Each declaration cites the reference interface it replaces (path:line in aulafy/qwen-mtp-mac).
 */
#ifndef QMTP_H_
#define QMTP_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define QMTP_OK 0
#define QMTP_ERR_SHAPE -1       /* unsupported or inconsistent sizes */
#define QMTP_ERR_ALIGN -2       /* a pointer is not 16-byte aligned */
#define QMTP_ERR_UNSUPPORTED -3 /* valid request this build does not implement */
#define QMTP_ERR_CUDA -4        /* CUDA launch/runtime error */
#define QMTP_ERR_ARG -5         /* null pointer or invalid argument value */

/* Human-readable text for a QMTP_* code. */
const char* qmtp_strerror(int code);

/* Library version as MAJOR*10000 + MINOR*100 + PATCH. */
int qmtp_version(void);

/* Reads (and with clear != 0 resets) the device error word of the current device: bit 0 = a
 * bounded wait gave up, bit 1 = a kernel saw an invalid runtime argument.  Synchronous. */
int qmtp_device_error(unsigned* out, int clear);

/* --------------------------------------------------------------------------------------------
 * Multi-row 4-bit GEMV, affine group 64 (MLX quantized_matmul(x, w, scales, biases, transpose=True,
 * group_size=64, bits=4); replaces the QuantizedLinear.__call__ route of qmv_kernel.py:104-113 and
 * the kernel qmv_nvfp4 of qmv_kernel.py:86-101 for the affine format).  Runs on the tensor cores
 * (tcgen05.mma kind::i8): every group of 64 activations is put on a block-floating-point grid
 * (x_q = RNE(x * 2^(19-E)), E = exponent of the group's largest |x|) and each group's dot product
 * with the 4-bit codes is an exact integer; the fp32 sequence after that is fixed (oracle
 * qo_qmv_affine).  Results do not depend on M, on the launch shape or on the entry point.
 *   x  bf16 [M, K]; w uint32 [N, K/8] (8 nibbles per word, low nibble = lowest k);
 *   scales, biases bf16 [N, K/64]; y bf16 [M, ldy] (columns 0..N-1 written).
 *   K % 512 == 0; any M >= 1 (processed 4 rows per launch); N >= 1.
 * This entry point needs no workspace: each CTA computes whole tiles of rows (for small N fewer CTAs
 * than SMs work; qmtp_qmv_affine_g64_split spreads the reduction over every SM). */
int qmtp_qmv_affine_g64(const void* x, const void* w, const void* scales, const void* biases,
                        void* y, int M, int N, int K, int ldy, void* stream);

/* qmtp_qmv_affine_g64 with a residual epilogue: y = bf16(res + bf16(x . W^T)) (the bf16 residual
 * add of a decoder layer fused into the projection; res may alias y).  res bf16 [M, ldy]. */
int qmtp_qmv_affine_g64_res(const void* x, const void* w, const void* scales, const void* biases,
                            void* y, const void* res, int M, int N, int K, int ldy, void* stream);

/* Workspace bytes for qmtp_qmv_affine_g64_split / _norm: 256 for every supported N x K (0 if K % 512
 * != 0).  The kernel no longer uses it -- a tile shared between CTAs is finished inside their
 * thread-block cluster -- and the argument is kept so existing callers keep working. */
size_t qmtp_qmv_workspace(int N, int K);

/* qmtp_qmv_affine_g64 (+ optional residual, res may be NULL) with strided rows: x rows at
 * x + m * ldx (elements; 0 = K).  Same bits as qmtp_qmv_affine_g64 (every entry point may share a
 * tile's 512-k slices between the CTAs of a cluster; the slice partials are added in order).
 * workspace / ws_bytes: ignored, may be NULL / 0. */
int qmtp_qmv_affine_g64_split(const void* x, long long ldx, const void* w, const void* scales,
                              const void* biases, void* y, const void* res, int M, int N, int K, int ldy,
                              void* workspace, size_t ws_bytes, void* stream);

/* qmtp_qmv_affine_g64_split on RMS-normalised rows: y = RMSNorm(x; norm_w, eps) . W^T (+ res), the
 * decoder's input_ln / post_ln (mlx_lm RMSNorm, the rmsnorm of qmtp_rmsnorm) computed by every CTA in
 * the kernel's prologue instead of a separate launch.  Same bits as qmtp_rmsnorm followed by
 * qmtp_qmv_affine_g64.  x: the un-normalised rows (bf16 [M, ldx]); norm_w bf16 [K]; K % 1024 == 0,
 * K <= 32768.  workspace / ws_bytes: ignored, may be NULL / 0. */
int qmtp_qmv_affine_g64_norm(const void* x, long long ldx, const void* norm_w, float eps, const void* w,
                             const void* scales, const void* biases, void* y, const void* res, int M, int N,
                             int K, int ldy, void* workspace, size_t ws_bytes, void* stream);

/* qmtp_qmv_affine_g64_split with the SwiGLU of an MLP in front: y = (silu(gate) * up) . W^T (+ res), the
 * gate at gu[m, k] and the up projection at gu[m, K + k] (ldgu >= 2K elements; 0 = 2K); silu and the
 * bf16 roundings of the decoder's qmtp_swiglu, computed by every CTA while it builds its operand.  Same
 * bits as qmtp_swiglu followed by qmtp_qmv_affine_g64.  (mlx-lm's MLP: down(silu(gate(x)) * up(x)).) */
int qmtp_qmv_affine_g64_swiglu(const void* gu, long long ldgu, const void* w, const void* scales,
                               const void* biases, void* y, const void* res, int M, int N, int K, int ldy,
                               void* stream);

/* qmtp_qmv_affine_g64_split with the GatedDeltaNet output gate in front (gdn_fused.py:10,144, the
 * norm of qmtp_gdn_norm_gate): x = bf16(RMSNorm_head(yg; norm_w, eps) * silu(z)) over heads of 128,
 * yg fp32 [M, ldyg] (floats), z bf16 [M, ldz], norm_w bf16 [128].  Same bits as qmtp_gdn_norm_gate
 * followed by qmtp_qmv_affine_g64. */
int qmtp_qmv_affine_g64_gated(const float* yg, long long ldyg, const void* z, long long ldz, const void* norm_w,
                              float eps, const void* w, const void* scales, const void* biases, void* y,
                              const void* res, int M, int N, int K, int ldy, void* stream);

/* Tiling the affine kernel picks for an N x K matrix (split: ignored): weight
 * rows per tile, CTAs, work units (tile x 512-k slice) and CTAs per thread-block cluster (> 1: each
 * tile is shared by the CTAs of one cluster, whose first CTA adds the others' slice partials in order
 * through distributed shared memory; every entry point may pick this mode, it needs no workspace).
 * Host-only query (it may query the device's cluster occupancy once). */
int qmtp_qmv_plan(int N, int K, int split, int* rows_per_tile, int* grid, int* units, int* cluster);

/* Overrides the affine kernel's planner for every later call in the process (no counterpart in the
 * reference; for tests and measurements): 0 = cost model (default), 1 = whole tiles per CTA only,
 * 2 = cluster mode wherever the shape allows it.  Every mode gives the same bits. */
int qmtp_qmv_set_mode(int mode);

/* Multi-row 4-bit GEMV, NVFP4 (e2m1 nibbles, e4m3 scale per 16): qmv_kernel.py:86-101 qmv_nvfp4.
 *   x bf16 [M, K]; w uint32 [N, K/8]; scales uint8 [N, K/16]; y bf16 [M, ldy]. K % 1024 == 0. */
int qmtp_qmv_nvfp4_g16(const void* x, const void* w, const void* scales, void* y, int M, int N,
                       int K, int ldy, void* stream);

/* qmtp_qmv_nvfp4_g16 with a residual epilogue, y = bf16(res + bf16(x . W^T)) (res [M, ldy], may be y):
 * the decoder's o_proj / out_proj / down projections of an NVFP4 checkpoint. */
int qmtp_qmv_nvfp4_g16_res(const void* x, const void* w, const void* scales, void* y, const void* res, int M,
                           int N, int K, int ldy, void* stream);

/* Affine 4-bit group-64 quantizer (MLX mx.quantize(w, 64, 4) convention, min/max form; used by
 * the loader, qwen_ollama.py:45-50 / lm_head2.py:17):  w bf16 [N, K] -> wq uint32 [N, K/8],
 * scales, biases bf16 [N, K/64].  K % 64 == 0. */
int qmtp_quantize_affine_g64(const void* w, void* wq, void* scales, void* biases, int N, int K,
                             void* stream);

/* --------------------------------------------------------------------------------------------
 * Diagnostics (no counterpart in the reference; they let the test suite reach device building blocks).
 * qmtp_math_eval: out[i] = f(bf16 x[i]) as fp32 for the device functions every kernel shares: the
 * library's exp and log, and the bf16 activation formulas of gdn_fused.py:22-41 (sigmoid, silu,
 * softplus with a bf16 rounding after every op) plus the fp32 silu.  x bf16 [n], out fp32 [n]. */
#define QMTP_MATH_EXP 0
#define QMTP_MATH_LOG 1
#define QMTP_MATH_SIGMOID_BF 2
#define QMTP_MATH_SILU_BF 3
#define QMTP_MATH_SOFTPLUS_BF 4
#define QMTP_MATH_SILU_F32 5
int qmtp_math_eval(int fn, const void* x, int n, float* out, void* stream);

/* qmtp_wait_selftest: one kernel waits on an mbarrier phase that never completes, with the bounded
 * wait every kernel of the library uses, limited to `limit` polls (1 .. 2^20).  The wait gives up,
 * records bit 0 (timeout) in the device error word and writes 0 to *result (device int); the kernel
 * returns normally.  Shows that a wait that runs out ends the kernel instead of hanging the GPU. */
int qmtp_wait_selftest(unsigned limit, int* result, void* stream);

/* --------------------------------------------------------------------------------------------
 * GatedDeltaNet recurrent step with per-token state snapshots: gdn_kernel.py:75-88
 * gated_delta_snapshot(q, k, v, g, beta, state) -> (y, state_out, state_mid).
 *   q, k bf16 [B, T, Hk, Dk]; v bf16 [B, T, Hv, Dv]; g, beta fp32 [B, T, Hv];
 *   state_in fp32 [B, Hv, Dv, Dk] -> y bf16 [B, T, Hv, Dv], state_out fp32 [B, Hv, Dv, Dk],
 *   state_mid fp32 [T-1, B, Hv, Dv, Dk] (state after tokens 1..T-1; may be NULL when T == 1).
 *   Dk == 128, Hv % Hk == 0 (GQA: value head hv reads key head hv / (Hv/Hk)). */
int qmtp_gdn_step(const void* q, const void* k, const void* v, const float* g, const float* beta,
                  const float* state_in, void* y, float* state_out, float* state_mid, int B, int T,
                  int Hk, int Hv, int Dk, int Dv, void* stream);

/* Fused GatedDeltaNet middle section, B = 1: gdn_fused.py:43-112 (gdn_core) as called by
 * gdn_middle (gdn_fused.py:149-167).  Causal conv over the window (KC taps) + silu, q/k RMS norm
 * (q / Dk, k * Dk^-1/2), g = exp(-exp(A_log) * softplus(a + dt_bias)), beta = sigmoid(b), delta
 * rule with snapshots.
 *   win bf16 [S+KC-1, C] (C = 2*Hk*Dk + Hv*Dv: conv state rows then the S new qkv rows);
 *   conv_w bf16 [C, KC]; a, b bf16 [S, >= Hv] (row stride ld_ab); A_log fp32 [Hv];
 *   dt_bias bf16 [Hv]; state_in fp32 [Hv, Dv, Dk]
 *   -> y fp32 [S, Hv, Dv] (bf16-rounded values, input of the gated norm), state_out,
 *      state_mid fp32 [S-1, Hv, Dv, Dk] when snap != 0.  Dk == 128, S <= 64. */
int qmtp_gdn_fused(const void* win, const void* conv_w, const void* a, const void* b, int ld_ab,
                   const float* A_log, const void* dt_bias, const float* state_in, float* y,
                   float* state_out, float* state_mid, int S, int Hk, int Hv, int Dk, int Dv, int KC,
                   int snap, void* stream);

/* General form of qmtp_gdn_fused for graph-captured decoding: the window is read from two
 * sources (conv rows at a device-side row offset, qkv rows with their own stride), the next
 * window can be written out, and the state can live in a ring of slots indexed by a device int
 * (state after token t -> slot (cur + t + 1) % ring_slots).  Rolling back to `keep` tokens is then
 * cur = (cur + keep) % ring_slots and conv_row_off = keep, with no copy (mtp.py:136-140 restore). */
typedef struct qmtp_gdn_args {
  const void* conv_src;      /* bf16 rows 0..KC-2 of the window start at row *conv_row_off */
  long long ld_conv;
  const int* conv_row_off;   /* device int, or NULL for 0 */
  const void* qkv;           /* bf16 [S, >= C] new conv inputs */
  long long ld_qkv;
  void* win_out;             /* bf16 [KC-1+S, C] or NULL */
  const int* win_out_row_off;/* device int: win_out starts *win_out_row_off rows later (NULL: 0) */
  const void* conv_w;
  const void* a;
  const void* b;
  long long ld_ab;
  const float* A_log;
  const void* dt_bias;
  const float* state_in;     /* explicit-state mode (ring == NULL) */
  float* state_out;
  float* state_mid;
  float* ring;               /* ring mode: ring_slots slots of Hv*Dv*Dk floats */
  const int* ring_cur;       /* device int: slot holding the state before token 0 */
  int ring_slots;            /* > S */
  float* y;                  /* fp32 [S, Hv, Dv] */
  int S, Hk, Hv, Dk, Dv, KC, snap;
  /* Optional gated RMS norm of the same step (gdn_fused.py:114-129, qmtp_gdn_norm_gate below):
   * gate_out bf16 [S, >= Hv*Dv] (row stride ld_gate_out) = bf16(R(gate_w * R(y * r)) * silu(gate_z)),
   * gate_z bf16 [S, >= Hv*Dv] (row stride ld_gate_z), gate_w bf16 [Dv].  NULL gate_out: no norm.
   * With the decode shape (S <= 4, KC == 4, Dk == Dv == 128, 16-byte aligned conv_w, 8-byte aligned
   * window rows) the norm runs inside the step's launch (an 8-CTA cluster per value head sums
   * y^2 over distributed shared memory); otherwise as a second launch. */
  const void* gate_z;
  long long ld_gate_z;
  const void* gate_w;
  void* gate_out;
  long long ld_gate_out;
  float gate_eps;
  /* Nonzero: the control words, the state (state_in or the ring slot) and the conv rows at conv_src
   * are read before the kernel's dependency wait, overlapping the previous launch.  Only valid when
   * none of them was written by the launch directly before this one on the stream, and that launch
   * is a libqmtp GEMV (qmtp_qmv_*: it signals its successor only after its own dependency wait), or
   * there is no programmatic dependency at all.  The decoder's in_proj -> step sequence qualifies. */
  int preload;
} qmtp_gdn_args;

int qmtp_gdn_fused_ex(const qmtp_gdn_args* args, void* stream);

/* Kernel choice of qmtp_gdn_fused / qmtp_gdn_fused_ex, for tests: 0 = automatic (the decode-shape
 * kernel where it applies), 1 = always the general kernel (and a separate gated-norm launch).  Both
 * give the same bits.  Returns the previous mode. */
int qmtp_gdn_set_mode(int mode);

/* Gated RMS norm of gdn_fused.py:114-129 (gdn_norm_gate): per (token, head) row of Dv,
 * out = bf16(R(w * R(y * r)) * silu_f32(z)), r = 1/sqrt(mean(y^2) + eps).
 *   y fp32 [S, H, Dv]; z bf16 [S, >= H*Dv] (row stride ld_z); w bf16 [Dv];
 *   out bf16 [S, >= H*Dv] (row stride ld_out).  Dv == 128. */
int qmtp_gdn_norm_gate(const float* y, const void* z, int ld_z, const void* w, void* out, int ld_out,
                       int S, int H, int Dv, float eps, void* stream);

/* --------------------------------------------------------------------------------------------
 * Two-stage lm_head: lm_head2.py:23-29 TwoStageHead.__call__ (coarse quantized logits ->
 * argpartition top-k -> take the k bf16 weight rows -> exact logits) plus the greedy argmax of
 * engine.py:121-124.  Ties are resolved as (value descending, vocab index ascending).
 *   h bf16 [M, K]; wq/scales/biases: affine g64 coarse head [V, K]; w_fine bf16 [V, K];
 *   -> out_idx int32 [M, k] (candidates in that order), out_fine bf16 [M, k] (exact logits),
 *      out_argmax int32 [M] (may be NULL), coarse_out bf16 [M, V] (may be NULL).
 *   workspace: qmtp_lmhead2_workspace(M, V, k) bytes, 16-B aligned.  k <= 2048 (above 256 the selection is a radix select and the rescoring runs across the SMs), K % 512 == 0. */
size_t qmtp_lmhead2_workspace(int M, int V, int k);
int qmtp_lmhead2(const void* h, const void* wq, const void* scales, const void* biases,
                 const void* w_fine, int M, int V, int K, int k, int* out_idx, void* out_fine,
                 int* out_argmax, void* coarse_out, void* workspace, size_t ws_bytes, void* stream);

/* qmtp_lmhead2 with the reference's own coarse format (lm_head2.py:19: NVFP4, group 16): coarse
 * logits by qmtp_qmv_nvfp4_g16 (wq uint32 [V, K/8] e2m1 nibbles, scales uint8 [V, K/16] e4m3),
 * then the same top-k selection, exact bf16 rescoring and argmax.  K % 1024 == 0; workspace:
 * qmtp_lmhead2_workspace(M, V, k). */
int qmtp_lmhead2_nvfp4(const void* h, const void* wq, const void* scales, const void* w_fine, int M, int V,
                       int K, int k, int* out_idx, void* out_fine, int* out_argmax, void* coarse_out,
                       void* workspace, size_t ws_bytes, void* stream);

/* Two-stage head sharded by vocabulary over G GPUs (lm_head2.py:111-117 split by output rows; the
 * NCCL exchange between the two calls is the host's, e.g. torch.distributed all_gather):
 *   qmtp_lmhead2_shard: on the rank holding vocabulary rows [v0, v0 + Vs): coarse logits of the shard,
 *     its top k (value descending, index ascending) and their exact bf16 logits.  out_words uint64
 *     [M, k]: (order key of the coarse logit << 32) | (0xFFFFFFFF - global index), so a larger word is
 *     a better candidate; out_fine bf16 [M, k].  workspace: qmtp_lmhead2_shard_workspace(M, Vs, k).
 *   qmtp_lmhead2_merge: every rank's lists gathered rank-major (words [G, M, k], fine [G, M, k]) ->
 *     the same out_idx / out_fine / out_argmax as qmtp_lmhead2 on the whole vocabulary, bit for bit
 *     (each shard's list holds its own best k, so the best k of the union are the global best k).
 *     G * k <= 4096. */
size_t qmtp_lmhead2_shard_workspace(int M, int Vs, int k);
int qmtp_lmhead2_shard(const void* h, const void* wq, const void* scales, const void* biases,
                       const void* w_fine, int M, int Vs, int K, int k, long long v0, void* out_words,
                       void* out_fine, void* workspace, size_t ws_bytes, void* stream);
int qmtp_lmhead2_merge(const void* words, const void* fine, int G, int M, int k, int* out_idx,
                       void* out_fine, int* out_argmax, void* stream);

/* The two-stage head of qmtp_lmhead2 for callers that cannot allocate device memory (a plugin
 * living inside another framework's memory pool, code that may run during stream capture, a
 * serving loop that must not synchronise the device through cudaMalloc).  This entry point has no
 * counterpart in the reference.  It takes no workspace: it uses a scratch area that is a static
 * __device__ array of the library (2 MiB + 64 KiB on every GPU that loads the library, until exit).
 * Limits: M <= 4 rows, V <= 262144, k <= 64 (larger requests return QMTP_ERR_SHAPE).  The first
 * call in a CUDA context looks up the scratch address there (cudaGetSymbolAddress) and caches it
 * for that context; make that first call before any stream capture.  A failed lookup is not cached,
 * and a new context (after cudaDeviceReset) gets a fresh lookup.  All calls share the one scratch
 * area, so calls that can overlap on the GPU (different streams, or concurrent host threads) race;
 * serialise them.  Results are identical to qmtp_lmhead2. */
int qmtp_lmhead2_noalloc(const void* h, const void* wq, const void* scales, const void* biases,
                         const void* w_fine, int M, int V, int K, int k, int* out_idx, void* out_fine,
                         int* out_argmax, void* stream);

/* Stage 2 alone: exact top-k of bf16 rows vals [M, ld] (first V columns) and, when w_fine is
 * given, the rescoring of the candidates against w_fine [V, K] with h [M, K] and their argmax
 * (lm_head2.py:25-29).  workspace: qmtp_topk_workspace(M, V, k) bytes. */
size_t qmtp_topk_workspace(int M, int V, int k);
int qmtp_topk_rescore(const void* vals, int ld, int M, int V, int k, const void* w_fine,
                      const void* h, int K, int* out_idx, void* out_fine, int* out_argmax,
                      void* workspace, size_t ws_bytes, void* stream);

/* Greedy token of bf16 logits rows (mtp.py:165-167 DraftHead.token / mx.argmax, ties -> lowest
 * index): vals [M, ld] -> out int32 [M].  workspace: qmtp_argmax_workspace(M, V) bytes. */
size_t qmtp_argmax_workspace(int M, int V);
int qmtp_argmax_bf16(const void* vals, int ld, int M, int V, int* out, void* workspace,
                     size_t ws_bytes, void* stream);

/* qmtp_argmax_bf16 for a head over a vocabulary subset (mtp.py:156-167 DraftHead with ids,
 * load_draft_head(vocab, quant, freq, extra_ids)): row i of vals scores vocabulary id ids[i] (int32
 * [V], may be NULL for ids[i] = i); out[m] = ids[argmax], out_local[m] (may be NULL) = the argmax row
 * itself.  Same tie rule (lower row) and workspace as qmtp_argmax_bf16. */
int qmtp_argmax_bf16_ids(const void* vals, int ld, int M, int V, const int* ids, int* out, int* out_local,
                         void* workspace, size_t ws_bytes, void* stream);

/* --------------------------------------------------------------------------------------------
 * Decoder ops of the synthetic Qwen3.5 model (mtp.py:143-153 backbone, mtp.py:35-45 MTP layer;
 * layer structure of mlx-lm qwen3_5, cross-checked with transformers' Qwen3.5).  Positions may come
 * from a device int (pos_ptr, + pos_add + row), so the calls can sit in a replayed CUDA graph. */

/* Quantized embedding gather (affine g64 rows): out[t] = bf16(fma(s, q, b)) of row tokens[t]. */
int qmtp_embed(const int* tokens, int T, const void* wq, const void* scales, const void* biases, int V,
               int D, void* out, int ld_out, void* stream);

/* Quantized embedding gather, NVFP4 rows (the embed_tokens of an NVFP4 checkpoint, qwen_ollama.py:50-51):
 * out[t][e] = bf16(e2m1(q) * e4m3(scale of 16)); wq uint32 [V, D/8], scales uint8 [V, D/16]. */
int qmtp_embed_nvfp4(const int* tokens, int T, const void* wq, const void* scales, int V, int D, void* out,
                     int ld_out, void* stream);

/* RMSNorm (mx.fast.rms_norm): out = bf16(w * bf16(x * r)), r = 1/sqrt(mean(x^2) + eps), D % 1024 == 0.
 * Row m reads x row (*row_sel + m) when row_sel != NULL. */
int qmtp_rmsnorm(const void* x, int ld_x, const int* row_sel, const void* w, float eps, void* out,
                 int ld_out, int M, int D, void* stream);

/* Embedding rows (affine g64 table, as qmtp_embed) and RMS norms (as qmtp_rmsnorm) in one launch:
 * row m of job 0 is the embedding of tok[m], written to raw (bf16 [M, >= D], row stride ld_raw; may be
 * NULL) and, RMS-normalised with w0, to out0; job 1 (x1 not NULL) is qmtp_rmsnorm of rows *row_sel1 + m
 * (row_sel1 may be NULL: 0) of x1 with w1 into out1.  The decoder uses it for the embedding + layer 0's
 * input norm of a verify step and for an MTP step's embedding + its two pre-fc norms (mtp.py:202-203). */
int qmtp_embed_rmsnorm(const int* tok, int M, const void* wq, const void* scales, const void* biases, int V, int D,
                       void* raw, int ld_raw, const void* w0, void* out0, int ld_out0, const void* x1, int ld_x1,
                       const int* row_sel1, const void* w1, void* out1, int ld_out1, float eps, void* stream);

/* Gated-attention input prep (Dh 256, rotary 64): per-head q/k RMS norm, rotate-half RoPE from the
 * cos/sin tables [max_pos][32], q and gate out [S, nq, Dh], k and v appended to the caches
 * [nkv, max_pos, Dh] at position *pos_ptr + pos_add + s.  qkv, qn_w, kn_w 16-byte aligned. */
int qmtp_attn_prep(const void* qkv, int ld, int S, int nq, int nkv, int Dh, int rotary, const void* qn_w,
                   const void* kn_w, float eps, const float* cos_t, const float* sin_t, const int* pos_ptr,
                   int pos_add, void* q_out, void* gate_out, void* k_cache, void* v_cache, int max_pos,
                   void* stream);

/* Causal decode attention over the caches (query s sees keys 0..pos+s) with the sigmoid output
 * gate: out bf16 [S, nq*Dh] = bf16(attn * sigmoid(gate)).  Dh 256. */
int qmtp_attention(const void* q, const void* gate, const void* k_cache, const void* v_cache, int max_pos,
                   int S, int nq, int nkv, int Dh, const int* pos_ptr, int pos_add, void* out,
                   void* stream);

/* qmtp_attn_prep followed by qmtp_attention in one launch, with the same results and cache writes:
 * the attention kernel prepares its own q row and the new key it needs from the projection output
 * qkv (the arguments of qmtp_attn_prep), reads the gate there, and writes the S new key / value rows
 * to the caches.  S <= 8; Dh 256, rotary 64; qkv, qn_w, kn_w, the caches 16-byte aligned. */
int qmtp_attention_fused(const void* qkv, int ld, int S, int nq, int nkv, int Dh, int rotary, const void* qn_w,
                         const void* kn_w, float eps, const float* cos_t, const float* sin_t, const int* pos_ptr,
                         int pos_add, void* k_cache, void* v_cache, int max_pos, void* out, void* stream);

/* SwiGLU of mlx-lm's MLP: out [S, I] = bf16(silu(gate) * up), gu [S, ld] = (gate | up) columns. */
int qmtp_swiglu(const void* gu, int ld, int S, int I, void* out, void* stream);

/* ---------------------------------------------------------------- MXFP4 / NVFP4 MoE
 * Replaces experiments/deepseek_moe/kernels.py:133-155 (moe_decode, batch 1) with the batched
 * decode of T tokens.  Weight layout as the reference (kernels.py:3-5): w uint32 [E, N, K/8],
 * 8 e2m1 nibbles per word, low nibble = lowest k; scales uint8 [E, N, K/G].
 * fmt 0 = MXFP4 (e8m0 scale per 32, kernels.py:31-32), fmt 1 = NVFP4 (e4m3 per 16, sign ignored
 * as qmv_kernel.py:26-28). */
#define QMTP_FP4_MXFP4 0
#define QMTP_FP4_NVFP4 1

/* Quantizes bf16 w [N, K] (K % G == 0) into (wq, scales); OCP MX rule for MXFP4, e4m3(amax/6) for
 * NVFP4, round-to-nearest-even e2m1 codes.  (The reference draws random bits instead,
 * bench_moe.py:24-31; the quantizer is this library's.) */
int qmtp_quantize_fp4(int fmt, const void* w, long long N, int K, void* wq, void* scales, void* stream);

/* Router (bench_moe.py:40-42 builds idx / scores the same way): logits fp32 [T, E] -> top_k experts by
 * logit (ties to the lower id), weights softmax-renormalised over the chosen k times routed_scale,
 * then n_shared shared experts E .. E+n_shared-1 with weight 1.  idx int32 / scores fp32
 * [T, top_k + n_shared].  E <= 1024, top_k + n_shared <= 16. */
int qmtp_moe_route(const void* logits, int T, int E, int top_k, int n_shared, float routed_scale, void* idx,
                   void* scores, void* stream);

/* Device workspace (bytes) of qmtp_moe for T tokens, S slots per token, E experts, hidden H, FFN I. */
size_t qmtp_moe_workspace(int T, int S, int E, int H, int I);

/* y bf16 [T, H] = sum_j scores[t,j] * Wd[e] (silu(min(Wg[e] x_t, L)) * clamp(Wu[e] x_t, -L, L)),
 * e = idx[t, j] (kernels.py:35-107).  x bf16 [T, H]; wg, wu [E, I, H/8]; wd [E, H, I/8]; limit = +inf
 * disables the clamp.  H, I multiples of 128; S <= 16; T*S <= 65535; E <= 1024; scale rows of one 128-row
 * tile must fit the kernel's scale buffers (H <= 4096 MXFP4 / 2048 NVFP4).  All pointers 16-B
 * aligned, workspace 256-B aligned.  An expert id outside [0, E) raises the device error word and
 * its slot contributes nothing. */
int qmtp_moe(int fmt, const void* x, const void* wg, const void* sg, const void* wu, const void* su, const void* wd,
             const void* sd, const void* idx, const void* scores, void* y, int T, int S, int E, int H, int I,
             float limit, void* workspace, size_t ws_bytes, void* stream);

/* Expert-parallel building blocks.  qmtp_moe_experts: partial[r] (fp32 [n, H]) = Wd[e] (silu(min(Wg[e] x_r, L)) *
 * clamp(Wu[e] x_r, -L, L)) for each row r with expert e = expert[r] (int32 [n]), i.e. one (token, slot) entry per
 * row without the routing weight; rows keep their input order.  Same limits as qmtp_moe (S = 1); the workspace is
 * qmtp_moe_workspace(n, 1, E, H, I).
 * expert[r] = -1 marks an empty row: it is skipped and partial[r] is left unwritten.
 * qmtp_moe_combine: y[t] (bf16) = sum_j scores[t, j] * partials[row_of[t, j]] (fp32 [*, H]) in slot order j;
 * row_of < 0 skips a slot.  H % 4 == 0, S <= 16. */
int qmtp_moe_experts(int fmt, const void* x, const void* wg, const void* sg, const void* wu, const void* su,
                     const void* wd, const void* sd, const void* expert, void* partial, int n, int E, int H, int I,
                     float limit, void* workspace, size_t ws_bytes, void* stream);
int qmtp_moe_combine(const void* partials, const void* row_of, const void* scores, int T, int S, int H, void* y,
                     void* stream);

/* Fixed-capacity dispatch of one expert-parallel MoE layer (no counterpart in the reference, whose MoE
 * runs on one device).  `world` ranks, rank r owning routed experts [r * per, (r + 1) * per), per =
 * n_routed / world; ids >= n_routed are shared experts, computed by every rank for its own tokens.
 * For this rank's T tokens, idx int32 [T, S] and x bf16 [T, H]:
 *   send_x bf16 [world * cap, H], send_e int32 [world * cap]: the rows for rank d at d * cap + p (p in
 *     (t, j) order) with the local expert id e - d * per; unused slots have id -1;
 *   sh_x bf16 [T * S, H], sh_e int32 [T * S]: the shared-expert rows, local id per + e - n_routed
 *     (the layout of a rank's expert table: its routed shard, then the shared experts); unused -1;
 *   pos int32 [T * S]: the row of entry (t, j) in the table [partials sent back by the ranks
 *     (world * cap rows) ; this rank's expert pass over its world * cap received rows, then its shared
 *     rows], i.e. d * cap + p for a routed entry and 2 * world * cap + q for the q-th shared entry;
 *   counts int32 [world + 1]: entries sent to each rank, then the shared entries.
 * Every size is fixed, so the all-to-alls of send_x / send_e and of the partials use equal splits and
 * the layer needs no host synchronisation.  cap must cover the routed entries this rank sends to any one
 * rank (T * S always does); an entry beyond cap, or with an invalid id, is dropped (pos = -1) and the
 * device error word records it.  H % 8 == 0; x, send_x, sh_x 16-byte aligned. */
int qmtp_moe_dispatch(const void* idx, int T, int S, const void* x, int H, int n_routed, int n_shared, int world,
                      int cap, void* send_x, void* send_e, void* sh_x, void* sh_e, void* pos, void* counts,
                      void* stream);

/* Control block of the device-side speculative loop (int32 [QMTP_CTRL_SIZE]). */
#define QMTP_CTRL_SLOT 0      /* GatedDeltaNet state ring slot before the next verify */
#define QMTP_CTRL_CONV_ROW 1  /* row of the conv state inside the [2 * win_rows, C] window buffer */
#define QMTP_CTRL_WOUT_ROW 2  /* row where the next window is written */
#define QMTP_CTRL_WPAR 3      /* window buffer parity */
#define QMTP_CTRL_POS 4       /* tokens in the trunk KV caches */
#define QMTP_CTRL_MPOS 5      /* committed entries of the MTP KV cache */
#define QMTP_CTRL_KEEP 6      /* tokens kept by the last verify (1..k+1) */
#define QMTP_CTRL_SEL 7       /* KEEP - 1 */
#define QMTP_CTRL_NOUT 8      /* tokens emitted so far */
#define QMTP_CTRL_CYCLES 9    /* verify cycles */
#define QMTP_CTRL_ACC0 10     /* accepted-draft counters per draft position */
#define QMTP_CTRL_NUSE 18     /* adaptive k: drafts the next verify may accept (0: all k) */
#define QMTP_CTRL_VERIFIED 19 /* drafts verified so far (sum over cycles of the accept limit) */
#define QMTP_CTRL_EMIT0 20    /* tokens emitted by the last cycle (KEEP of them) */
#define QMTP_CTRL_MAX_K 8
#define QMTP_CTRL_RNG 29      /* sampling: calls of qmtp_sample so far (the Philox call counter) */
#define QMTP_CTRL_SEED_LO 30  /* sampling: Philox key, low word (set by the caller) */
#define QMTP_CTRL_SEED_HI 31  /* sampling: Philox key, high word */
#define QMTP_CTRL_SIZE 32

/* Greedy verification + rollback bookkeeping (mtp.py:275-294, engine.py:121-128, mtp.py:136-140):
 * a = verify argmax [k+1], in = [t, d_1..d_k]; keep = 1 + leading drafts equal to a; appends
 * a[0..keep) to out_tokens (forced_keep > 0: keep = forced_keep, nothing emitted, prefill);
 * advances POS, the state-ring slot and the conv window by keep. */
int qmtp_mtp_accept(const int* a, const int* in, int k, int* ctrl, int* out_tokens, int out_cap,
                    int ring_slots, int win_rows, int forced_keep, void* stream);

/* Adaptive draft count (mtp.py:217-238: draft_chain(..., with_probs) and n_drafts(probs, tau)):
 *   qmtp_draft_prob: prob = softmax(logits)[token] = 1 / sum_j exp(l_j - l_token) of the draft head's
 *     bf16 logits [V] at its argmax token (device int); fixed reduction order (oracle qo_draft_prob).
 *   qmtp_mtp_nuse: ctrl[QMTP_CTRL_NUSE] = n_drafts(probs[0..k), tau) (running product in double, at
 *     least 1); qmtp_mtp_accept then accepts at most that many drafts and adds it to
 *     ctrl[QMTP_CTRL_VERIFIED].  ctrl[QMTP_CTRL_NUSE] = 0 (the reset value) keeps all k. */
int qmtp_draft_prob(const void* logits, int V, const int* token, float* prob, void* stream);
int qmtp_mtp_nuse(const float* probs, int k, double tau, int* ctrl, void* stream);

/* MPOS += KEEP (the MTP cache keeps the real pairs of this cycle; mtp.py:291-294). */
int qmtp_mtp_advance(int* ctrl, void* stream);

/* Next verify input: in = [a[SEL], drafts[0..k)]. */
int qmtp_next_tokens(const int* a, const int* drafts, int k, const int* ctrl, int* in, void* stream);

/* Sampling parameters (engine.py:29-35 Sampling): temperature > 0; top_k 0 = off; top_p in (0, 1],
 * 1 = off; min_p in [0, 1], 0 = off. */
typedef struct {
  float temperature;
  int top_k;
  float top_p;
  float min_p;
} qmtp_sampling;

/* Exact speculative sampling over the two-stage head's candidates (engine.py:91-152: Engine._dist,
 * _sample_first, _verify).  idx int32 / fine bf16 [rows, ld]: K <= 2048 candidates per row (vocabulary
 * ids and exact logits, as qmtp_topk_rescore writes them).
 *   first_row < 0 (verify): drafts[0..k); draft i is accepted with probability p_i(d_i), else a token
 *     is drawn from p_i without d_i and the cycle stops; all accepted -> a bonus draw from row k.
 *     out[0..n_acc] = the emitted tokens (accepted drafts, then the drawn token), so a following
 *     qmtp_mtp_accept(out, [t, drafts]) counts n_acc and commits n_acc + 1 tokens.
 *   first_row >= 0: one draw from that row into out[first_row] (the first token after a prompt).
 * Random numbers: Philox4x32-10 keyed by ctrl[QMTP_CTRL_SEED_LO/HI], counter (ctrl[QMTP_CTRL_RNG],
 * row, use, 0); every call increments ctrl[QMTP_CTRL_RNG].  V = vocabulary size (top_k >= V is off). */
int qmtp_sample(const int* idx, const void* fine, int K, int ld, const int* drafts, int k, int first_row,
                const qmtp_sampling* sp, int V, int* ctrl, int* out, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* QMTP_H_ */
