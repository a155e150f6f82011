/*
 * tropical_b200.h -- C ABI of the B200 (sm_100a) tropical / max-plus kernels.
 *
 * Conventions shared by every entry point
 * ---------------------------------------
 *  - Plain pointers and sizes only; no framework types.  All pointers are
 *    device pointers on the CURRENT CUDA device unless stated otherwise.
 *  - Sizes are int64_t element counts; strides are in ELEMENTS (not bytes).
 *  - `stream` is a cudaStream_t passed as void* (NULL = legacy default stream).
 *    Every launch is asynchronous on that stream; no entry point synchronises
 *    the device.  No entry point allocates device memory, with one exception:
 *    the large fp32 forward's stream-K schedule (tp_set_stream_k) draws a
 *    stream-ordered workspace of up to ~27 MB from a library-owned memory
 *    pool that keeps its memory between calls; tp_set_stream_k(0) turns that
 *    off (results are identical either way).
 *  - Every function returns int: 0 (TP_OK) on success, a negative TP_ERR_*
 *    value when host-side validation rejects the arguments (nothing is
 *    launched), or a positive cudaError_t value if a CUDA call failed.
 *    tp_status_string() turns any of them into text.
 *  - Outputs that the reference accumulated into caller-zeroed buffers
 *    (gradients) are fully OVERWRITTEN here; callers need not zero them.
 *
 * Reference interface being replaced: Mediocr3Mik3/MK_III_Technologies_TSRN
 * cuda/maxplus_gemm.cu:297-341 (three void launchers on the legacy stream, no
 * error reporting) and the PyTorch expressions they were meant to accelerate:
 * tropformer.py:127-145 (TropicalLinear), tropformer.py:87-97 (_tropical_max),
 * deep_tropical_net.py:148-150 (tropical attention score),
 * research/tsrn_dml.py:438-460 (log-sum-exp tropical score) and
 * research/tsrn_dml.py:961-972 (TropicalSSM max-plus scan).
 */
#ifndef TROPICAL_B200_H
#define TROPICAL_B200_H

#include <stdint.h>
#ifndef __cplusplus
#include <stdbool.h>
#endif

#if defined(__GNUC__)
#define TP_API __attribute__((visibility("default")))
#else
#define TP_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes ------------------------------------------------------ */
#define TP_OK 0
#define TP_ERR_INVALID_ARG (-1)   /* negative size, bad stride, bad mode     */
#define TP_ERR_NULL_POINTER (-2)  /* required pointer is NULL                */
#define TP_ERR_MISALIGNED (-3)    /* pointer/stride violates an alignment rule */
#define TP_ERR_UNSUPPORTED (-4)   /* dtype / mode / layout not supported     */
#define TP_ERR_TOO_LARGE (-5)     /* size exceeds a documented limit         */
#define TP_ERR_BAD_POINTER (-6)   /* pointer is not device memory of the current device */
#define TP_ERR_WORKSPACE (-7)     /* workspace missing or too small          */

/* ---- enums ------------------------------------------------------------- */
#define TP_DTYPE_F32 0   /* operands stored as IEEE fp32                       */
#define TP_DTYPE_BF16 1  /* operands stored as bf16; arithmetic is exact fp32  */
#define TP_DTYPE_BF16_ARITH 2  /* bf16 storage AND bf16 arithmetic: every sum
                                  x + w rounded to bf16 (ties to even) as torch
                                  does on bf16 tensors; exact max; the max is
                                  returned in fp32, bias/scale applied in fp32.
                                  Forward only (tp_maxplus_fwd[_strided]). */

#define TP_BWD_STE 1     /* d/ds of sum(softmax(s/tau)*s): TropicalLinear train mode */
#define TP_BWD_LSE 2     /* softmax(s/tau): gradient of tau*logsumexp(s/tau) (Maslov) */

/* Text for a status code (static storage, never NULL). */
TP_API const char* tp_status_string(int status);

/* ABI version of this library (bumped on any signature change). */
TP_API int tp_abi_version(void);

/* Enable (1) or disable (0) the per-call host check that every pointer argument
 * is device memory of the current device (cudaPointerGetAttributes).  Enabled
 * by default.  Returns the previous setting. */
TP_API int tp_set_pointer_checks(int enable);

/* ======================================================================== *
 *  Max-plus GEMM forward
 *
 *    s[m,n,k] = x[m,k] + w[n,k]                  (one rounded fp32 add)
 *    mx[m,n]  = max_k s[m,n,k]                   (exact; NaN propagates)
 *    y[m,n]   = (bias ? mx + bias[n] : mx) * scale   (scale applied iff != 1)
 *    argmax[m,n] = lowest k attaining mx (first NaN if mx is NaN; 0 for K==0
 *                  or an all -inf row, matching torch.max(dim=-1).indices)
 *
 *  Replaces: tropformer.py:131-141 (scores.max(-1) + bias) and
 *  cuda/maxplus_gemm.cu:297-315 maxplus_forward_cuda.  Bit-exact with the
 *  reference's fp32 torch expression for values and indices.
 *  argmax may be NULL (value-only, faster).  K == 0 gives y = -inf.
 * ======================================================================== */
TP_API int tp_maxplus_fwd(int dtype, int64_t M, int64_t N, int64_t K,
                   const void* x, int64_t ldx,
                   const void* w, int64_t ldw,
                   const float* bias,
                   float* y, int64_t ldy,
                   int32_t* argmax, int64_t ld_argmax,
                   void* stream);

/* Tropical linear followed by its Legendre-Fenchel dual activation, fused
 * into the forward epilogue (inference: values only, no argmax).
 * Replaces trop_up + lf_act of TropicalHybridFFN / DTNHybridFFN
 * (tropformer.py:447, deep_tropical_net.py:206; LFDualActivation,
 * tropformer.py:224-289):  v = max_k(x + w) + bias, then
 *   act_mode 0 (primal):  max_p (v*slopes[p] + piece_bias[p])
 *   act_mode 1 (dual):    max_p (v*x_grid[p] - f(x_grid[p])), f the primal
 *   act_mode 2 (blend):   gate[n]*primal + (1 - gate[n])*dual, gate = sigmoid(blend_gate)
 * Products and sums are rounded separately, as the reference evaluates them,
 * so the result is bit-exact with it (given the same gate values).
 * pieces <= 16; slopes, piece_bias, x_grid, gate are device arrays. */
TP_API int tp_maxplus_fwd_lfdual(int dtype, int64_t M, int64_t N, int64_t K,
                                 const void* x, int64_t ldx, const void* w, int64_t ldw,
                                 const float* bias, float* y, int64_t ldy,
                                 int act_mode, int pieces, const float* slopes,
                                 const float* piece_bias, const float* x_grid,
                                 const float* gate, void* stream);

/* Fully strided, two-level batched form of tp_maxplus_fwd.  Batch index
 * (b1, b2) in [0,B1) x [0,B2) offsets every operand by b1*s_b1 + b2*s_b2;
 * element (m,k) of x is x[m*sx_m + k*sx_k], element (n,k) of w is
 * w[n*sw_n + k*sw_k].  Used for the batched tropical attention score
 * S[b,h,i,j] = max_f(Q[b,h,i,f] + K[b,h,j,f]) * scale
 * (deep_tropical_net.py:148-150, tropformer.py:378-381) with Q/K as strided
 * head views of [B, L, H*dk], and for A (x) B with B stored [K,N]
 * (cuda/maxplus_gemm.cu:331-339: sw_n = 1, sw_k = ldb). */
TP_API int tp_maxplus_fwd_strided(int dtype,
                           int64_t B1, int64_t B2, int64_t M, int64_t N, int64_t K,
                           const void* x, int64_t sx_b1, int64_t sx_b2, int64_t sx_m, int64_t sx_k,
                           const void* w, int64_t sw_b1, int64_t sw_b2, int64_t sw_n, int64_t sw_k,
                           const float* bias,
                           float* y, int64_t sy_b1, int64_t sy_b2, int64_t sy_m, int64_t sy_n,
                           int32_t* argmax, int64_t sa_b1, int64_t sa_b2, int64_t sa_m, int64_t sa_n,
                           float scale, void* stream);

/* Column-sharded max-plus GEMM with the all-gather fused into the epilogue.
 * This rank computes the columns [col0, col0 + N_shard) of y = max_k(x + w):
 * x [M,K] (row stride ldx), w_shard [N_shard,K] (row stride ldw), optional
 * bias_shard [N_shard].  Every output (and its int32 argmax, when argmax_dst is
 * not NULL) is stored into each of the n_dst (1..8) full-size row-major
 * buffers y_dst[d] [M, ldy] (argmax_dst[d] [M, ldy]) at column col0 + n.
 * y_dst[0] / argmax_dst[0] must be this device's memory; the others may be
 * peer buffers of the other ranks of one NVLink domain (P2P-mapped), so one
 * launch per rank fills every rank's full output -- no separate all-gather.
 * Synchronising the ranks around the launch is the caller's job.  Same
 * numerics as tp_maxplus_fwd (bit-exact values and argmax).  Shards that the
 * TMA kernel does not take (small or unaligned) are computed locally and then
 * copied into the other destinations.  Replaces the reference's single-device
 * forward (tropformer.py:127-145) for the multi-GPU sweep. */
TP_API int tp_maxplus_fwd_sharded(int64_t M, int64_t N_shard, int64_t K,
                                  const float* x, int64_t ldx,
                                  const float* w_shard, int64_t ldw,
                                  const float* bias_shard,
                                  float* const* y_dst, int32_t* const* argmax_dst, int n_dst,
                                  int64_t ldy, int64_t col0, void* stream);

/* Smooth (Maslov) forward: y[m,n] = (tau*log(sum_k exp(s[m,n,k]/tau)) [+bias[n]]) * scale.
 * tau = 1 is the TSRN tropical attention score LSE_c(Q+K)
 * (research/tsrn_dml.py:438-460, tsrn_dml.py:348-368); general tau is
 * tropical_logsumexp (research/tropical_optimizers.py:750-763) and the smooth
 * branch of _tropical_max (tropformer.py:95-97).  Same stride conventions as
 * tp_maxplus_fwd_strided.  Accuracy: relative 1e-5 of an fp64 evaluation. */
TP_API int tp_maxplus_lse_fwd_strided(int dtype, float tau,
                               int64_t B1, int64_t B2, int64_t M, int64_t N, int64_t K,
                               const void* x, int64_t sx_b1, int64_t sx_b2, int64_t sx_m, int64_t sx_k,
                               const void* w, int64_t sw_b1, int64_t sw_b2, int64_t sw_n, int64_t sw_k,
                               const float* bias,
                               float* y, int64_t sy_b1, int64_t sy_b2, int64_t sy_m, int64_t sy_n,
                               float scale, void* stream);

/* ======================================================================== *
 *  Max-plus backward
 * ======================================================================== */

/* Argmax (hard) backward -- autograd of scores.max(-1).values in eval mode
 * (tropformer.py:141, tropformer.py:93-94):
 *   gx[m,k] = sum_{n: argmax[m,n]==k} gy[m,n] * scale
 *   gw[n,k] = sum_{m: argmax[m,n]==k} gy[m,n] * scale
 *   gbias[n] = sum_m gy[m,n] * scale        (gbias may be NULL)
 * gx, gw are overwritten (zeroed, then scattered).  Strided/batched like the
 * forward; gx uses x's strides (sgx_*), gw uses w's (sgw_*).  gw may be NULL.
 * Summation order differs from torch: results agree to fp32 rounding. */
TP_API int tp_maxplus_bwd_argmax_strided(int64_t B1, int64_t B2, int64_t M, int64_t N, int64_t K,
                                  const int32_t* argmax, int64_t sa_b1, int64_t sa_b2, int64_t sa_m, int64_t sa_n,
                                  const float* gy, int64_t sg_b1, int64_t sg_b2, int64_t sg_m, int64_t sg_n,
                                  float* gx, int64_t sgx_b1, int64_t sgx_b2, int64_t sgx_m, int64_t sgx_k,
                                  float* gw, int64_t sgw_b1, int64_t sgw_b2, int64_t sgw_n, int64_t sgw_k,
                                  float* gbias, float scale, void* stream);

/* Workspace bytes needed by tp_maxplus_bwd_smooth for `batch` (M, N, K)
 * problems: six [M][N] stat planes per batch (three, and the same three
 * transposed for the input-gradient pass), plus per-slice partial sums
 * when the gradient outputs are too small to fill the GPU and the reduced
 * index is cut into slices (a function of the shapes only). */
TP_API int64_t tp_maxplus_bwd_smooth_workspace_bytes(int64_t batch, int64_t M, int64_t N,
                                                     int64_t K);

/* Smooth backward on `batch` contiguous row-major problems x[b][M][K],
 * w[b][N][K], gy[b][M][N] (mode TP_BWD_STE or TP_BWD_LSE; p = softmax(s/tau)
 * over k):
 *   STE (tropformer.py:133-139, TropicalLinear train mode):
 *        dS = gy * p * (1 + (s - sum_k p*s)/tau)
 *   LSE (tropformer.py:95-97 smooth _tropical_max; the intent of
 *        cuda/maxplus_gemm.cu:181-259):  dS = gy * p
 *   gx[b,m,k] = sum_n dS, gw[b,n,k] = sum_m dS, gbias[n] = sum_{b,m} gy[b,m,n].
 * gx, gw overwritten; gw and gbias may be NULL.  workspace must hold
 * tp_maxplus_bwd_smooth_workspace_bytes(batch,M,N,K) bytes, 16-byte aligned.
 * Deterministic (no atomics).  batch <= 65535.  Tolerance vs fp64: 1e-5
 * relative to the gradient scale. */
TP_API int tp_maxplus_bwd_smooth(int mode, float tau, int dtype,
                                 int64_t batch, int64_t M, int64_t N, int64_t K,
                                 const void* x, const void* w, const float* gy,
                                 float* gx, float* gw, float* gbias,
                                 void* workspace, int64_t workspace_bytes, void* stream);

/* The same, given the forward's maxima ref_max[b][m][n] = max_k (x + w) (before
 * bias; NULL: computed here).  Saves the stats pass's own max sweep over K
 * (a TropicalLinear forward has these values: the STE forward is the hard
 * max).  Any finite ref_max close to the max gives the same gradients within
 * the stated tolerance; a non-finite entry gives that output zero weight. */
TP_API int tp_maxplus_bwd_smooth_ref(int mode, float tau, int dtype,
                                     int64_t batch, int64_t M, int64_t N, int64_t K,
                                     const void* x, const void* w, const float* gy,
                                     const float* ref_max, float* gx, float* gw, float* gbias,
                                     void* workspace, int64_t workspace_bytes, void* stream);

/* Kernel choice for a forward with argmax: problems with M*N*K below this many
 * terms (default 2^30) run the per-term generic kernel, larger contiguous fp32
 * ones the TMA kernel, whose deferred argmax search has a fixed cost of about
 * 0.17 ms per launch.  Both give identical results.  Returns the previous
 * value; process-wide.  (Tuning; no reference counterpart.) */
TP_API int64_t tp_set_argmax_tma_min_terms(int64_t terms);

/* Schedule of the large fp32 forward (TMA kernel): 0 = each CTA takes whole
 * 128x128 tiles; 1 (default) = when K >= 4096 and the tile count leaves the
 * last wave partly idle (with argmax: at least 5% of the run), whole-tile
 * waves up to the last full one, then the remaining tiles either split
 * evenly by 64-k chunks over the CTAs or (argmax kernel, when a cost model
 * of the three options picks it) cut into two k-aligned halves, or left as
 * whole tiles; 2 = the even split whenever there are at least as many tiles
 * as CTAs; 3 = the k-aligned pieces (2 or 4 per tile, argmax kernel) whenever
 * K allows them, else as 2.  Tiles shared by CTAs are merged exactly (values
 * and argmax identical to the whole-tile schedule), using a stream-ordered
 * workspace from a library-owned pool (skipped under stream capture).
 * Co-residency: in the even split (mode 2, and mode 1 when it picks it) the
 * CTA holding a tile's head chunks waits for the LATER CTA that computes its
 * tail, so every CTA of the persistent grid (one per SM) must be resident at
 * once -- true on a whole GPU, not under an SM partition (MPS thread
 * percentage, green contexts).  There use mode 0 or 3 (k-aligned pieces wait
 * only on pieces of earlier rounds).  A wait that cannot complete ends after
 * the wait budget with TP_DEVERR_FLAG_TIMEOUT in tp_device_error().  Returns
 * the previous mode; process-wide.  (Tuning; no reference counterpart.) */
TP_API int tp_set_stream_k(int mode);

/* Smooth (STE / LSE) backward: 1 (default) lets shapes that allow it form gx
 * and gW in one pass (one exponential per term instead of one per gradient;
 * fp32, M, N, K multiples of 4, gx tiles filling the GPU, gW partials of at
 * most 64 MiB), 0 keeps one pass per gradient.  Both are deterministic and
 * agree to fp32 summation order.  Returns the previous setting. */
TP_API int tp_set_smooth_fused(int enable);

/* ======================================================================== *
 *  TSRN attention prologue (research/tsrn_dml.py:472-500: q_norm / k_norm,
 *  rope, and the view/permute to heads) in one pass.  qkv: [B*T, ld] rows, the
 *  Q, K, V projections of token (b, t) at columns [0, H*dh), [koff, koff+H*dh),
 *  [voff, voff+H*dh).  Per head: LayerNorm over dh channels (biased variance,
 *  eps) with q_gamma/q_beta (Q) or k_gamma/k_beta (K), then the rotary
 *  embedding of position pos0 + t: channel c < dh/2 paired with c + dh/2,
 *  out_c = x_c cos - x_{c+dh/2} sin, out_{c+dh/2} = x_{c+dh/2} cos + x_c sin,
 *  cos/sin from tables [npos, dh/2] (row p = position p).  Outputs Q, K, V are
 *  [B, H, T, dh] contiguous (the layout tp_tsrn_attention_fwd reads).  dh even,
 *  at most 128.  (Replaces the reference's PyTorch chain; no C counterpart.)
 * ======================================================================== */
TP_API int tp_tsrn_attention_prologue(int64_t B, int64_t T, int64_t H, int64_t dh,
                                      const float* qkv, int64_t ld, int64_t koff, int64_t voff,
                                      const float* q_gamma, const float* q_beta,
                                      const float* k_gamma, const float* k_beta, float eps,
                                      const float* cos_table, const float* sin_table,
                                      int64_t npos, int64_t pos0, float* Q, float* K, float* V,
                                      void* stream);

/* Backward of LayerNorm over rows of D channels (training): the pre-norms of
 * the TSRN block's tropical branches (research/tsrn_dml.py:1096-1106,
 * nn.LayerNorm(d_model) before the attention, the reservoir and the SSM).
 * x [rows, D] is the LayerNorm's input, dy the gradient of its output; writes
 * dx [rows, D] and, when not NULL, dgamma [D] and dbeta [D] (the row
 * statistics are recomputed; gamma NULL means ones).  D a multiple of 128, at
 * most 1024; x, dy, dx, gamma 16-byte aligned.  workspace:
 * tp_layernorm_bwd_workspace_bytes(rows, D) bytes (-1: unsupported D) for the
 * parameter gradients' per-block partials, summed in a fixed order
 * (deterministic).  (Replaces PyTorch's LayerNorm backward; no C counterpart
 * in the reference.) */
TP_API int64_t tp_layernorm_bwd_workspace_bytes(int64_t rows, int64_t D);
TP_API int tp_layernorm_bwd(int64_t rows, int64_t D, const float* x, const float* dy,
                            const float* gamma, float eps, float* dx, float* dgamma,
                            float* dbeta, void* workspace, int64_t workspace_bytes,
                            void* stream);

/* Backward of tp_tsrn_attention_prologue (training): from the gradients of Q,
 * K, V ([B, H, T, dh] contiguous) and the projections qkv, the gradient of qkv
 * (dqkv, same [B*T, ld] layout: Q, K, V columns at 0, koff, voff) and of the
 * four LayerNorm parameters, dparams [4][dh] = d q_gamma, d q_beta,
 * d k_gamma, d k_beta (the autograd of research/tsrn_dml.py:472-500; the
 * LayerNorm statistics are recomputed, the rotation transposed).  workspace:
 * tp_tsrn_attention_prologue_bwd_workspace_bytes(B, T, H, dh) bytes for the
 * parameter gradients' per-block partials, summed in a fixed order
 * (deterministic).  (Replaces the reference's PyTorch chain; no C counterpart.) */
TP_API int64_t tp_tsrn_attention_prologue_bwd_workspace_bytes(int64_t B, int64_t T, int64_t H,
                                                              int64_t dh);
TP_API int tp_tsrn_attention_prologue_bwd(int64_t B, int64_t T, int64_t H, int64_t dh,
                                          const float* qkv, int64_t ld, int64_t koff,
                                          int64_t voff, const float* q_gamma,
                                          const float* k_gamma, float eps,
                                          const float* cos_table, const float* sin_table,
                                          int64_t npos, int64_t pos0, const float* dQ,
                                          const float* dK, const float* dV, float* dqkv,
                                          float* dparams, void* workspace,
                                          int64_t workspace_bytes, void* stream);

/* ======================================================================== *
 *  Fused TSRN tropical top-k attention, forward (inference)
 *  Replaces research/tsrn_dml.py:462-548 (TropicalAttention.forward) from the
 *  scores on: the tropical score (:438-460, log-sum-exp over channels), the
 *  ALiBi bias (:509-514), the causal mask (:516-518), the top-k threshold
 *  (:520-521), the softmax and the product with V (:522-524).  Q/K/V come
 *  after the projections, QK-norm and RoPE.
 *    S[i,j] = log sum_c exp(Q[i,c] + K[j,c]) - slope[h] * |i - (j - Tc)|
 *             (-inf when causal and j - Tc > i)
 *    thr_i  = top_k-th largest of S[i,:] (ties counted, as torch.topk)
 *    out[i] = sum over {j : S[i,j] >= thr_i} of softmax(S[i,:])_j * V[j]
 *  Q [B,H,T,dh], K and V [B,H,Tkv,dh] contiguous fp32; keys j < Tc are the
 *  cross-window cached keys (positions j - Tc < 0), Tkv = Tc + T when they
 *  are used.  alibi_slopes [H].  Two kernels:
 *    tensor cores (dh <= 96, top_k <= 16, any Tkv): the exp-feature dots as
 *      3xTF32 tcgen05 MMAs into tensor memory, two passes over the keys;
 *    CUDA cores (dh <= 128, top_k <= 64, Tkv <= 6144): fp32 FMA dots, the
 *      score block of 16 rows in shared memory.
 *  tp_tsrn_attention_set_path selects; the default takes the tensor-core
 *  kernel where it applies and T >= 128, else the CUDA-core kernel (and
 *  tensor cores again beyond the CUDA-core limits).  The scores match the reference's fp32
 *  log-sum-exp within 1e-5; rows whose top_k-th and next scores lie within
 *  that distance may select differently.
 *  workspace: tp_tsrn_attention_workspace_bytes(...) bytes (enough for either
 *  kernel), 16-byte aligned.
 * ======================================================================== */
TP_API int64_t tp_tsrn_attention_workspace_bytes(int64_t B, int64_t H, int64_t T, int64_t Tkv,
                                                 int64_t dh);
TP_API int tp_tsrn_attention_fwd(int64_t B, int64_t H, int64_t T, int64_t Tkv, int64_t Tc,
                                 int64_t dh, const float* Q, const float* K, const float* V,
                                 const float* alibi_slopes, int top_k, int causal, float* out,
                                 void* workspace, int64_t workspace_bytes, void* stream);

/* Training form of the fused attention: the sparse backward of the reference
 * module's autograd (research/tsrn_dml.py:438-460, :509-524 differentiated;
 * the top-k threshold detached, as the reference detaches it).
 *
 * tp_tsrn_attention_fwd_lists: tp_tsrn_attention_fwd on the tensor-core
 *   kernel (dh <= 96, top_k <= 16; else TP_ERR_UNSUPPORTED) that also saves,
 *   per query row (b, h, i), its kept keys and softmax weights:
 *   kept_keys [B*H*T][TP_ATT_LIST] int32 (-1 past the row's entries),
 *   kept_weights [B*H*T][TP_ATT_LIST] fp32, kept_lse [B*H*T][TP_ATT_LIST] fp32
 *   (L_ij = logsumexp_c(Q_ic + K_jc): the kernel's score with its ALiBi term
 *   added back), kept_count [B*H*T] int32 (-1 when ties kept more keys than
 *   the lists hold: use a dense backward then).
 * tp_tsrn_attention_bwd_rows: per row, dP = dO_i . V_j and
 *   dS = P (dP - sum P dP) for every kept j, and
 *   dQ_i = sum_j dS_ij exp(Q_i + K_j - L_ij); stores dS per entry (entry_ds
 *   [B*H*T][TP_ATT_LIST]).  S = B*H.  Keys outside [0, Tkv) (in these and in
 *   tp_tsrn_attention_bwd_group) count as empty slots.
 * tp_tsrn_attention_bwd_group: groups the entries of each slice by key,
 *   rows ascending inside a key (a stable counting sort, one CTA per slice;
 *   Tkv up to 17000 keys, else TP_ERR_TOO_LARGE): entry ids
 *   (row * TP_ATT_LIST + slot) into order [S*T*TP_ATT_LIST] (slice s's in its
 *   own segment from s*T*TP_ATT_LIST), and per key (slice * Tkv + j) the start
 *   key_begin and length key_count of its run.
 * tp_tsrn_attention_bwd_keys: dK_j = sum_i dS_ij exp(Q_i + K_j - L_ij) and
 *   dV_j = sum_i P_ij dO_i over each key's run.  Every key of every slice is
 *   written (zero when nothing kept it).  All three backward kernels add in a
 *   fixed order: results repeat bit for bit. */
#define TP_ATT_LIST 32
TP_API int tp_tsrn_attention_fwd_lists(int64_t B, int64_t H, int64_t T, int64_t Tkv, int64_t Tc,
                                       int64_t dh, const float* Q, const float* K,
                                       const float* V, const float* alibi_slopes, int top_k,
                                       int causal, float* out, int32_t* kept_keys,
                                       float* kept_weights, float* kept_lse,
                                       int32_t* kept_count, void* workspace,
                                       int64_t workspace_bytes, void* stream);
TP_API int tp_tsrn_attention_bwd_rows(int64_t S, int64_t T, int64_t Tkv, int64_t dh,
                                      const float* Q, const float* K, const float* V,
                                      const float* dO, const int32_t* kept_keys,
                                      const float* kept_weights, const float* kept_lse,
                                      const int32_t* kept_count, float* dQ, float* entry_ds,
                                      void* stream);
TP_API int tp_tsrn_attention_bwd_group(int64_t S, int64_t T, int64_t Tkv,
                                       const int32_t* kept_keys, int32_t* order,
                                       int32_t* key_begin, int32_t* key_count, void* stream);
TP_API int tp_tsrn_attention_bwd_keys(int64_t S, int64_t T, int64_t Tkv, int64_t dh,
                                      const float* Q, const float* K, const float* dO,
                                      const float* kept_weights, const float* kept_lse,
                                      const float* entry_ds, const int32_t* order,
                                      const int32_t* key_begin, const int32_t* key_count,
                                      float* dK, float* dV, void* stream);

/* Kernel choice of tp_tsrn_attention_fwd for this process: TP_ATT_PATH_AUTO
 * (tensor cores where supported and T >= 128, else CUDA cores within their
 * limits, else tensor cores), TP_ATT_PATH_CUDA_CORES,
 * or TP_ATT_PATH_TENSOR_CORES (shapes it does not support then return
 * TP_ERR_UNSUPPORTED).  Stores the previous choice in *previous when it is
 * not NULL.  (No reference counterpart.) */
#define TP_ATT_PATH_AUTO 0
#define TP_ATT_PATH_CUDA_CORES 1
#define TP_ATT_PATH_TENSOR_CORES 2
TP_API int tp_tsrn_attention_set_path(int path, int* previous);

/* ======================================================================== *
 *  Echo-state reservoir recurrences, forward (inference), whole sequence in
 *  one launch.  h_{-1} = 0; for t = 0..T-1, H[:, t] = h_t.
 *
 *  tp_esn_gru_fwd replaces the per-timestep loop of the GRU-gated
 *  EchoStateReservoir.forward (research/tsrn_dml.py:808-843, loop :834-840):
 *    z = sigmoid(h Wzh^T + Uz_t);  r = sigmoid(h Wrh^T + Ur_t)
 *    h~ = tanh((r * h) Ws^T + U_t);  h = (1 - z) * h + z * h~
 *  with U = W_in(x), Uz = U Wz_u^T + b_z, Ur = U Wr_u^T + b_r.
 *
 *  tp_esn_leaky_fwd replaces the loop of the leaky EchoStateReservoir.forward
 *  (tsrn_gpu.py:466-487):  h = (1 - lk) * h + lk * tanh(h Ws^T + U_t),
 *  U = W_in(x); `leak` points to the device scalar lk = sigmoid(leak).
 *
 *  U, Uz, Ur, H: [B, T, dr] contiguous fp32.  Weights [dr, dr] with row
 *  stride ld >= dr (Wzh / Wrh may be the first dr columns of W_z / W_r
 *  weights in place: ld = 2 dr); Ws = the spectrally scaled W_res.  Each
 *  group of batch rows runs on one thread-block cluster (no grid barrier, no
 *  waits beyond hardware cluster barriers).  Weights that do not fit in
 *  shared memory are read from L2, which needs dr and ld multiples of 4 and
 *  16-byte aligned weights (else TP_ERR_UNSUPPORTED).  Matches the reference
 *  within the fp32 rounding of the dot products (summation order) and of
 *  sigmoid / tanh (1e-5 on h).
 * ======================================================================== */
TP_API int tp_esn_gru_fwd(int64_t B, int64_t T, int64_t dr, const float* U, const float* Uz,
                          const float* Ur, const float* Wzh, int64_t ld_wzh, const float* Wrh,
                          int64_t ld_wrh, const float* Ws, int64_t ld_ws, float* H,
                          void* stream);
TP_API int tp_esn_leaky_fwd(int64_t B, int64_t T, int64_t dr, const float* U, const float* Ws,
                            int64_t ld_ws, const float* leak, float* H, void* stream);

/* Segments of a longer sequence: T steps starting from state h0 ([B] rows of
 * ld_h0 >= dr floats; NULL: zeros), with U, Uz, Ur and H rows t_stride >= T
 * steps apart (a time window [t0, t0 + T) of [B, t_stride, dr] tensors is the
 * base pointer + t0 * dr).  Running [0, T) in consecutive segments, each
 * starting from the previous segment's last state H[:, t0 - 1], equals one
 * call over [0, T) bit for bit. */
TP_API int tp_esn_gru_fwd_seg(int64_t B, int64_t T, int64_t t_stride, int64_t dr,
                              const float* U, const float* Uz, const float* Ur,
                              const float* Wzh, int64_t ld_wzh, const float* Wrh,
                              int64_t ld_wrh, const float* Ws, int64_t ld_ws, const float* h0,
                              int64_t ld_h0, float* H, void* stream);
TP_API int tp_esn_leaky_fwd_seg(int64_t B, int64_t T, int64_t t_stride, int64_t dr,
                                const float* U, const float* Ws, int64_t ld_ws,
                                const float* leak, const float* h0, int64_t ld_h0, float* H,
                                void* stream);

/* Backward through time of both recurrences (training), one launch each:
 * the reverse-time loops of reservoir autograd (research/tsrn_dml.py:834-840
 * and tsrn_gpu.py:480-484 differentiated), with the per-step factors formed
 * beforehand for all steps.  g = 0 after the last step; for t = T-1 .. 0:
 *   GRU (tp_esn_gru_bwd):   dh = dH_t + g;  dAh_t = dh fa_t;
 *     dm = dAh_t Ws;  dAr_t = dm fr_t;  dAz_t = dh fz_t;
 *     g = dh keep_t + dm r_t + dAz_t Wzh + dAr_t Wrh
 *   with fa = z (1 - h~^2), fz = (h~ - h_{t-1}) z (1 - z),
 *   fr = h_{t-1} r (1 - r), keep = 1 - z and r the reset gate; dAh, dAz, dAr
 *   are the gradients of the pre-activations of h~, z and r.
 *   leaky (tp_esn_leaky_bwd): dh = dH_t + g;  dA_t = dh fa_t;
 *     g = dh (1 - lk) + dA_t Ws;  dHs_t = dh   (fa = lk (1 - s^2)).
 * Weights are passed TRANSPOSED (WzhT = Wzh^T etc., [dr, dr], row stride
 * ld >= dr).  All [B, T, dr] tensors contiguous fp32.  Same cluster layout,
 * limits and bounded waits as the forward; matches the reference loop
 * within fp32 rounding of the dot products.  (No reference counterpart: the
 * reference differentiates its Python loop with autograd.) */
TP_API int tp_esn_gru_bwd(int64_t B, int64_t T, int64_t dr, const float* dH, const float* fa,
                          const float* fz, const float* fr, const float* keep, const float* r,
                          const float* WzhT, int64_t ld_wz, const float* WrhT, int64_t ld_wr,
                          const float* WsT, int64_t ld_ws, float* dAh, float* dAz, float* dAr,
                          void* stream);
TP_API int tp_esn_leaky_bwd(int64_t B, int64_t T, int64_t dr, const float* dH, const float* fa,
                            const float* WsT, int64_t ld_ws, const float* leak, float* dA,
                            float* dHs, void* stream);

/* x = hi + lo for n fp32 values: hi = x with its 13 low mantissa bits cleared
 * (exact in TF32), lo = x - hi (exact; 0 where x is not finite).  x, hi, lo
 * 16-byte aligned.  With it, three TF32 tensor-core GEMMs (hi.hi + hi.lo +
 * lo.hi) reproduce an fp32 GEMM to ~2e-6 relative: the nn.Linear projections
 * around the tropical branches (research/tsrn_dml.py:462-548, 808-843,
 * 917-980) run that way in inference.  (Utility; no reference counterpart.) */
TP_API int tp_split_tf32(const float* x, int64_t n, float* hi, float* lo, void* stream);

/* The same split written row-concatenated: for x [rows, cols] (row-major,
 * cols a multiple of 4), out [rows, nparts cols] (nparts 1 to 3) holds the
 * parts of each row side by side, part p the lo part where bit p of lo_mask is
 * set, else the hi part.  With A = [xh | xl] (lo_mask 2) and B = [wl | wh]
 * (lo_mask 1), A B^T is the two correction products hi.lo + lo.hi as one
 * TF32 GEMM of depth 2 cols, accumulated onto hi.hi (its own GEMM: the small
 * terms are not summed inside the tensor cores' accumulation of the large
 * ones).  x, out 16-byte aligned.  (Utility; no reference counterpart.) */
TP_API int tp_split_tf32_cat(const float* x, int64_t rows, int64_t cols, float* out,
                             int nparts, int lo_mask, void* stream);

/* Copy `rows` rows of width_bytes from src (row pitch src_pitch bytes) to dst
 * (pitch dst_pitch), host or device memory on either side (pinned host memory
 * for an asynchronous copy), on `stream`: the strided time windows the
 * segmented reservoir entries read.  (Utility; no reference counterpart.) */
TP_API int tp_memcpy2d_async(void* dst, int64_t dst_pitch, const void* src, int64_t src_pitch,
                             int64_t width_bytes, int64_t rows, void* stream);

/* ======================================================================== *
 *  Maslov softmax of attention scores, optionally gated (one warp per row).
 *
 *  tp_maslov_softmax_fwd replaces MaslovTemperature.forward
 *  (tropformer.py:206-212) and, with C != NULL, the score blend before it in
 *  DTNAttention.forward (deep_tropical_net.py:152-160):
 *    s = C ? g*T + (1-g)*C : T;   s = -1e9 where mask != 0;
 *    P = softmax(s / tau[h]) over the last dimension.
 *  T, C, P: [B, H, Lq, Lk] contiguous fp32 (T = the tropical scores, C = the
 *  classical ones); g: the gate sigmoid(score_gate(x)) read at
 *  g[b*gsb + i*gsi + h*gsh] (NULL iff C is NULL); mask: bytes, nonzero where
 *  the module's mask == 0, at mask[b*msb + h*msh + i*msi + j*msj] (strides
 *  may be 0 to broadcast), or NULL; tau: [H] device temperatures.  The blend
 *  and the division round like the PyTorch expression; the softmax differs
 *  from PyTorch's only in exp rounding and summation order.
 *
 *  tp_maslov_softmax_bwd is the autograd backward of that chain, given P and
 *  dP = dL/dP: dz = P*(dP - sum_j P*dP), ds = dz / tau (0 where masked),
 *  dT = g*ds (ds without C), dC = (1-g)*ds, dg[b,i,h] (strides of g) =
 *  sum_j ds*T - sum_j ds*C, dtau_rows[row] = sum_j dz*s (row = (b*H+h)*Lq+i);
 *  the caller forms dL/dtau[h] = -(sum of h's dtau_rows) / tau[h]^2.  Any
 *  output may be NULL.
 * ======================================================================== */
TP_API int tp_maslov_softmax_fwd(int64_t B, int64_t H, int64_t Lq, int64_t Lk, const float* T,
                                 const float* C, const float* g, int64_t gsb, int64_t gsi,
                                 int64_t gsh, const unsigned char* mask, int64_t msb,
                                 int64_t msh, int64_t msi, int64_t msj, const float* tau,
                                 float* P, void* stream);
TP_API int tp_maslov_softmax_bwd(int64_t B, int64_t H, int64_t Lq, int64_t Lk, const float* T,
                                 const float* C, const float* g, int64_t gsb, int64_t gsi,
                                 int64_t gsh, const unsigned char* mask, int64_t msb,
                                 int64_t msh, int64_t msi, int64_t msj, const float* tau,
                                 const float* P, const float* dP, float* dT, float* dC,
                                 float* dg, float* dtau_rows, void* stream);

/* ======================================================================== *
 *  Tropical (max-plus) diagonal SSM scan  (research/tsrn_dml.py:917-980)
 *
 *    u[b,t,c] = bb[b,t,c] + xx[b,t,c]     (xx may be NULL: u = bb)
 *    h[b,-1,c] = h0 ? h0[b,c] : h_init
 *    h[b,t,c]  = max(a[c] + h[b,t-1,c], u[b,t,c])   sequential fp32 recurrence
 *
 *  All [B,T,C] tensors are contiguous with C fastest; a is [C]; h0, gh0 are
 *  [B,C].  Results are bit-exact with the sequential recurrence for every
 *  mode: rounding is monotone, so fl(a + max(p,q)) = max(fl(a+p), fl(a+q))
 *  and a carry entering a time segment can be replayed exactly.
 *  win_mask (optional, [B, ceil(T/32), C] uint32): bit (t%32) of word
 *  [b, t/32, c] is 1 when the input won step t (u >= a + h_prev; the input
 *  wins ties, matching torch.cummax's last-index rule used by the reference
 *  closed form, research/tsrn_dml.py:968).
 * ======================================================================== */
TP_API int tp_scan_fwd(int64_t B, int64_t T, int64_t C,
                const float* bb, const float* xx, const float* a,
                float h_init, const float* h0,
                float* h, uint32_t* win_mask, void* stream);

/* Argmax-path backward of tp_scan_fwd.  Needs either win_mask (from the
 * forward) or (bb, xx, h) to recompute the winners.  With G the total
 * gradient reaching h[b,t,c]:
 *   gu[b,t,c] = win ? G : 0     (= grad of bb and of xx)
 *   ga[c]     = sum_{b,t} (!win ? G : 0)      (ga may be NULL)
 *   gh0[b,c]  = (!win at t=0) ? G[b,0,c] : 0  (gh0 may be NULL)
 * ga is reduced deterministically through `workspace` (B*C floats, may be
 * NULL only when ga is NULL). */
TP_API int tp_scan_bwd(int64_t B, int64_t T, int64_t C,
                const float* gh,
                const float* bb, const float* xx, const float* a,
                float h_init, const float* h0, const float* h,
                const uint32_t* win_mask,
                float* gu, float* ga, float* gh0,
                float* workspace, void* stream);

/* ---- chunk-parallel scan --------------------------------------------------
 * The same recurrence for shapes whose B * C lanes cannot fill the GPU (the
 * kernels above run one warp per 32 channels of a batch row: B=2, C=1024 is
 * 64 warps): time is cut into chunks of `chunk` steps (a multiple of 32; 0 =
 * the library's choice, tp_scan_chunk_length) that run in parallel.  The
 * forward computes each chunk from -inf, then every chunk's exact starting
 * state (the carry through a chunk is `chunk` rounded adds of a, combined
 * with the chunk's own result by a max; rounding is monotone, so the two
 * separate exactly), then reruns every chunk from it: h and win_mask are
 * BIT-EXACT with tp_scan_fwd.  The backward likewise finds the exact
 * gradient entering every chunk, so gu and gh0 are bit-exact with
 * tp_scan_bwd; ga sums per-chunk partials (ascending batch, descending
 * chunk), which agrees with tp_scan_bwd's single running sum to rounding.
 * Caller-owned workspace of tp_scan_chunked_workspace_bytes(B, T, C, chunk)
 * bytes, 256-byte aligned (TP_ERR_WORKSPACE / TP_ERR_MISALIGNED otherwise).
 * Reference: research/tsrn_dml.py:961-972 evaluates the scan in parallel over
 * T through a closed form (t*A + cummax), whose rounding differs from the
 * recurrence; this mode is parallel over T without that difference. */
TP_API int64_t tp_scan_chunked_workspace_bytes(int64_t B, int64_t T, int64_t C, int chunk);
TP_API int tp_scan_chunk_length(int64_t B, int64_t T, int64_t C);
TP_API int tp_scan_fwd_chunked(int64_t B, int64_t T, int64_t C,
                               const float* bb, const float* xx, const float* a,
                               float h_init, const float* h0,
                               float* h, uint32_t* win_mask, int chunk,
                               void* workspace, int64_t workspace_bytes, void* stream);
TP_API int tp_scan_bwd_chunked(int64_t B, int64_t T, int64_t C,
                               const float* gh,
                               const float* bb, const float* xx, const float* a,
                               float h_init, const float* h0, const float* h,
                               const uint32_t* win_mask,
                               float* gu, float* ga, float* gh0, int chunk,
                               void* workspace, int64_t workspace_bytes, void* stream);

/* Allocation-free form of tp_scan_bwd, for callers that cannot allocate
 * device memory themselves: a thin FFI binding that only forwards pointers of
 * buffers some other runtime already owns, or a process whose device memory
 * belongs entirely to another framework's pool, where a raw cudaMalloc would
 * synchronise the device and fragment that pool.  There is no counterpart in
 * the reference.
 *
 * Same arguments, results and validation as tp_scan_bwd, without the
 * workspace: the [B, C] partial sums behind ga live in one fixed array of this
 * library's device memory (1 MiB per GPU that loads the library, held until
 * the process exits).  Limit: when ga is requested and T > 0, B*C <= 262144,
 * else the call returns TP_ERR_TOO_LARGE (after the argument checks of
 * tp_scan_bwd) and launches nothing.  The array's address is cached per
 * device: do not call after cudaDeviceReset in the same process.  No allocation or free
 * happens in this call.  The first call on a device looks up that device's
 * array address (cudaGetSymbolAddress) -- make that first call outside any
 * stream capture.  Every entry of the array that a call reads it has written
 * first, so nothing needs clearing, but all calls share the one array: calls
 * whose kernels overlap on the GPU (other streams, other host threads) race
 * and must be serialised by the caller. */
TP_API int tp_scan_bwd_noalloc(int64_t B, int64_t T, int64_t C,
                               const float* gh,
                               const float* bb, const float* xx, const float* a,
                               float h_init, const float* h0, const float* h,
                               const uint32_t* win_mask,
                               float* gu, float* ga, float* gh0, void* stream);

/* Exact bf16 -> fp32 widening of n contiguous elements (dst may not overlap
 * src).  Lets bf16-stored GEMM operands (the bf16 half of the M=N=K sweep)
 * run on the fp32 TMA kernel: the results equal fp32 max-plus on the upcast
 * inputs bit for bit.  No reference counterpart (the reference's fp16 kernel
 * template, cuda/maxplus_gemm.cu:18, was never instantiated). */
TP_API int tp_convert_bf16_to_f32(int64_t n, const void* src, float* dst, void* stream);

/* ======================================================================== *
 *  Roofline probe: register-only add+max loop measuring the CUDA-core
 *  max-plus term rate.  form 0: FADD + 2-input FMNMX per term;
 *  form 1: packed add.f32x2 + 3-input max per two terms; form 2: form 1 with
 *  NaN-propagating max; form 3: two scalar adds + 3-input NaN max per two
 *  terms; form 4: forms 2 and 3 alternating; form 5: packed add.bf16x2 +
 *  max.bf16x2 per two terms (bf16 arithmetic); form 6: form 5 with the
 *  NaN-propagating max; form 7: fp32 fma (a term is one FMA, 2 flops: the
 *  CUDA-core peak of dot products); form 8: the smooth backward's per-term
 *  shape with one ex2.approx per term (a term is one exponential: the SFU
 *  peak of the STE / LSE passes); form 9: packed fp32 FMA pairs
 *  (fma.rn.f32x2, a term is one FMA).  Each of `threads` threads runs `iters`
 *  iterations of 128 terms; the caller times the launch.  sink receives one float per
 *  thread (keeps the work live).
 * ======================================================================== */
TP_API int tp_probe_addmax(int form, int64_t blocks, int64_t threads, int64_t iters,
                    float* sink, void* stream);

/* ======================================================================== *
 *  Reference-compatible symbols (cuda/maxplus_gemm.cu:297-341) so that the
 *  reference's ctypes binding can load this library in place of
 *  maxplus_gemm.so.  Same signatures and argument meaning as declared there
 *  (W first, then x), fp32, legacy default stream, void return.  Unlike the
 *  reference they compute -inf-correct values, and maxplus_backward_cuda
 *  OVERWRITES rather than accumulates (the reference binding zeroes first, so
 *  the observable result is the same).  Errors are reported through
 *  tp_last_error().
 * ======================================================================== */
TP_API void maxplus_forward_cuda(const float* W, const float* x, float* y, const float* bias,
                          int batch_size, int in_features, int out_features, bool use_tiled);
TP_API void maxplus_backward_cuda(const float* W, const float* x, const float* grad_y,
                           float* grad_W, float* grad_x, float* grad_bias,
                           float ste_temp, int batch_size, int in_features, int out_features);
TP_API void maxplus_matmul_cuda(const float* A, const float* B, float* C, int M, int K, int N);

/* Status of the last reference-compatible call on this host thread. */
TP_API int tp_last_error(void);

/* ---- device-side failures ------------------------------------------------
 * Every wait inside a kernel (TMA pipeline mbarriers, the reservoir's cluster
 * exchange, the stream-K merge flags) is bounded by a budget of %globaltimer
 * time.  A wait that runs out records a code in the device error word of its
 * GPU and the kernel returns early (its outputs are then incomplete), so the
 * context stays usable.  The word keeps the FIRST code recorded. */
#define TP_DEVERR_BARRIER_TIMEOUT 1   /* an mbarrier wait ran out of budget  */
#define TP_DEVERR_FLAG_TIMEOUT 2      /* a flag wait ran out of budget       */

/* Device-side error word of the current device: 0 when no kernel reported a
 * problem, else a TP_DEVERR_* code.  Synchronises with the device (it reads
 * device memory).  reset != 0 clears the word afterwards.  Returns
 * -cudaError_t on failure.  The word's address is cached per device for the
 * life of the process: do not call the library after cudaDeviceReset in the
 * same process. */
TP_API int tp_device_error(int reset);

/* Budget of every bounded device-side wait on the current device, in ns of
 * %globaltimer (default 2e9 = 2 s; accepted range [1e3, 6e10]).  Stores the
 * previous budget in *previous when it is not NULL.  Synchronous (a copy to
 * device memory): not during stream capture.  (No reference counterpart.) */
#define TP_WAIT_BUDGET_MIN_NS 1000LL
#define TP_WAIT_BUDGET_MAX_NS 60000000000LL
TP_API int tp_set_wait_budget_ns(int64_t ns, int64_t* previous);

/* Failure-path self-test: launches one single-warp kernel whose bounded wait
 * can never complete -- kind 0: an mbarrier phase that receives one of its
 * two arrivals; kind 1: the flag word at `flag` (device memory, caller keeps
 * it 0), polled with the same acquire-load wait the stream-K merges use.
 * After the wait budget the kernel records TP_DEVERR_BARRIER_TIMEOUT (kind 0)
 * or TP_DEVERR_FLAG_TIMEOUT (kind 1) and returns; nothing faults or hangs.
 * For tests of the error path (set a short budget first).  (No reference
 * counterpart.) */
TP_API int tp_selftest_bounded_wait(int kind, const unsigned* flag, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* TROPICAL_B200_H */
