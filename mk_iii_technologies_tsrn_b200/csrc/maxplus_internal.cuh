// maxplus_internal.cuh -- argument structs and launcher declarations shared
// between the kernel files and the C-ABI layer (capi.cu).
#pragma once

#include "common.cuh"

namespace tp {

// One strided, two-level batched max-plus problem (see tp_maxplus_fwd_strided).
// Legendre-Fenchel dual activation applied in a forward epilogue
// (tropformer.py:224-289, LFDualActivation), value only.  mode: -1 none,
// 0 primal f(v) = max_k(v*s_k + b_k), 1 dual f*(v) = max_j(v*x_j - f(x_j)),
// 2 blend g_n*f(v) + (1-g_n)*f*(v) with g = sigmoid(blend_gate) given per
// output column.  Products and sums are separately rounded, as the reference
// evaluates them (no fused multiply-add).
constexpr int LF_MAX_PIECES = 16;
struct LfAct {
  int mode;
  int pieces;
  const float* s;       // [pieces] slopes
  const float* b;       // [pieces] biases
  const float* xg;      // [pieces] x grid
  const float* gate;    // [N] sigmoid(blend_gate) (blend only)
};

// params staged in shared memory: sm[0..P) s, [16..) b, [32..) x_grid, [48..) f(x_j)
__device__ __forceinline__ void lf_stage(const LfAct& a, float* sm) {
  const int t = threadIdx.x;
  if (t < a.pieces) {
    sm[t] = a.s[t];
    sm[16 + t] = a.b[t];
    sm[32 + t] = a.xg[t];
    const float x = a.xg[t];
    float f = -__int_as_float(0x7f800000);
    bool nan = false;
    for (int k = 0; k < a.pieces; ++k) {
      const float piece = __fadd_rn(__fmul_rn(x, a.s[k]), a.b[k]);
      nan |= piece != piece;
      f = fmaxf(f, piece);
    }
    sm[48 + t] = nan ? __int_as_float(0x7fc00000) : f;
  }
}

__device__ __forceinline__ float lf_apply(const LfAct& a, const float* sm, int64_t n, float v) {
  const float NEG_INF = -__int_as_float(0x7f800000);
  float p = NEG_INF, d = NEG_INF;
  bool pnan = false, dnan = false;
  if (a.mode != 1) {
    for (int k = 0; k < a.pieces; ++k) {
      const float piece = __fadd_rn(__fmul_rn(v, sm[k]), sm[16 + k]);
      pnan |= piece != piece;
      p = fmaxf(p, piece);
    }
    if (pnan) p = __int_as_float(0x7fc00000);
    if (a.mode == 0) return p;
  }
  for (int j = 0; j < a.pieces; ++j) {
    const float piece = __fsub_rn(__fmul_rn(v, sm[32 + j]), sm[48 + j]);
    dnan |= piece != piece;
    d = fmaxf(d, piece);
  }
  if (dnan) d = __int_as_float(0x7fc00000);
  if (a.mode == 1) return d;
  const float g = a.gate[n];
  const float omg = __fsub_rn(1.0f, g);
  return __fadd_rn(__fmul_rn(g, p), __fmul_rn(omg, d));
}

struct StridedMaxPlus {
  int dtype;
  int64_t B1, B2, M, N, K;
  const void* x;
  int64_t sx_b1, sx_b2, sx_m, sx_k;
  const void* w;
  int64_t sw_b1, sw_b2, sw_n, sw_k;
  const float* bias;
  float* y;
  int64_t sy_b1, sy_b2, sy_m, sy_n;
  int32_t* am;
  int64_t sa_b1, sa_b2, sa_m, sa_n;
  float scale;
  float tau;
  LfAct act{-1, 0, nullptr, nullptr, nullptr, nullptr};   // forward epilogue (value only)
};

struct ScatterArgs {
  int64_t B1, B2, M, N, K;
  const int32_t* am;
  int64_t sa_b1, sa_b2, sa_m, sa_n;
  const float* gy;
  int64_t sg_b1, sg_b2, sg_m, sg_n;
  float* gx;
  int64_t sgx_b1, sgx_b2, sgx_m, sgx_k;
  float* gw;
  int64_t sgw_b1, sgw_b2, sgw_n, sgw_k;
  float* gbias;
  float scale;
};

struct SmoothArgs {
  int mode;
  float tau;
  int dtype;
  int64_t batch;  // contiguous batches: x[b] = x + b*M*K, w[b] = w + b*N*K, ...
  int64_t M, N, K;
  const void* x;
  const void* w;
  const float* gy;
  float* gx;
  float* gw;
  float* gbias;
  float* ws;  // per batch 3 planes of [M][N]: reference max, A, B; then, after all
              // batches, the same planes transposed ([N][M]) when `async_stage`
  bool async_stage;  // fp32, M, N, K multiples of 4: grad kernels stage with cp.async
  // Splits of the reduced index for gx (over n) and gw (over m); > 1 only when
  // the output tiles alone cannot fill the GPU.  Partial sums then go to
  // `part` ([batch][splits][rows][K], after the stat planes in the workspace)
  // and are added in split order.
  int64_t splits_x, splits_w;
  float* part;
  // optional [batch][M][N] maxima max_k(x + w) from the forward: the stats
  // pass then skips its own max pass
  const float* ref;
  // both gradients in one pass (smooth_fused_ok shapes, gw requested): the
  // per-row-tile gW partials go to `part` ([batch][ceil(M/64)][N][K])
  bool fused_gw;
};

// Number of slices the smooth backward cuts the reduced index Q into for an
// output of `rows` x K per batch.  Depends on the shapes only, so the
// workspace size is known before the call.
int64_t smooth_splits(int64_t batch, int64_t rows, int64_t Q, int64_t K);
// Workspace floats of the smooth backward (stat planes + split partials).
int64_t smooth_workspace_floats(int64_t batch, int64_t M, int64_t N, int64_t K);
bool smooth_fused_ok(int64_t batch, int64_t M, int64_t N, int64_t K);

// maxplus_generic.cu
int launch_maxplus_fwd_generic(const StridedMaxPlus& p, cudaStream_t stream);
int launch_maxplus_lse_fwd_generic(const StridedMaxPlus& p, cudaStream_t stream);
int launch_maxplus_bwd_argmax(const ScatterArgs& p, cudaStream_t stream);
int launch_maxplus_bwd_smooth(const SmoothArgs& p, cudaStream_t stream);
int launch_bf16_to_f32(const void* src, float* dst, int64_t n, cudaStream_t stream);
int launch_strided_zero(float* base, int64_t B1, int64_t B2, int64_t R, int64_t C, int64_t s_b1,
                        int64_t s_b2, int64_t s_r, int64_t s_c, cudaStream_t stream);
int launch_column_sum(const float* g, int64_t B1, int64_t B2, int64_t M, int64_t N, int64_t s_b1,
                      int64_t s_b2, int64_t s_m, int64_t s_n, float scale, float* out,
                      cudaStream_t stream);

// maxplus_tma.cu: large contiguous fp32 GEMM.  Returns TP_ERR_UNSUPPORTED
// when the problem does not meet its layout rules (caller falls back).
bool maxplus_tma_eligible(const StridedMaxPlus& p);
// smallest M*N*K for which a forward with argmax takes the TMA kernel
int64_t argmax_tma_min_terms();
int64_t set_argmax_tma_min_terms(int64_t terms);
int set_stream_k(int mode);
int launch_maxplus_fwd_tma(const StridedMaxPlus& p, cudaStream_t stream);
// Same, additionally storing every output into ndst (<= 8) further buffers
// at column offset col0 (same row strides as y / argmax).
int launch_maxplus_fwd_tma_dests(const StridedMaxPlus& p, float* const* ydst,
                                 int32_t* const* adst, int ndst, int64_t col0,
                                 cudaStream_t stream);

// scan.cu
struct ScanArgs {
  int64_t B, T, C;
  const float* bb;
  const float* xx;
  const float* a;
  float h_init;
  const float* h0;
  float* h;
  uint32_t* win;
  // backward
  const float* gh;
  const uint32_t* win_in;
  float* gu;
  float* ga;
  float* gh0;
  float* ws;
  int* err;
};
int launch_scan_fwd(const ScanArgs& p, cudaStream_t stream);
int launch_scan_bwd(const ScanArgs& p, cudaStream_t stream);
// scan_chunked.cu: chunk-parallel scan (workspace from the caller)
int scan_chunk_pick(int64_t B, int64_t T, int64_t C);
int64_t scan_chunked_workspace_bytes(int64_t B, int64_t T, int64_t C, int chunk);
int launch_scan_fwd_chunked(const ScanArgs& p, int chunk, void* ws, int64_t ws_bytes,
                            cudaStream_t stream);
int launch_scan_bwd_chunked(const ScanArgs& p, int chunk, void* ws, int64_t ws_bytes,
                            cudaStream_t stream);
// capi.cu: the pointer checks of tp_scan_bwd (shared with its allocation-free form)
int check_scan_bwd_pointers(int64_t T, const float* gh, const float* bb, const float* xx,
                            const float* a, const float* h0, const float* h,
                            const uint32_t* win_mask, const float* gu, const float* ga,
                            const float* gh0);
// capi.cu: failure-path self-test (tp_selftest_bounded_wait)
int launch_selftest_wait(int kind, const unsigned* flag, cudaStream_t stream);

// probe.cu
int launch_probe_addmax(int form, int64_t blocks, int64_t threads, int64_t iters, float* sink,
                        cudaStream_t stream);

// tsrn_attention.cu: fused TSRN tropical top-k attention forward
int64_t tsrn_attention_workspace_floats(int64_t B, int64_t H, int64_t T, int64_t Tkv, int64_t dh);
int launch_tsrn_attention_fwd(int64_t B, int64_t H, int64_t T, int64_t Tkv, int64_t Tc, int64_t dh,
                              const float* Q, const float* K, const float* V,
                              const float* slopes, int top_k, int causal, float* out,
                              float* ws, cudaStream_t stream);

// tsrn_attention_tc.cu: the same forward with the score contraction on tcgen05
int& tsrn_attention_path();   // TP_ATT_PATH_*
bool tsrn_attention_tc_supported(int64_t dh, int top_k);
int64_t tsrn_attention_tc_workspace_floats(int64_t B, int64_t H, int64_t T, int64_t Tkv);
int launch_tsrn_attention_tc(int64_t B, int64_t H, int64_t T, int64_t Tkv, int64_t Tc, int64_t dh,
                             const float* Q, const float* K, const float* V, const float* slopes,
                             int top_k, int causal, float* out, float* ws, cudaStream_t stream,
                             int* kj = nullptr, float* kp = nullptr, float* kl = nullptr,
                             int* kn = nullptr);
constexpr int TSRN_ATT_LIST = 32;   // kept keys per row in the saved lists (two halves of 16)
int launch_tsrn_attention_bwd_rows(int64_t S, int64_t T, int64_t Tkv, int64_t dh, const float* Q,
                                   const float* K, const float* V, const float* dO,
                                   const int* kj, const float* kp, const float* kl,
                                   const int* kn, float* dQ, float* eds, cudaStream_t stream);
int launch_tsrn_attention_bwd_group(int64_t S, int64_t T, int64_t Tkv, const int* kj, int* order,
                                    int* key_begin, int* key_count, cudaStream_t stream);
int launch_tsrn_attention_bwd_keys(int64_t S, int64_t T, int64_t Tkv, int64_t dh, const float* Q,
                                   const float* K, const float* dO, const float* kp,
                                   const float* eds, const float* kl, const int* order,
                                   const int* key_begin, const int* key_count, float* dK,
                                   float* dV, cudaStream_t stream);

// tsrn_prologue.cu: QK LayerNorm + rotary embedding + head-major layout of Q/K/V
int launch_tsrn_prologue(int64_t B, int64_t T, int64_t H, int64_t dh, const float* qkv, int64_t ld,
                         int64_t koff, int64_t voff, const float* qg, const float* qb,
                         const float* kg, const float* kb, float eps, const float* cosb,
                         const float* sinb, int64_t pos0, float* Q, float* K, float* V,
                         cudaStream_t stream);
int layernorm_bwd_blocks(int64_t rows);
bool layernorm_bwd_supported(int64_t D);
int launch_layernorm_bwd(int64_t rows, int64_t D, const float* x, const float* dy,
                         const float* gamma, float eps, float* dx, float* dgamma, float* dbeta,
                         float* part, cudaStream_t stream);
int tsrn_prologue_bwd_blocks(int64_t B, int64_t T, int64_t H);
int launch_tsrn_prologue_bwd(int64_t B, int64_t T, int64_t H, int64_t dh, const float* qkv,
                             int64_t ld, int64_t koff, int64_t voff, const float* qg,
                             const float* kg, float eps, const float* cosb, const float* sinb,
                             int64_t pos0, const float* dQ, const float* dK, const float* dV,
                             float* dqkv, float* dparams, float* part, cudaStream_t stream);

// esn.cu: echo-state reservoir recurrences (GRU-gated when gru, else leaky);
// W[0..2] = Wzh, Wrh, Ws for GRU, W[0] = Ws for leaky
int launch_esn_fwd(bool gru, int64_t B, int64_t T, int64_t dr, const float* U, const float* Uz,
                   const float* Ur, const float* const W[3], const int64_t ld[3],
                   const float* leak, float* H, cudaStream_t stream, int64_t ts = 0,
                   const float* h0 = nullptr, int64_t ld_h0 = 0);
int launch_split_tf32(const float* x, int64_t n, float* hi, float* lo, cudaStream_t stream);
int launch_split_tf32_cat(const float* x, int64_t rows, int64_t cols, float* out, int nparts,
                          int lo_mask, cudaStream_t stream);
int launch_esn_bwd(bool gru, int64_t B, int64_t T, int64_t dr, const float* dH,
                   const float* const F[5], const float* const WT[3], const int64_t ld[3],
                   const float* leak, float* const out[3], cudaStream_t stream);

// maslov.cu: (gated) Maslov softmax of attention scores.  Scores T, C, P, dP,
// dT, dC: [rows = B*H*Lq, Lk] contiguous; g / dg at b*gsb + i*gsi + h*gsh;
// mask bytes (nonzero = masked) at b*msb + h*msh + i*msi + j*msj.
struct MaslovArgs {
  int64_t rows, H, Lq, Lk;
  const float* T;
  const float* C;
  const float* g;
  int64_t gsb, gsi, gsh;
  const unsigned char* mask;
  int64_t msb, msh, msi, msj;
  const float* tau;
  float* P;            // forward: output; backward: input
  const float* dP;
  float* dT;
  float* dC;
  float* dg;
  float* dtau_rows;
};
int launch_maslov(const MaslovArgs& a, bool backward, cudaStream_t stream);

}  // namespace tp
