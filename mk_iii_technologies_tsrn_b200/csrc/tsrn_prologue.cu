// tsrn_prologue.cu -- the prologue of the TSRN tropical attention
// (research/tsrn_dml.py:472-500) in one pass: from the Q/K/V projections of a
// [B, T, d] sequence (one [B*T, ld] matrix holding the three at column
// offsets 0, koff, voff), per head h of dh channels
//   Q[b,h,t] = rope_t(LayerNorm_dh(q[b,t,h]; q_gamma, q_beta))
//   K[b,h,t] = rope_t(LayerNorm_dh(k[b,t,h]; k_gamma, k_beta))
//   V[b,h,t] = v[b,t,h]
// written [B, H, T, dh] contiguous -- the layout the fused attention reads.
// rope_t pairs channel c with c + dh/2 (c < dh/2) and rotates the pair by the
// angle of position pos0 + t: out_c = x_c cos - x_{c+dh/2} sin,
// out_{c+dh/2} = x_{c+dh/2} cos + x_c sin, with cos/sin read from caller
// tables [npos, dh/2] and each product and sum rounded separately (no FMA
// contraction), as the reference's q*cos + rotate_half(q)*sin evaluates.
// PyTorch runs the same chain as a dozen kernels with as many passes over
// [B, H, T, dh]; here each row is read once and written once.
//
// One warp per (b, t, h) row, lanes over channels (dh <= 128: at most four per
// lane); the normalised row is staged in shared memory so that each lane can
// read its rotation partner.
#include "maxplus_internal.cuh"

namespace tp {

namespace {

constexpr int PRO_WARPS = 4;
constexpr int PRO_MAX_DH = 128;

struct ProArgs {
  int64_t B, T, H, dh;
  const float* qkv;
  int64_t ld, koff, voff;
  const float* qg;
  const float* qb;
  const float* kg;
  const float* kb;
  float eps;
  const float* cosb;
  const float* sinb;
  int64_t pos0;
  float* Q;
  float* K;
  float* V;
};

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// LayerNorm of one dh-channel row held four channels per lane (c = lane + 32 i),
// then the rotation; the result goes to out[0..dh)
__device__ __forceinline__ void norm_rope_row(const float* src, const float* g, const float* bta,
                                              float eps, const float* cs, const float* sn,
                                              int dh, int lane, float* stage, float* out) {
  float x[4];
  float s = 0.0f;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int c = lane + 32 * i;
    x[i] = c < dh ? __ldg(src + c) : 0.0f;
    s += x[i];
  }
  const float mean = warp_sum(s) / (float)dh;
  float v = 0.0f;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int c = lane + 32 * i;
    const float dlt = c < dh ? x[i] - mean : 0.0f;
    v += dlt * dlt;
  }
  const float rstd = rsqrtf(warp_sum(v) / (float)dh + eps);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int c = lane + 32 * i;
    if (c < dh) stage[c] = (x[i] - mean) * rstd * __ldg(g + c) + __ldg(bta + c);
  }
  __syncwarp();
  const int half = dh >> 1;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int c = lane + 32 * i;
    if (c < dh) {
      const int cc = c < half ? c : c - half;
      const float co = __ldg(cs + cc), si = __ldg(sn + cc);
      const float self = stage[c];
      const float part = stage[c < half ? c + half : c - half];
      // lower half: x_c cos - x_{c+half} sin; upper half: x_c cos + x_{c-half} sin
      const float a = __fmul_rn(self, co);
      const float b = __fmul_rn(part, si);
      out[c] = c < half ? __fsub_rn(a, b) : __fadd_rn(a, b);
    }
  }
  __syncwarp();
}

__global__ void __launch_bounds__(32 * PRO_WARPS) tsrn_prologue_kernel(const ProArgs p) {
  __shared__ float stage[PRO_WARPS][PRO_MAX_DH];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * PRO_WARPS + warp;   // (b, t, h), h fastest
  if (row >= p.B * p.T * p.H) return;
  const int64_t h = row % p.H;
  const int64_t bt = row / p.H;
  const int64_t t = bt % p.T, b = bt / p.T;
  const int dh = (int)p.dh;
  const float* src = p.qkv + bt * p.ld + h * p.dh;
  const int64_t dst = ((b * p.H + h) * p.T + t) * p.dh;
  const float* cs = p.cosb + (p.pos0 + t) * (p.dh >> 1);
  const float* sn = p.sinb + (p.pos0 + t) * (p.dh >> 1);
  norm_rope_row(src, p.qg, p.qb, p.eps, cs, sn, dh, lane, stage[warp], p.Q + dst);
  norm_rope_row(src + p.koff, p.kg, p.kb, p.eps, cs, sn, dh, lane, stage[warp], p.K + dst);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int c = lane + 32 * i;
    if (c < dh) p.V[dst + c] = __ldg(src + p.voff + c);
  }
}

}  // namespace

int launch_tsrn_prologue(int64_t B, int64_t T, int64_t H, int64_t dh, const float* qkv, int64_t ld,
                         int64_t koff, int64_t voff, const float* qg, const float* qb,
                         const float* kg, const float* kb, float eps, const float* cosb,
                         const float* sinb, int64_t pos0, float* Q, float* K, float* V,
                         cudaStream_t stream) {
  if (B * T * H == 0) return TP_OK;
  if (dh > PRO_MAX_DH || dh % 2 != 0) return TP_ERR_UNSUPPORTED;
  ProArgs p{B, T, H, dh, qkv, ld, koff, voff, qg, qb, kg, kb, eps, cosb, sinb, pos0, Q, K, V};
  const int64_t rows = B * T * H;
  tsrn_prologue_kernel<<<(unsigned)ceil_div(rows, PRO_WARPS), 32 * PRO_WARPS, 0, stream>>>(p);
  return launch_status();
}

}  // namespace tp
