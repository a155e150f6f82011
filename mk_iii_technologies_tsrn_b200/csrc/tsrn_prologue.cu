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

// ---------------------------------------------------------------------------
// Backward of the prologue (training): per (b, t, h) row, the LayerNorm
// statistics are recomputed from the projections, the rotation is transposed
//   dy_c = dout_c cos + dout_{c+dh/2} sin,  dy_{c+dh/2} = dout_{c+dh/2} cos - dout_c sin
// and the LayerNorm backward gives
//   dx = rstd (g dy - mean(g dy) - xhat mean(g dy xhat)),
// written into dqkv at the row's Q / K columns (V's gradient is copied to its
// columns).  The gamma / beta gradients (sums of dy xhat and dy over all rows)
// accumulate per warp over a fixed set of rows, then per block in warp order,
// and a second kernel adds the blocks' partials in block order: the sums are
// deterministic.
// ---------------------------------------------------------------------------
constexpr int PRO_BWD_WARPS = 8;

struct ProBwdArgs {
  int64_t B, T, H, dh;
  const float* qkv;
  int64_t ld, koff, voff;
  const float* qg;
  const float* kg;
  float eps;
  const float* cosb;
  const float* sinb;
  int64_t pos0;
  const float* dQ;
  const float* dK;
  const float* dV;
  float* dqkv;
  float* part;        // [blocks][4][dh]: q gamma, q beta, k gamma, k beta partials
};

// one row's LayerNorm + rotation backward; accumulates this lane's channels'
// gamma / beta gradients into ag / ab
__device__ __forceinline__ void norm_rope_row_bwd(const float* src, const float* g,
                                                  float eps, const float* cs, const float* sn,
                                                  const float* dout, int dh, int lane,
                                                  float* dst, float (&ag)[4], float (&ab)[4]) {
  float x[4], d[4];
  float s = 0.0f;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int c = lane + 32 * i;
    x[i] = c < dh ? __ldg(src + c) : 0.0f;
    d[i] = c < dh ? __ldg(dout + c) : 0.0f;
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
  // the rotation partner of channel c is c +- dh/2: with dh <= 128 and four
  // channels per lane (c = lane + 32 i) it sits in another lane; fetch it by
  // shuffle from the lane that holds it
  const int half = dh >> 1;
  float dy[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int c = lane + 32 * i;
    const int pc = c < half ? c + half : c - half;      // partner channel
    // every lane takes part in the shuffles (partner index clamped in range)
    const int pcs = c < dh ? pc : c;
    float pd = 0.0f;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const float got = __shfl_sync(0xffffffffu, d[k], pcs & 31);
      if ((pcs >> 5) == k) pd = got;
    }
    if (c < dh) {
      const int cc = c < half ? c : c - half;
      const float co = __ldg(cs + cc), si = __ldg(sn + cc);
      dy[i] = c < half ? d[i] * co + pd * si : d[i] * co - pd * si;
    } else {
      dy[i] = 0.0f;
    }
  }
  float m1 = 0.0f, m2 = 0.0f;
  float xh[4], gd[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int c = lane + 32 * i;
    xh[i] = c < dh ? (x[i] - mean) * rstd : 0.0f;
    gd[i] = c < dh ? dy[i] * __ldg(g + c) : 0.0f;
    m1 += gd[i];
    m2 += gd[i] * xh[i];
    ag[i] += dy[i] * xh[i];
    ab[i] += dy[i];
  }
  m1 = warp_sum(m1) / (float)dh;
  m2 = warp_sum(m2) / (float)dh;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int c = lane + 32 * i;
    if (c < dh) dst[c] = rstd * (gd[i] - m1 - xh[i] * m2);
  }
}

__global__ void __launch_bounds__(32 * PRO_BWD_WARPS) tsrn_prologue_bwd_kernel(const ProBwdArgs p) {
  __shared__ float red[PRO_BWD_WARPS][4][PRO_MAX_DH];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int dh = (int)p.dh;
  const int64_t rows = p.B * p.T * p.H;
  float qa[4] = {0, 0, 0, 0}, qb[4] = {0, 0, 0, 0}, ka[4] = {0, 0, 0, 0}, kb[4] = {0, 0, 0, 0};
  const int64_t stride = (int64_t)gridDim.x * PRO_BWD_WARPS;
  for (int64_t row = (int64_t)blockIdx.x * PRO_BWD_WARPS + warp; row < rows; row += stride) {
    const int64_t h = row % p.H;
    const int64_t bt = row / p.H;
    const int64_t t = bt % p.T, b = bt / p.T;
    const float* src = p.qkv + bt * p.ld + h * p.dh;
    float* dst = p.dqkv + bt * p.ld + h * p.dh;
    const int64_t hrow = ((b * p.H + h) * p.T + t) * p.dh;
    const float* cs = p.cosb + (p.pos0 + t) * (p.dh >> 1);
    const float* sn = p.sinb + (p.pos0 + t) * (p.dh >> 1);
    norm_rope_row_bwd(src, p.qg, p.eps, cs, sn, p.dQ + hrow, dh, lane, dst, qa, qb);
    norm_rope_row_bwd(src + p.koff, p.kg, p.eps, cs, sn, p.dK + hrow, dh, lane, dst + p.koff, ka,
                      kb);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int c = lane + 32 * i;
      if (c < dh) dst[p.voff + c] = __ldg(p.dV + hrow + c);
    }
  }
  // block partials: warps in order
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int c = lane + 32 * i;
    if (c < dh) {
      red[warp][0][c] = qa[i];
      red[warp][1][c] = qb[i];
      red[warp][2][c] = ka[i];
      red[warp][3][c] = kb[i];
    }
  }
  __syncthreads();
  for (int e = threadIdx.x; e < 4 * dh; e += blockDim.x) {
    const int k = e / dh, c = e - k * dh;
    float acc = 0.0f;
    for (int w = 0; w < PRO_BWD_WARPS; ++w) acc += red[w][k][c];
    p.part[((int64_t)blockIdx.x * 4 + k) * dh + c] = acc;
  }
}

// sums the blocks' partials in block order: out[k][c] for k = q gamma, q beta,
// k gamma, k beta
__global__ void tsrn_prologue_bwd_sum_kernel(const float* __restrict__ part, int blocks, int n,
                                             float* __restrict__ out) {
  const int e = blockIdx.x * blockDim.x + threadIdx.x;
  if (e >= n) return;
  float acc = 0.0f;
  for (int bl = 0; bl < blocks; ++bl) acc += part[(int64_t)bl * n + e];
  out[e] = acc;
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

namespace tp {

int tsrn_prologue_bwd_blocks(int64_t B, int64_t T, int64_t H) {
  int dev = 0, sms = 148;
  if (cudaGetDevice(&dev) == cudaSuccess)
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int64_t rows = B * T * H;
  const int64_t want = ceil_div(rows, (int64_t)PRO_BWD_WARPS);
  const int64_t cap = (int64_t)sms * 8;
  return (int)(want < cap ? (want > 0 ? want : 1) : cap);
}

int launch_tsrn_prologue_bwd(int64_t B, int64_t T, int64_t H, int64_t dh, const float* qkv,
                             int64_t ld, int64_t koff, int64_t voff, const float* qg,
                             const float* kg, float eps, const float* cosb, const float* sinb,
                             int64_t pos0, const float* dQ, const float* dK, const float* dV,
                             float* dqkv, float* dparams, float* part, cudaStream_t stream) {
  if (dh > PRO_MAX_DH || dh % 2 != 0 || dh < 2) return TP_ERR_UNSUPPORTED;
  const int blocks = tsrn_prologue_bwd_blocks(B, T, H);
  if (B * T * H > 0) {
    ProBwdArgs p{B, T, H, dh, qkv, ld, koff, voff, qg, kg, eps, cosb, sinb, pos0, dQ, dK, dV,
                 dqkv, part};
    tsrn_prologue_bwd_kernel<<<(unsigned)blocks, 32 * PRO_BWD_WARPS, 0, stream>>>(p);
  } else {
    cudaMemsetAsync(part, 0, sizeof(float) * 4 * dh * blocks, stream);
  }
  const int n = 4 * (int)dh;
  tsrn_prologue_bwd_sum_kernel<<<(unsigned)ceil_div((int64_t)n, (int64_t)128), 128, 0, stream>>>(
      part, blocks, n, dparams);
  return launch_status();
}

}  // namespace tp
