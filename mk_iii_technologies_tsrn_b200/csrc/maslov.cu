// maslov.cu -- Maslov (per-head temperature) softmax of attention scores,
// optionally after the DTN tropical/classical gate, forward and backward.
//
// Replaces, in DTNAttention.forward (deep_tropical_net.py:152-160), the chain
//   s    = g * trop + (1 - g) * class      g = sigmoid(score_gate(x)) [B, Lq, H]
//   s    = masked_fill(s, mask == 0, -1e9)
//   attn = softmax(s / tau_h, dim=-1)      MaslovTemperature.forward (tropformer.py:206-212)
// and the autograd backward of that chain; without the classical scores it is
// MaslovTemperature alone (s = trop).  One warp per score row; a row of up to
// 256 keys is held in registers (lane l owns keys l, l+32, ...), longer rows
// are streamed three times from memory.
//
// The forward rounds the blend and the division like the PyTorch expression
// (fl(g*T) + fl(fl(1-g)*C), then fl(s / tau), no contraction); the softmax is
// max, sum of exp(z - max), exp / sum, each lane summing its keys in order and
// the warp combining by xor butterflies.  Every access is in bounds by
// construction (row < rows, key < Lk); there is no wait of any kind.
#include "maxplus_internal.cuh"

namespace tp {

namespace {

constexpr int MAS_THREADS = 256;
constexpr int MAS_ROWS = MAS_THREADS / 32;

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// per-row view of the arguments
struct MasRow {
  const float* T;
  const float* C;          // null without the gate
  bool gated;
  const unsigned char* m;  // null without a mask
  int64_t msj;
  float gv, omg, tau;
  int64_t gidx;            // offset of g[b, i, h]
};

__device__ __forceinline__ MasRow mas_row(const MaslovArgs& a, int64_t row) {
  MasRow r;
  const int64_t i = row % a.Lq;
  const int64_t bh = row / a.Lq;
  const int64_t h = bh % a.H, b = bh / a.H;
  r.T = a.T + row * a.Lk;
  r.gated = a.g != nullptr;
  r.C = r.gated ? a.C + row * a.Lk : nullptr;
  r.m = a.mask ? a.mask + b * a.msb + h * a.msh + i * a.msi : nullptr;
  r.msj = a.msj;
  r.gidx = b * a.gsb + i * a.gsi + h * a.gsh;
  r.gv = r.gated ? a.g[r.gidx] : 1.0f;
  r.omg = __fsub_rn(1.0f, r.gv);
  r.tau = a.tau[h];
  return r;
}

// s after the blend and the mask (PyTorch's rounding)
__device__ __forceinline__ float mas_score(const MasRow& r, int64_t j) {
  float s = r.gated ? __fadd_rn(__fmul_rn(r.gv, r.T[j]), __fmul_rn(r.omg, r.C[j])) : r.T[j];
  if (r.m && r.m[j * r.msj]) s = -1e9f;
  return s;
}

template <int NPL>
__global__ void __launch_bounds__(MAS_THREADS) maslov_fwd_kernel(MaslovArgs a) {
  const int lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * MAS_ROWS + (threadIdx.x >> 5);
  if (row >= a.rows) return;                       // whole warp leaves together
  const MasRow r = mas_row(a, row);
  float* P = a.P + row * a.Lk;
  const float NEG_INF = -__int_as_float(0x7f800000);
  if constexpr (NPL > 0) {
    float z[NPL];
    float m = NEG_INF;
#pragma unroll
    for (int u = 0; u < NPL; ++u) {
      const int64_t j = lane + 32 * u;
      z[u] = j < a.Lk ? __fdiv_rn(mas_score(r, j), r.tau) : NEG_INF;
      m = fmaxf(m, z[u]);
    }
    m = warp_max(m);
    float sum = 0.0f;
#pragma unroll
    for (int u = 0; u < NPL; ++u) {
      z[u] = (lane + 32 * u < a.Lk) ? expf(z[u] - m) : 0.0f;
      sum += z[u];
    }
    sum = warp_sum(sum);
#pragma unroll
    for (int u = 0; u < NPL; ++u) {
      const int64_t j = lane + 32 * u;
      if (j < a.Lk) P[j] = __fdiv_rn(z[u], sum);
    }
  } else {
    float m = NEG_INF;
    for (int64_t j = lane; j < a.Lk; j += 32) m = fmaxf(m, __fdiv_rn(mas_score(r, j), r.tau));
    m = warp_max(m);
    float sum = 0.0f;
    for (int64_t j = lane; j < a.Lk; j += 32) sum += expf(__fdiv_rn(mas_score(r, j), r.tau) - m);
    sum = warp_sum(sum);
    for (int64_t j = lane; j < a.Lk; j += 32)
      P[j] = __fdiv_rn(expf(__fdiv_rn(mas_score(r, j), r.tau) - m), sum);
  }
}

// dz = P (dP - sum P dP); ds = dz / tau (0 where masked);
// dT = g ds (ds without the gate), dC = (1 - g) ds, dg = sum ds T - sum ds C,
// dtau_rows = sum dz s  (s after the mask, as the division saw it).  Since
// sum_j dz_j = 0, dtau_rows is formed as sum dz (s - max s): the same value
// without the cancellation of -1e9 entries of a fully masked row.
template <int NPL>
__global__ void __launch_bounds__(MAS_THREADS) maslov_bwd_kernel(MaslovArgs a) {
  const int lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * MAS_ROWS + (threadIdx.x >> 5);
  if (row >= a.rows) return;
  const MasRow r = mas_row(a, row);
  const float* P = a.P + row * a.Lk;
  const float* dP = a.dP + row * a.Lk;
  float* dT = a.dT ? a.dT + row * a.Lk : nullptr;
  float* dC = a.dC ? a.dC + row * a.Lk : nullptr;
  const float NEG_INF = -__int_as_float(0x7f800000);
  float rs = 0.0f, sgT = 0.0f, sgC = 0.0f;
  auto elem = [&](int64_t j, float p, float d, float dot, float s, float smax) {
    const float dz = __fmul_rn(p, __fsub_rn(d, dot));
    rs = fmaf(dz, s - smax, rs);
    const bool masked = r.m && r.m[j * r.msj];
    const float ds = masked ? 0.0f : __fdiv_rn(dz, r.tau);
    if (r.gated) {
      if (dT) dT[j] = __fmul_rn(r.gv, ds);
      if (dC) dC[j] = __fmul_rn(r.omg, ds);
      sgT = fmaf(ds, r.T[j], sgT);
      sgC = fmaf(ds, r.C[j], sgC);
    } else if (dT) {
      dT[j] = ds;
    }
  };
  if constexpr (NPL > 0) {
    float p[NPL], d[NPL], sc[NPL];
    float dot = 0.0f, smax = NEG_INF;
#pragma unroll
    for (int u = 0; u < NPL; ++u) {
      const int64_t j = lane + 32 * u;
      const bool in = j < a.Lk;
      p[u] = in ? P[j] : 0.0f;
      d[u] = in ? dP[j] : 0.0f;
      sc[u] = in ? mas_score(r, j) : NEG_INF;
      dot = fmaf(p[u], d[u], dot);
      smax = fmaxf(smax, sc[u]);
    }
    dot = warp_sum(dot);
    smax = warp_max(smax);
#pragma unroll
    for (int u = 0; u < NPL; ++u) {
      const int64_t j = lane + 32 * u;
      if (j < a.Lk) elem(j, p[u], d[u], dot, sc[u], smax);
    }
  } else {
    float dot = 0.0f, smax = NEG_INF;
    for (int64_t j = lane; j < a.Lk; j += 32) {
      dot = fmaf(P[j], dP[j], dot);
      smax = fmaxf(smax, mas_score(r, j));
    }
    dot = warp_sum(dot);
    smax = warp_max(smax);
    for (int64_t j = lane; j < a.Lk; j += 32) elem(j, P[j], dP[j], dot, mas_score(r, j), smax);
  }
  rs = warp_sum(rs);
  sgT = warp_sum(sgT);
  sgC = warp_sum(sgC);
  if (lane == 0) {
    if (a.dtau_rows) a.dtau_rows[row] = rs;
    if (a.dg && r.gated) a.dg[r.gidx] = sgT - sgC;
  }
}

template <int N>
void mas_launch(const MaslovArgs& a, bool backward, dim3 grid, cudaStream_t stream) {
  if (backward)
    maslov_bwd_kernel<N><<<grid, MAS_THREADS, 0, stream>>>(a);
  else
    maslov_fwd_kernel<N><<<grid, MAS_THREADS, 0, stream>>>(a);
}

}  // namespace

int launch_maslov(const MaslovArgs& a, bool backward, cudaStream_t stream) {
  const int64_t blocks = (a.rows + MAS_ROWS - 1) / MAS_ROWS;
  if (blocks > 0x7fffffff) return TP_ERR_TOO_LARGE;
  const dim3 grid((unsigned)blocks);
  if (a.Lk <= 32)
    mas_launch<1>(a, backward, grid, stream);
  else if (a.Lk <= 64)
    mas_launch<2>(a, backward, grid, stream);
  else if (a.Lk <= 128)
    mas_launch<4>(a, backward, grid, stream);
  else if (a.Lk <= 256)
    mas_launch<8>(a, backward, grid, stream);
  else
    mas_launch<0>(a, backward, grid, stream);
  return launch_status();
}

}  // namespace tp
