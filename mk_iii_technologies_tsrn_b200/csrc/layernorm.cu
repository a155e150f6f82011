// layernorm.cu -- backward of LayerNorm over rows of D channels: the pre-norms
// of the TSRN block's tropical branches (research/tsrn_dml.py:1096-1106,
// nn.LayerNorm(d_model) before the attention, the reservoir and the SSM) in
// training.  One pass over x and dy: per row the statistics are recomputed
// (two-pass mean and variance of the row held in registers), then
//   dx = rstd * (g - mean(g) - xhat * mean(g * xhat)),  g = dy * gamma,
// while dgamma = sum over rows of dy * xhat and dbeta = sum of dy accumulate
// per warp in registers, per block over its warps in a fixed order, and over
// the blocks in a fixed order by a second kernel: the parameter gradients are
// the same bits on every call.  PyTorch's backward for this shape ([65536,
// 640] per branch) spends ~0.6 ms in its gamma/beta reduction alone.
//
// One warp per row, D = 128 * NV (NV <= 8): each lane holds NV float4s.
#include "maxplus_internal.cuh"

namespace tp {

namespace {

constexpr int LN_WARPS = 4;
constexpr int LN_MAX_NV = 8;

__device__ __forceinline__ float ln_warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

template <int NV>
__global__ void __launch_bounds__(32 * LN_WARPS) layernorm_bwd_kernel(
    const float* __restrict__ x, const float* __restrict__ dy, const float* __restrict__ gamma,
    float eps, int64_t rows, float* __restrict__ dx, float* __restrict__ part) {
  constexpr int D = 128 * NV;
  __shared__ float s_acc[LN_WARPS][2 * D];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  float gm[4 * NV], ag[4 * NV], ab[4 * NV];
#pragma unroll
  for (int v = 0; v < NV; ++v) {
    float4 t = make_float4(1.0f, 1.0f, 1.0f, 1.0f);
    if (gamma != nullptr) t = __ldg(reinterpret_cast<const float4*>(gamma) + lane + 32 * v);
    gm[4 * v] = t.x; gm[4 * v + 1] = t.y; gm[4 * v + 2] = t.z; gm[4 * v + 3] = t.w;
  }
#pragma unroll
  for (int i = 0; i < 4 * NV; ++i) {
    ag[i] = 0.0f;
    ab[i] = 0.0f;
  }
  const float inv_d = 1.0f / (float)D;
  const int64_t stride = (int64_t)gridDim.x * LN_WARPS;
  for (int64_t r = (int64_t)blockIdx.x * LN_WARPS + warp; r < rows; r += stride) {
    const float4* xr = reinterpret_cast<const float4*>(x + r * D);
    const float4* dr = reinterpret_cast<const float4*>(dy + r * D);
    float xv[4 * NV], dv[4 * NV];
#pragma unroll
    for (int v = 0; v < NV; ++v) {
      const float4 a = __ldcs(xr + lane + 32 * v);
      const float4 d = __ldcs(dr + lane + 32 * v);
      xv[4 * v] = a.x; xv[4 * v + 1] = a.y; xv[4 * v + 2] = a.z; xv[4 * v + 3] = a.w;
      dv[4 * v] = d.x; dv[4 * v + 1] = d.y; dv[4 * v + 2] = d.z; dv[4 * v + 3] = d.w;
    }
    float s = 0.0f;
#pragma unroll
    for (int i = 0; i < 4 * NV; ++i) s += xv[i];
    const float mean = ln_warp_sum(s) * inv_d;
    float q = 0.0f;
#pragma unroll
    for (int i = 0; i < 4 * NV; ++i) {
      xv[i] -= mean;
      q += xv[i] * xv[i];
    }
    const float rstd = rsqrtf(ln_warp_sum(q) * inv_d + eps);
    float s1 = 0.0f, s2 = 0.0f;
#pragma unroll
    for (int i = 0; i < 4 * NV; ++i) {
      xv[i] *= rstd;                          // xhat
      const float g = dv[i] * gm[i];
      s1 += g;
      s2 += g * xv[i];
      ag[i] += dv[i] * xv[i];
      ab[i] += dv[i];
    }
    const float m1 = ln_warp_sum(s1) * inv_d;
    const float m2 = ln_warp_sum(s2) * inv_d;
    float4* out = reinterpret_cast<float4*>(dx + r * D);
#pragma unroll
    for (int v = 0; v < NV; ++v) {
      float o[4];
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const int i = 4 * v + k;
        o[k] = rstd * (dv[i] * gm[i] - m1 - xv[i] * m2);
      }
      __stcs(out + lane + 32 * v, make_float4(o[0], o[1], o[2], o[3]));
    }
  }
  // this block's parameter-gradient partials: its warps in order
#pragma unroll
  for (int v = 0; v < NV; ++v) {
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const int c = 4 * (lane + 32 * v) + k;
      s_acc[warp][c] = ag[4 * v + k];
      s_acc[warp][D + c] = ab[4 * v + k];
    }
  }
  __syncthreads();
  for (int e = threadIdx.x; e < 2 * D; e += blockDim.x) {
    float t = 0.0f;
#pragma unroll
    for (int w = 0; w < LN_WARPS; ++w) t += s_acc[w][e];
    part[(int64_t)blockIdx.x * 2 * D + e] = t;
  }
}

// dgamma / dbeta: the blocks' partials summed in block order
__global__ void layernorm_bwd_sum_kernel(const float* __restrict__ part, int blocks, int D,
                                         float* __restrict__ dgamma, float* __restrict__ dbeta) {
  const int e = blockIdx.x * blockDim.x + threadIdx.x;
  if (e >= 2 * D) return;
  float acc = 0.0f;
  for (int bl = 0; bl < blocks; ++bl) acc += part[(int64_t)bl * 2 * D + e];
  if (e < D) {
    if (dgamma) dgamma[e] = acc;
  } else if (dbeta) {
    dbeta[e - D] = acc;
  }
}

}  // namespace

int layernorm_bwd_blocks(int64_t rows) {
  const int64_t want = ceil_div(rows, (int64_t)LN_WARPS);
  const int64_t cap = (int64_t)num_sms() * 4;
  return (int)(want < cap ? (want > 0 ? want : 1) : cap);
}

bool layernorm_bwd_supported(int64_t D) {
  return D >= 128 && D <= 128 * LN_MAX_NV && D % 128 == 0;
}

int launch_layernorm_bwd(int64_t rows, int64_t D, const float* x, const float* dy,
                         const float* gamma, float eps, float* dx, float* dgamma, float* dbeta,
                         float* part, cudaStream_t stream) {
  if (!layernorm_bwd_supported(D)) return TP_ERR_UNSUPPORTED;
  const int blocks = layernorm_bwd_blocks(rows);
  if (rows > 0) {
    const unsigned g = (unsigned)blocks;
    const int t = 32 * LN_WARPS;
    switch (D / 128) {
      case 1: layernorm_bwd_kernel<1><<<g, t, 0, stream>>>(x, dy, gamma, eps, rows, dx, part); break;
      case 2: layernorm_bwd_kernel<2><<<g, t, 0, stream>>>(x, dy, gamma, eps, rows, dx, part); break;
      case 3: layernorm_bwd_kernel<3><<<g, t, 0, stream>>>(x, dy, gamma, eps, rows, dx, part); break;
      case 4: layernorm_bwd_kernel<4><<<g, t, 0, stream>>>(x, dy, gamma, eps, rows, dx, part); break;
      case 5: layernorm_bwd_kernel<5><<<g, t, 0, stream>>>(x, dy, gamma, eps, rows, dx, part); break;
      case 6: layernorm_bwd_kernel<6><<<g, t, 0, stream>>>(x, dy, gamma, eps, rows, dx, part); break;
      case 7: layernorm_bwd_kernel<7><<<g, t, 0, stream>>>(x, dy, gamma, eps, rows, dx, part); break;
      default: layernorm_bwd_kernel<8><<<g, t, 0, stream>>>(x, dy, gamma, eps, rows, dx, part); break;
    }
  } else {
    const cudaError_t e = cudaMemsetAsync(part, 0, sizeof(float) * 2 * D * blocks, stream);
    if (e != cudaSuccess) return cuda_status(e);
  }
  layernorm_bwd_sum_kernel<<<(unsigned)ceil_div(2 * D, (int64_t)128), 128, 0, stream>>>(
      part, blocks, (int)D, dgamma, dbeta);
  return launch_status();
}

}  // namespace tp
