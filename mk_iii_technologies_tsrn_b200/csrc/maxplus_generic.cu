// maxplus_generic.cu -- strided / batched max-plus kernels for every shape.
//
// These kernels accept any strides, two batch levels, fp32 or bf16 operands,
// and any M, N, K (including K not a multiple of anything).  They are the
// path for the batched tropical attention scores (deep_tropical_net.py:148-150,
// tropformer.py:378-381: per-head GEMMs of 64x64x32), for small tropical
// linears, for A (x) B with B stored [K,N] (cuda/maxplus_gemm.cu:269-290), and
// for everything the TMA kernel in maxplus_tma.cu does not take.
//
// Forward with argmax tracks (value, index) exactly per term, scanning k in
// ascending order with "strictly greater, or first NaN" as the update rule.
// That reproduces torch.max(dim=-1) on the reference's broadcast tensor
// (tropformer.py:131-141): lowest index on ties, first NaN wins, index 0 for
// an all -inf row.
#include "maxplus_internal.cuh"

namespace tp {

namespace {

constexpr int GB_M = 64;
constexpr int GB_N = 64;
constexpr int GB_K = 16;
constexpr int G_THREADS = 256;

struct BatchOffsets {
  int64_t x, w, y, a;
};

__device__ __forceinline__ void batch_index(int64_t bz, int64_t B2, int64_t& b1, int64_t& b2) {
  b1 = bz / B2;
  b2 = bz - b1 * B2;
}

// Load a [GB_K x 64] slab of an operand (rows r0.., k0..) into smem as
// dst[kk][rr], converting to fp32.  Out-of-range k gives `kfill`, out-of-range
// rows give 0.
template <typename T>
__device__ __forceinline__ void load_slab(float (*dst)[GB_M + 4], const T* base, int64_t s_row,
                                          int64_t s_k, int64_t rows, int64_t K, int64_t r0,
                                          int64_t k0, float kfill) {
#pragma unroll
  for (int r = 0; r < (GB_M * GB_K) / G_THREADS; ++r) {
    int e = threadIdx.x + r * G_THREADS;
    int rr = e / GB_K;
    int kk = e % GB_K;
    int64_t gr = r0 + rr;
    int64_t gk = k0 + kk;
    float v;
    if (gk >= K) {
      v = kfill;
    } else if (gr >= rows) {
      v = 0.0f;
    } else {
      v = tp_load_as_f32<T>(base + gr * s_row + gk * s_k);
    }
    dst[kk][rr] = v;
  }
}

// load_slab for a tile of ROWS rows loaded by THREADS threads
template <typename T, int ROWS, int THREADS>
__device__ __forceinline__ void load_slab_rows(float (*dst)[ROWS + 4], const T* base,
                                               int64_t s_row, int64_t s_k, int64_t rows,
                                               int64_t K, int64_t r0, int64_t k0, float kfill) {
  static_assert((ROWS * GB_K) % THREADS == 0, "slab must split evenly over the threads");
#pragma unroll
  for (int r = 0; r < (ROWS * GB_K) / THREADS; ++r) {
    const int e = threadIdx.x + r * THREADS;
    const int rr = e / GB_K;
    const int kk = e % GB_K;
    const int64_t gr = r0 + rr;
    const int64_t gk = k0 + kk;
    float v;
    if (gk >= K) {
      v = kfill;
    } else if (gr >= rows) {
      v = 0.0f;
    } else {
      v = tp_load_as_f32<T>(base + gr * s_row + gk * s_k);
    }
    dst[kk][rr] = v;
  }
}

// ---------------------------------------------------------------------------
// forward (hard max, optional argmax)
// ---------------------------------------------------------------------------
// TYR rows of 16 threads, 4 x 4 outputs each: tiles of (4 TYR) x 64.  Shapes
// with few tiles take TYR = 8 or 4 (32- or 16-row tiles) so that more CTAs
// share the work (config 1's 1024 x 256 output: 64 CTAs at TYR = 16, 256 at
// TYR = 4).
// kBf16Sum: every sum is rounded to bf16 (ties to even) before the max, the
// arithmetic torch applies to bf16 tensors (TP_DTYPE_BF16_ARITH).
template <typename T, bool kArgmax, bool kBf16Sum = false, int TYR = 16>
__global__ void __launch_bounds__(16 * TYR)
    maxplus_fwd_generic_kernel(StridedMaxPlus p) {
  constexpr int ROWS = 4 * TYR, THREADS = 16 * TYR;
  __shared__ float xs[GB_K][ROWS + 4];
  __shared__ float ws[GB_K][GB_N + 4];
  __shared__ float lf_sm[64];
  if (!kArgmax && p.act.mode >= 0) {
    lf_stage(p.act, lf_sm);
    __syncthreads();
  }
  const int tx = threadIdx.x % 16;
  const int ty = threadIdx.x / 16;
  const int64_t m0 = (int64_t)blockIdx.y * ROWS;
  const int64_t n0 = (int64_t)blockIdx.x * GB_N;
  const T* xg = static_cast<const T*>(p.x);
  const T* wg = static_cast<const T*>(p.w);
  const float NEG_INF = -__int_as_float(0x7f800000);

  for (int64_t bz = blockIdx.z; bz < p.B1 * p.B2; bz += gridDim.z) {
    int64_t b1, b2;
    batch_index(bz, p.B2, b1, b2);
    const T* xb = xg + b1 * p.sx_b1 + b2 * p.sx_b2;
    const T* wb = wg + b1 * p.sw_b1 + b2 * p.sw_b2;

    float acc[4][4];
    int idx[4][4];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        acc[i][j] = NEG_INF;
        idx[i][j] = 0;
      }

    for (int64_t k0 = 0; k0 < p.K; k0 += GB_K) {
      __syncthreads();
      load_slab_rows<T, ROWS, THREADS>(xs, xb, p.sx_m, p.sx_k, p.M, p.K, m0, k0, NEG_INF);
      load_slab_rows<T, GB_N, THREADS>(ws, wb, p.sw_n, p.sw_k, p.N, p.K, n0, k0, 0.0f);
      __syncthreads();
#pragma unroll
      for (int kk = 0; kk < GB_K; ++kk) {
        float a[4], b[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) a[i] = xs[kk][ty + TYR * i];
#pragma unroll
        for (int j = 0; j < 4; ++j) b[j] = ws[kk][tx + 16 * j];
        const int k = (int)(k0 + kk);
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            float s = a[i] + b[j];
            if (kBf16Sum) s = __bfloat162float(__float2bfloat16_rn(s));
            if (kArgmax) {
              bool upd = (s > acc[i][j]) | ((s != s) & (acc[i][j] == acc[i][j]));
              acc[i][j] = upd ? s : acc[i][j];
              idx[i][j] = upd ? k : idx[i][j];
            } else {
              acc[i][j] = tp_max_nan(acc[i][j], s);
            }
          }
      }
    }

    float* yb = p.y + b1 * p.sy_b1 + b2 * p.sy_b2;
    int32_t* ab = kArgmax ? p.am + b1 * p.sa_b1 + b2 * p.sa_b2 : nullptr;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      int64_t m = m0 + ty + TYR * i;
      if (m >= p.M) continue;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        int64_t n = n0 + tx + 16 * j;
        if (n >= p.N) continue;
        float v = acc[i][j];
        if (p.bias) v = v + p.bias[n];
        if (p.scale != 1.0f) v = v * p.scale;
        if (!kArgmax && p.act.mode >= 0) v = lf_apply(p.act, lf_sm, n, v);
        yb[m * p.sy_m + n * p.sy_n] = v;
        if (kArgmax) ab[m * p.sa_m + n * p.sa_n] = idx[i][j];
      }
    }
  }
}

// ---------------------------------------------------------------------------
// smooth forward: y = tau * log(sum_k exp(s/tau)), two passes over K
// ---------------------------------------------------------------------------
template <typename T>
__global__ void __launch_bounds__(G_THREADS) maxplus_lse_fwd_generic_kernel(StridedMaxPlus p) {
  __shared__ float xs[GB_K][GB_M + 4];
  __shared__ float ws[GB_K][GB_N + 4];
  const int tx = threadIdx.x % 16;
  const int ty = threadIdx.x / 16;
  const int64_t m0 = (int64_t)blockIdx.y * GB_M;
  const int64_t n0 = (int64_t)blockIdx.x * GB_N;
  const T* xg = static_cast<const T*>(p.x);
  const T* wg = static_cast<const T*>(p.w);
  const float NEG_INF = -__int_as_float(0x7f800000);
  const float L = 1.4426950408889634f / p.tau;  // log2(e) / tau

  for (int64_t bz = blockIdx.z; bz < p.B1 * p.B2; bz += gridDim.z) {
    int64_t b1, b2;
    batch_index(bz, p.B2, b1, b2);
    const T* xb = xg + b1 * p.sx_b1 + b2 * p.sx_b2;
    const T* wb = wg + b1 * p.sw_b1 + b2 * p.sw_b2;

    float mx[4][4], sum[4][4];
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        mx[i][j] = NEG_INF;
        sum[i][j] = 0.0f;
      }
    for (int pass = 0; pass < 2; ++pass) {
      float ref[4][4];
      if (pass == 1) {
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
          for (int j = 0; j < 4; ++j) ref[i][j] = isfinite(mx[i][j]) ? mx[i][j] : 0.0f;
      }
      for (int64_t k0 = 0; k0 < p.K; k0 += GB_K) {
        __syncthreads();
        load_slab<T>(xs, xb, p.sx_m, p.sx_k, p.M, p.K, m0, k0, NEG_INF);
        load_slab<T>(ws, wb, p.sw_n, p.sw_k, p.N, p.K, n0, k0, 0.0f);
        __syncthreads();
#pragma unroll
        for (int kk = 0; kk < GB_K; ++kk) {
          float a[4], b[4];
#pragma unroll
          for (int i = 0; i < 4; ++i) a[i] = xs[kk][ty + 16 * i];
#pragma unroll
          for (int j = 0; j < 4; ++j) b[j] = ws[kk][tx + 16 * j];
#pragma unroll
          for (int i = 0; i < 4; ++i)
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              float s = a[i] + b[j];
              if (pass == 0) {
                mx[i][j] = tp_max_nan(mx[i][j], s);
              } else {
                sum[i][j] += exp2f((s - ref[i][j]) * L);
              }
            }
        }
      }
    }

    float* yb = p.y + b1 * p.sy_b1 + b2 * p.sy_b2;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      int64_t m = m0 + ty + 16 * i;
      if (m >= p.M) continue;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        int64_t n = n0 + tx + 16 * j;
        if (n >= p.N) continue;
        float v = mx[i][j];
        if (isfinite(v)) v = v + p.tau * logf(sum[i][j]);
        if (p.bias) v = v + p.bias[n];
        if (p.scale != 1.0f) v = v * p.scale;
        yb[m * p.sy_m + n * p.sy_n] = v;
      }
    }
  }
}

// ---------------------------------------------------------------------------
// zero a strided [B1][B2][R][C] region
// ---------------------------------------------------------------------------
__global__ void strided_zero_kernel(float* base, int64_t B1, int64_t B2, int64_t R, int64_t C,
                                    int64_t s_b1, int64_t s_b2, int64_t s_r, int64_t s_c) {
  const int64_t total = B1 * B2 * R * C;
  for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < total;
       e += (int64_t)gridDim.x * blockDim.x) {
    int64_t c = e % C;
    int64_t t = e / C;
    int64_t r = t % R;
    t /= R;
    int64_t b2 = t % B2;
    int64_t b1 = t / B2;
    base[b1 * s_b1 + b2 * s_b2 + r * s_r + c * s_c] = 0.0f;
  }
}

// ---------------------------------------------------------------------------
// argmax backward: scatter gy into gx / gw at the argmax index
// ---------------------------------------------------------------------------
__global__ void maxplus_bwd_scatter_kernel(ScatterArgs p) {
  const int64_t total = p.B1 * p.B2 * p.M * p.N;
  for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < total;
       e += (int64_t)gridDim.x * blockDim.x) {
    int64_t n = e % p.N;
    int64_t t = e / p.N;
    int64_t m = t % p.M;
    t /= p.M;
    int64_t b2 = t % p.B2;
    int64_t b1 = t / p.B2;
    int32_t k = p.am[b1 * p.sa_b1 + b2 * p.sa_b2 + m * p.sa_m + n * p.sa_n];
    if (k < 0 || (int64_t)k >= p.K) continue;  // K == 0, or a corrupt index
    float g = p.gy[b1 * p.sg_b1 + b2 * p.sg_b2 + m * p.sg_m + n * p.sg_n] * p.scale;
    atomicAdd(p.gx + b1 * p.sgx_b1 + b2 * p.sgx_b2 + m * p.sgx_m + (int64_t)k * p.sgx_k, g);
    if (p.gw) atomicAdd(p.gw + b1 * p.sgw_b1 + b2 * p.sgw_b2 + n * p.sgw_n + (int64_t)k * p.sgw_k, g);
  }
}

// gbias[n] = scale * sum over (b1, b2, m) of g[b1, b2, m, n]; deterministic.
// One block per 32 columns, CS_WARPS warps: warp w sums rows w, w+CS_WARPS, ...
// into 4 interleaved accumulators (independent loads in flight), and the
// partials are added in a fixed order.  Rows are walked with an incremental
// (b1, b2, m) counter, no division in the loop.
constexpr int CS_WARPS = 32;
__global__ void __launch_bounds__(CS_WARPS * 32)
    column_sum_kernel(const float* g, int64_t B1, int64_t B2, int64_t M, int64_t N, int64_t s_b1,
                      int64_t s_b2, int64_t s_m, int64_t s_n, float scale, float* out) {
  __shared__ float part[CS_WARPS][33];
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int64_t n = (int64_t)blockIdx.x * 32 + lane;
  float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
  if (n < N) {
    const float* gn = g + n * s_n;
    // rows are (b1, b2, m) in row-major order; when they collapse to one
    // stride the loop is a plain strided walk
    const bool flat = (B2 == 1 || s_b2 == M * s_m) && (B1 == 1 || s_b1 == B2 * M * s_m);
    const int64_t rows = B1 * B2 * M;
    if (flat) {
      int64_t r = warp;
      for (; r + 3 * CS_WARPS < rows; r += 4 * CS_WARPS) {
#pragma unroll
        for (int u = 0; u < 4; ++u) acc[u] += gn[(r + u * CS_WARPS) * s_m];
      }
      for (; r < rows; r += CS_WARPS) acc[0] += gn[r * s_m];
    } else {
      for (int64_t b1 = 0; b1 < B1; ++b1)
        for (int64_t b2 = 0; b2 < B2; ++b2) {
          const float* gb = gn + b1 * s_b1 + b2 * s_b2;
          for (int64_t m = warp; m < M; m += CS_WARPS) acc[0] += gb[m * s_m];
        }
    }
  }
  part[warp][lane] = (acc[0] + acc[1]) + (acc[2] + acc[3]);
  __syncthreads();
  if (warp == 0 && n < N) {
    float s = 0.0f;
#pragma unroll
    for (int w = 0; w < CS_WARPS; ++w) s += part[w][lane];
    out[n] = s * scale;
  }
}

// ---------------------------------------------------------------------------
// smooth backward (contiguous x[M,K], w[N,K], gy[M,N]).
//
// Everything runs in the base-2 domain scaled by L = log2(e)/tau: operands
// are multiplied by L when staged, so a term is sL = xL + wL and its weight
// 2^(sL - refL) = exp((s - ref)/tau) costs one ex2.approx.
//   pass 1 (stats): per (m,n): refL = max_k sL; with tL = sL - refL and
//          e = 2^tL:  Z = sum e,  S1 = sum e*tL
//          STE: Bp = g / (Z*log2e),  A = g/Z - Bp*S1/Z
//          LSE: Bp = 0,              A = g/Z
//          so that dS = e * (A + Bp*tL)  [= g p (1 + (s - sbar)/tau) for STE].
//   pass 2 (gx): gx[m,k] = sum_n dS      pass 3 (gw): gw[n,k] = sum_m dS
// A term whose tL is -inf (an operand of -inf) contributes nothing: tL is
// clamped at -256, where 2^tL is already 0, so e*(A + Bp*tL) is 0 and not
// 0*inf; the clamp keeps NaN (max.NaN), so NaN operands still give NaN.
// Thread (tx, ty) of a 64 x 64 tile owns rows 4*ty..4*ty+3 and columns
// 4*tx..4*tx+3: both operand fragments are one 16-byte shared load.
// ---------------------------------------------------------------------------
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kClampL = -256.0f;

// load_slab with every staged value multiplied by `mul` (fills unscaled)
template <typename T>
__device__ __forceinline__ void load_slab_scaled(float (*dst)[GB_M + 4], const T* base,
                                                 int64_t rows, int64_t K, int64_t r0, int64_t k0,
                                                 float kfill, float mul) {
#pragma unroll
  for (int r = 0; r < (GB_M * GB_K) / G_THREADS; ++r) {
    int e = threadIdx.x + r * G_THREADS;
    int rr = e / GB_K;
    int kk = e % GB_K;
    int64_t gr = r0 + rr;
    int64_t gk = k0 + kk;
    float v;
    if (gk >= K) {
      v = kfill;
    } else if (gr >= rows) {
      v = 0.0f;
    } else {
      v = tp_load_as_f32<T>(base + gr * K + gk) * mul;
    }
    dst[kk][rr] = v;
  }
}

__device__ __forceinline__ float4 lds_f4(const float* p) {
  return *reinterpret_cast<const float4*>(p);
}

template <typename T>
__global__ void __launch_bounds__(G_THREADS, 3) smooth_stats_kernel(SmoothArgs p) {
  __shared__ __align__(16) float xs[GB_K][GB_M + 4];
  __shared__ __align__(16) float ws[GB_K][GB_N + 4];
  const int tx = threadIdx.x % 16;
  const int ty = threadIdx.x / 16;
  const int64_t m0 = (int64_t)blockIdx.y * GB_M;
  const int64_t n0 = (int64_t)blockIdx.x * GB_N;
  const int64_t bz = blockIdx.z;
  const T* xg = static_cast<const T*>(p.x) + bz * p.M * p.K;
  const T* wg = static_cast<const T*>(p.w) + bz * p.N * p.K;
  const float* gyb = p.gy + bz * p.M * p.N;
  float* wsb = p.ws + bz * 3 * p.M * p.N;
  const float NEG_INF = -__int_as_float(0x7f800000);
  const float L = kLog2e / p.tau;

  // pass 0: refL = max_k (xL + wL) (or L times the forward's max, when given)
  float mx[4][4];
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) mx[i][j] = NEG_INF;
  if (p.ref) {
    const float* rb = p.ref + bz * p.M * p.N;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int64_t m = m0 + 4 * ty + i;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int64_t n = n0 + 4 * tx + j;
        if (m < p.M && n < p.N) mx[i][j] = rb[m * p.N + n] * L;
      }
    }
  }
  for (int64_t k0 = 0; !p.ref && k0 < p.K; k0 += GB_K) {
    __syncthreads();
    load_slab_scaled<T>(xs, xg, p.M, p.K, m0, k0, NEG_INF, L);
    load_slab_scaled<T>(ws, wg, p.N, p.K, n0, k0, 0.0f, L);
    __syncthreads();
#pragma unroll
    for (int kk = 0; kk < GB_K; ++kk) {
      const float4 a4 = lds_f4(&xs[kk][4 * ty]);
      const float4 b4 = lds_f4(&ws[kk][4 * tx]);
      const float a[4] = {a4.x, a4.y, a4.z, a4.w};
      const float b[4] = {b4.x, b4.y, b4.z, b4.w};
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) mx[i][j] = tp_max_nan(mx[i][j], a[i] + b[j]);
    }
  }

  // pass 1: Z and S1 relative to refL, two columns per packed instruction.
  // Outputs whose max is not finite use refL = 0 and get zero weights (bit
  // 4*i+j of `finite` clear).
  float2 nref[4][2], Z[4][2], S1[4][2];
  uint32_t finite = 0;
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const bool f0 = isfinite(mx[i][2 * h]), f1 = isfinite(mx[i][2 * h + 1]);
      finite |= (f0 ? 1u : 0u) << (4 * i + 2 * h);
      finite |= (f1 ? 1u : 0u) << (4 * i + 2 * h + 1);
      nref[i][h] = make_float2(f0 ? -mx[i][2 * h] : 0.0f, f1 ? -mx[i][2 * h + 1] : 0.0f);
      Z[i][h] = make_float2(0.0f, 0.0f);
      S1[i][h] = make_float2(0.0f, 0.0f);
    }
  for (int64_t k0 = 0; k0 < p.K; k0 += GB_K) {
    __syncthreads();
    load_slab_scaled<T>(xs, xg, p.M, p.K, m0, k0, NEG_INF, L);
    load_slab_scaled<T>(ws, wg, p.N, p.K, n0, k0, 0.0f, L);
    __syncthreads();
#pragma unroll 4
    for (int kk = 0; kk < GB_K; ++kk) {
      const float4 a4 = lds_f4(&xs[kk][4 * ty]);
      const float4 b4 = lds_f4(&ws[kk][4 * tx]);
      const float a[4] = {a4.x, a4.y, a4.z, a4.w};
      const float2 bp[2] = {make_float2(b4.x, b4.y), make_float2(b4.z, b4.w)};
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float2 ap = make_float2(a[i], a[i]);
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          float2 t = tp_add2(tp_add2(ap, bp[h]), nref[i][h]);
          t.x = tp_max_nan(t.x, kClampL);
          t.y = tp_max_nan(t.y, kClampL);
          const float2 e = make_float2(tp_ex2(t.x), tp_ex2(t.y));
          Z[i][h] = tp_add2(Z[i][h], e);
          S1[i][h] = tp_fma2(e, t, S1[i][h]);
        }
      }
    }
  }

  const int64_t MN = p.M * p.N;
  const float inv_log2e = 1.0f / kLog2e;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int64_t m = m0 + 4 * ty + i;
    if (m >= p.M) continue;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int64_t n = n0 + 4 * tx + j;
      if (n >= p.N) continue;
      const float z = j & 1 ? Z[i][j >> 1].y : Z[i][j >> 1].x;
      const float s1 = j & 1 ? S1[i][j >> 1].y : S1[i][j >> 1].x;
      const float g = gyb[m * p.N + n];
      float A = 0.0f, Bp = 0.0f, ref = 0.0f;
      if (((finite >> (4 * i + j)) & 1u) && z > 0.0f) {
        ref = -(j & 1 ? nref[i][j >> 1].y : nref[i][j >> 1].x);
        const float invZ = 1.0f / z;
        if (p.mode == TP_BWD_STE) {
          Bp = g * invZ * inv_log2e;
          A = g * invZ - Bp * s1 * invZ;
        } else {
          A = g * invZ;
        }
      }
      wsb[m * p.N + n] = ref;
      wsb[MN + m * p.N + n] = A;
      wsb[2 * MN + m * p.N + n] = Bp;
      if (p.async_stage) {
        // transposed planes [N][M] for the input-gradient kernel
        float* wt = p.ws + 3 * p.batch * MN + bz * 3 * MN;
        wt[n * p.M + m] = ref;
        wt[MN + n * p.M + m] = A;
        wt[2 * MN + n * p.M + m] = Bp;
      }
    }
  }
}

// Stats pass for fp32 operands: the same results as smooth_stats_kernel, with
// the [16 k x 64 rows] slabs of x and w copied by 4-byte cp.async into one of
// two shared buffers while the other is consumed.  Slabs hold raw values (the
// scale L enters as fma(a + b, L, -refL)); the K tail is cut by the loop bound.
__global__ void __launch_bounds__(G_THREADS, 3) smooth_stats_async_kernel(SmoothArgs p) {
  __shared__ __align__(16) float xs[2][GB_K][GB_M + 4];
  __shared__ __align__(16) float ws[2][GB_K][GB_N + 4];
  const int tx = threadIdx.x % 16;
  const int ty = threadIdx.x / 16;
  const int64_t m0 = (int64_t)blockIdx.y * GB_M;
  const int64_t n0 = (int64_t)blockIdx.x * GB_N;
  const int64_t bz = blockIdx.z;
  const float* xg = static_cast<const float*>(p.x) + bz * p.M * p.K;
  const float* wg = static_cast<const float*>(p.w) + bz * p.N * p.K;
  const float* gyb = p.gy + bz * p.M * p.N;
  float* wsb = p.ws + bz * 3 * p.M * p.N;
  const float NEG_INF = -__int_as_float(0x7f800000);
  const float L = kLog2e / p.tau;
  const int nslab = (int)ceil_div(p.K, (int64_t)GB_K);

  // slab `sl` -> buffer b: element (row rr, k kk) of each operand, kk fastest
  auto issue = [&](int b, int sl) {
    const int64_t k0 = (int64_t)sl * GB_K;
#pragma unroll
    for (int r = 0; r < (GB_M * GB_K) / G_THREADS; ++r) {
      const int e = threadIdx.x + r * G_THREADS;
      const int rr = e / GB_K, kk = e % GB_K;
      const int64_t k = k0 + kk, mr = m0 + rr, nr = n0 + rr;
      const bool okx = k < p.K && mr < p.M, okw = k < p.K && nr < p.N;
      tp_cp_async4(&xs[b][kk][rr], okx ? xg + mr * p.K + k : xg, okx ? 4 : 0);
      tp_cp_async4(&ws[b][kk][rr], okw ? wg + nr * p.K + k : wg, okw ? 4 : 0);
    }
    tp_cp_async_commit();
  };
  // run `body(buffer, k-count)` over all slabs with the next slab in flight
  auto sweep = [&](auto&& body) {
    if (nslab > 0) issue(0, 0);
    for (int sl = 0; sl < nslab; ++sl) {
      const int b = sl & 1;
      if (sl + 1 < nslab) {
        issue(b ^ 1, sl + 1);
        tp_cp_async_wait<1>();
      } else {
        tp_cp_async_wait<0>();
      }
      __syncthreads();
      const int64_t krem = p.K - (int64_t)sl * GB_K;
      body(b, krem < GB_K ? (int)krem : GB_K);
      __syncthreads();
    }
  };

  // pass 0: raw max of x + w (or the forward's, when given)
  float mx[4][4];
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) mx[i][j] = NEG_INF;
  if (p.ref) {
    const float* rb = p.ref + bz * p.M * p.N;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int64_t m = m0 + 4 * ty + i;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int64_t n = n0 + 4 * tx + j;
        if (m < p.M && n < p.N) mx[i][j] = rb[m * p.N + n];
      }
    }
  } else sweep([&](int b, int kn) {
    for (int kk = 0; kk < kn; ++kk) {
      const float4 a4 = lds_f4(&xs[b][kk][4 * ty]);
      const float4 b4 = lds_f4(&ws[b][kk][4 * tx]);
      const float a[4] = {a4.x, a4.y, a4.z, a4.w};
      const float bv[4] = {b4.x, b4.y, b4.z, b4.w};
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) mx[i][j] = tp_max_nan(mx[i][j], a[i] + bv[j]);
    }
  });

  // pass 1: Z and S1 relative to refL = L * max
  float2 nref[4][2], Z[4][2], S1[4][2];
  uint32_t finite = 0;
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const bool f0 = isfinite(mx[i][2 * h]), f1 = isfinite(mx[i][2 * h + 1]);
      finite |= (f0 ? 1u : 0u) << (4 * i + 2 * h);
      finite |= (f1 ? 1u : 0u) << (4 * i + 2 * h + 1);
      nref[i][h] = make_float2(f0 ? -(mx[i][2 * h] * L) : 0.0f,
                               f1 ? -(mx[i][2 * h + 1] * L) : 0.0f);
      Z[i][h] = make_float2(0.0f, 0.0f);
      S1[i][h] = make_float2(0.0f, 0.0f);
    }
  const float2 Lp = make_float2(L, L);
  sweep([&](int b, int kn) {
#pragma unroll 4
    for (int kk = 0; kk < kn; ++kk) {
      const float4 a4 = lds_f4(&xs[b][kk][4 * ty]);
      const float4 b4 = lds_f4(&ws[b][kk][4 * tx]);
      const float a[4] = {a4.x, a4.y, a4.z, a4.w};
      const float2 bp[2] = {make_float2(b4.x, b4.y), make_float2(b4.z, b4.w)};
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float2 ap = make_float2(a[i], a[i]);
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          float2 t = tp_fma2(tp_add2(ap, bp[h]), Lp, nref[i][h]);
          t.x = tp_max_nan(t.x, kClampL);
          t.y = tp_max_nan(t.y, kClampL);
          const float2 e = make_float2(tp_ex2(t.x), tp_ex2(t.y));
          Z[i][h] = tp_add2(Z[i][h], e);
          S1[i][h] = tp_fma2(e, t, S1[i][h]);
        }
      }
    }
  });

  const int64_t MN = p.M * p.N;
  const float inv_log2e = 1.0f / kLog2e;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int64_t m = m0 + 4 * ty + i;
    if (m >= p.M) continue;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int64_t n = n0 + 4 * tx + j;
      if (n >= p.N) continue;
      const float z = j & 1 ? Z[i][j >> 1].y : Z[i][j >> 1].x;
      const float s1 = j & 1 ? S1[i][j >> 1].y : S1[i][j >> 1].x;
      const float g = gyb[m * p.N + n];
      float A = 0.0f, Bp = 0.0f, ref = 0.0f;
      if (((finite >> (4 * i + j)) & 1u) && z > 0.0f) {
        ref = -(j & 1 ? nref[i][j >> 1].y : nref[i][j >> 1].x);
        const float invZ = 1.0f / z;
        if (p.mode == TP_BWD_STE) {
          Bp = g * invZ * inv_log2e;
          A = g * invZ - Bp * s1 * invZ;
        } else {
          A = g * invZ;
        }
      }
      wsb[m * p.N + n] = ref;
      wsb[MN + m * p.N + n] = A;
      wsb[2 * MN + m * p.N + n] = Bp;
      if (p.async_stage) {
        float* wt = p.ws + 3 * p.batch * MN + bz * 3 * MN;
        wt[n * p.M + m] = ref;
        wt[MN + n * p.M + m] = A;
        wt[2 * MN + n * p.M + m] = Bp;
      }
    }
  }
}

// gx[m,k] (kOut == 0) or gw[n,k] (kOut == 1).  Tile over (r, k) with r = m or
// n; loop over this block's slice of the other index q (n or m) in slabs of
// QS.  The three stat planes are staged interleaved ({refL, A, Bp} per (q, r))
// so that a row's stats are one 16-byte shared load.
template <typename T, int kOut>
__global__ void __launch_bounds__(G_THREADS, 3) smooth_grad_kernel(SmoothArgs p) {
  constexpr int QS = 32;
  __shared__ __align__(16) float os[QS][GB_N];      // other operand, scaled: [q][k]
  __shared__ __align__(16) float4 st[QS][GB_M];     // stats: [q][r] {refL, A, Bp, -}
  const int tx = threadIdx.x % 16;
  const int ty = threadIdx.x / 16;
  const int64_t r0 = (int64_t)blockIdx.y * GB_M;
  const int64_t k0 = (int64_t)blockIdx.x * GB_N;
  const int64_t S = kOut == 0 ? p.splits_x : p.splits_w;
  const int64_t bz = blockIdx.z / S;
  const int64_t split = blockIdx.z % S;
  const T* xb = static_cast<const T*>(p.x) + bz * p.M * p.K;
  const T* wb = static_cast<const T*>(p.w) + bz * p.N * p.K;
  const float* wsb = p.ws + bz * 3 * p.M * p.N;
  const T* mine = kOut == 0 ? xb : wb;
  const T* other = kOut == 0 ? wb : xb;
  const int64_t R = kOut == 0 ? p.M : p.N;
  const int64_t Q = kOut == 0 ? p.N : p.M;
  const float L = kLog2e / p.tau;
  const int64_t MN = p.M * p.N;
  // this block's slice [qbeg, qend) of the reduced index, in whole slabs
  const int64_t qchunk = ceil_div(ceil_div(Q, S), (int64_t)QS) * QS;
  const int64_t qbeg = split * qchunk;
  const int64_t qend = (qbeg + qchunk < Q) ? qbeg + qchunk : Q;

  float2 own[4][2], acc[4][2];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int64_t r = r0 + 4 * ty + i;
    float v[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int64_t k = k0 + 4 * tx + j;
      v[j] = (r < R && k < p.K) ? tp_load_as_f32<T>(mine + r * p.K + k) * L : 0.0f;
    }
    own[i][0] = make_float2(v[0], v[1]);
    own[i][1] = make_float2(v[2], v[3]);
    acc[i][0] = make_float2(0.0f, 0.0f);
    acc[i][1] = make_float2(0.0f, 0.0f);
  }

  for (int64_t q0 = qbeg; q0 < qend; q0 += QS) {
    __syncthreads();
    for (int e = threadIdx.x; e < QS * GB_N; e += G_THREADS) {
      const int qq = e / GB_N, kk = e % GB_N;
      const int64_t q = q0 + qq, k = k0 + kk;
      os[qq][kk] = (q < qend && k < p.K) ? tp_load_as_f32<T>(other + q * p.K + k) * L : 0.0f;
    }
    // stats are stored [M][N]: read along n for coalescing
    for (int e = threadIdx.x; e < 3 * QS * GB_M; e += G_THREADS) {
      const int pl = e / (QS * GB_M);
      const int rem = e % (QS * GB_M);
      int qq, rr;
      if (kOut == 0) {  // r = m, q = n
        rr = rem / QS;
        qq = rem % QS;
      } else {          // r = n, q = m
        qq = rem / GB_M;
        rr = rem % GB_M;
      }
      const int64_t q = q0 + qq, r = r0 + rr;
      float v = 0.0f;
      if (q < qend && r < R) {
        const int64_t m = kOut == 0 ? r : q;
        const int64_t n = kOut == 0 ? q : r;
        v = wsb[pl * MN + m * p.N + n];
      }
      reinterpret_cast<float*>(&st[qq][rr])[pl] = v;
    }
    __syncthreads();
    const int qmax = (int)((qend - q0) < QS ? (qend - q0) : QS);
#pragma unroll 2
    for (int qq = 0; qq < qmax; ++qq) {
      const float4 o4 = *reinterpret_cast<const float4*>(&os[qq][4 * tx]);
      const float2 ob[2] = {make_float2(o4.x, o4.y), make_float2(o4.z, o4.w)};
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float4 sv = st[qq][4 * ty + i];
        const float2 nref = make_float2(-sv.x, -sv.x);
        const float2 A = make_float2(sv.y, sv.y);
        const float2 Bp = make_float2(sv.z, sv.z);
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          float2 t = tp_add2(tp_add2(own[i][h], ob[h]), nref);
          t.x = tp_max_nan(t.x, kClampL);
          t.y = tp_max_nan(t.y, kClampL);
          const float2 e = make_float2(tp_ex2(t.x), tp_ex2(t.y));
          acc[i][h] = tp_fma2(e, tp_fma2(Bp, t, A), acc[i][h]);
        }
      }
    }
  }
  float* out = S > 1 ? p.part + ((int64_t)blockIdx.z) * R * p.K
                     : (kOut == 0 ? p.gx + bz * p.M * p.K : p.gw + bz * p.N * p.K);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int64_t r = r0 + 4 * ty + i;
    if (r >= R) continue;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int64_t k = k0 + 4 * tx + j;
      const float v = j & 1 ? acc[i][j >> 1].y : acc[i][j >> 1].x;
      if (k < p.K) out[r * p.K + k] = v;
    }
  }
}

// gx (kOut == 0) or gw (kOut == 1) for fp32 operands with M, N, K multiples of
// 4: the same arithmetic as smooth_grad_kernel, but each QS-row slab of the
// other operand and of the stats (read from planes laid out [q][r], r
// contiguous) is copied with 16-byte cp.async into one of two shared buffers
// while the previous slab is being consumed.  The other operand is staged
// unscaled and scaled inside the first packed fma.
template <int kOut>
__global__ void __launch_bounds__(G_THREADS, 3) smooth_grad_async_kernel(SmoothArgs p) {
  constexpr int QS = 16;
  __shared__ __align__(16) float os[2][QS][GB_N];       // other operand (raw): [q][k]
  __shared__ __align__(16) float st[2][3][QS][GB_M];    // stats: [plane][q][r]
  const int tx = threadIdx.x % 16;
  const int ty = threadIdx.x / 16;
  const int64_t r0 = (int64_t)blockIdx.y * GB_M;
  const int64_t k0 = (int64_t)blockIdx.x * GB_N;
  const int64_t S = kOut == 0 ? p.splits_x : p.splits_w;
  const int64_t bz = blockIdx.z / S;
  const int64_t split = blockIdx.z % S;
  const int64_t MN = p.M * p.N;
  const float* xb = static_cast<const float*>(p.x) + bz * p.M * p.K;
  const float* wb = static_cast<const float*>(p.w) + bz * p.N * p.K;
  const float* mine = kOut == 0 ? xb : wb;
  const float* other = kOut == 0 ? wb : xb;
  const int64_t R = kOut == 0 ? p.M : p.N;
  const int64_t Q = kOut == 0 ? p.N : p.M;
  // planes [q][r]: gW reads the [M][N] planes, gx the transposed [N][M] ones
  const float* planes = (kOut == 0 ? p.ws + 3 * p.batch * MN : p.ws) + bz * 3 * MN;
  const float L = kLog2e / p.tau;
  const int64_t qchunk = ceil_div(ceil_div(Q, S), (int64_t)QS) * QS;
  const int64_t qbeg = split * qchunk;
  const int64_t qend = (qbeg + qchunk < Q) ? qbeg + qchunk : Q;

  float2 own[4][2], acc[4][2];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int64_t r = r0 + 4 * ty + i;
    float v[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int64_t k = k0 + 4 * tx + j;
      v[j] = (r < R && k < p.K) ? __ldg(mine + r * p.K + k) * L : 0.0f;
    }
    own[i][0] = make_float2(v[0], v[1]);
    own[i][1] = make_float2(v[2], v[3]);
    acc[i][0] = make_float2(0.0f, 0.0f);
    acc[i][1] = make_float2(0.0f, 0.0f);
  }

  // slab q0 -> buffer b: QS x 64 operand values (one quad per thread) and
  // 3 x QS x 64 stats (three quads per thread); out-of-range quads zero-filled
  auto issue = [&](int b, int64_t q0) {
    {
      const int qq = threadIdx.x / 16, kv = threadIdx.x % 16;
      const int64_t q = q0 + qq, k = k0 + 4 * kv;
      const bool ok = q < qend && k < p.K;
      tp_cp_async16(&os[b][qq][4 * kv], ok ? other + q * p.K + k : other, ok ? 16 : 0);
    }
#pragma unroll
    for (int c = 0; c < 3; ++c) {
      const int e = threadIdx.x + c * G_THREADS;
      const int pl = e / (QS * 16), rem = e % (QS * 16);
      const int qq = rem / 16, rv = rem % 16;
      const int64_t q = q0 + qq, r = r0 + 4 * rv;
      const bool ok = q < qend && r < R;
      tp_cp_async16(&st[b][pl][qq][4 * rv], ok ? planes + pl * MN + q * R + r : planes,
                    ok ? 16 : 0);
    }
    tp_cp_async_commit();
  };

  const float2 Lp = make_float2(L, L);
  int b = 0;
  if (qbeg < qend) issue(0, qbeg);
  for (int64_t q0 = qbeg; q0 < qend; q0 += QS, b ^= 1) {
    if (q0 + QS < qend) {
      issue(b ^ 1, q0 + QS);
      tp_cp_async_wait<1>();
    } else {
      tp_cp_async_wait<0>();
    }
    __syncthreads();
    const int qmax = (int)((qend - q0) < QS ? (qend - q0) : QS);
#pragma unroll 2
    for (int qq = 0; qq < qmax; ++qq) {
      const float4 o4 = *reinterpret_cast<const float4*>(&os[b][qq][4 * tx]);
      const float2 ob[2] = {make_float2(o4.x, o4.y), make_float2(o4.z, o4.w)};
      const float4 rf = *reinterpret_cast<const float4*>(&st[b][0][qq][4 * ty]);
      const float4 aa = *reinterpret_cast<const float4*>(&st[b][1][qq][4 * ty]);
      const float4 bb = *reinterpret_cast<const float4*>(&st[b][2][qq][4 * ty]);
      const float rfv[4] = {rf.x, rf.y, rf.z, rf.w};
      const float av[4] = {aa.x, aa.y, aa.z, aa.w};
      const float bv[4] = {bb.x, bb.y, bb.z, bb.w};
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float2 nref = make_float2(-rfv[i], -rfv[i]);
        const float2 A = make_float2(av[i], av[i]);
        const float2 Bp = make_float2(bv[i], bv[i]);
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          float2 t = tp_add2(tp_fma2(Lp, ob[h], own[i][h]), nref);
          t.x = tp_max_nan(t.x, kClampL);
          t.y = tp_max_nan(t.y, kClampL);
          const float2 e = make_float2(tp_ex2(t.x), tp_ex2(t.y));
          acc[i][h] = tp_fma2(e, tp_fma2(Bp, t, A), acc[i][h]);
        }
      }
    }
    __syncthreads();   // buffer b is refilled by the next iteration's issue
  }
  float* out = S > 1 ? p.part + ((int64_t)blockIdx.z) * R * p.K
                     : (kOut == 0 ? p.gx + bz * p.M * p.K : p.gw + bz * p.N * p.K);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int64_t r = r0 + 4 * ty + i;
    if (r >= R) continue;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int64_t k = k0 + 4 * tx + j;
      const float v = j & 1 ? acc[i][j >> 1].y : acc[i][j >> 1].x;
      if (k < p.K) out[r * p.K + k] = v;
    }
  }
}

// Both STE / LSE gradients in one pass over (m, n, k): the gx pass above
// (a block owns 64 rows of x and 64 k, walks all n, sums dS over n in
// registers) that also sums the same dS over its 64 rows into this block's
// partial gW[n][k] -- one exponential per term instead of one per term in each
// of two passes.  Threads map so that each warp holds 4 row groups (ty) of 8
// k-quads (tx): the row sum is a two-step xor shuffle within the warp, then
// four warp groups meet in shared memory.  Partials go to part[b][mt][N][K]
// (mt = the block's row tile) and are added in tile order afterwards
// (deterministic).  Needs fp32, M, N, K multiples of 4, one split (the gx
// tiles fill the GPU).
__global__ void __launch_bounds__(G_THREADS, 3) smooth_grad_fused_kernel(SmoothArgs p) {
  constexpr int QS = 16;
  __shared__ __align__(16) float os[2][QS][GB_N];       // w rows (raw): [n][k]
  __shared__ __align__(16) float st[2][3][QS][GB_M];    // stats: [plane][n][m]
  __shared__ __align__(16) float gws[4][QS][GB_N];      // gW partial per warp group
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int tx = (lane & 7) + 8 * (warp & 1);           // k quad: k0 + 4 tx
  const int ty = (lane >> 3) + 4 * (warp >> 1);         // row quad: r0 + 4 ty
  const int wg = warp >> 1;
  const int64_t r0 = (int64_t)blockIdx.y * GB_M;
  const int64_t k0 = (int64_t)blockIdx.x * GB_N;
  const int64_t bz = blockIdx.z;
  const int64_t MN = p.M * p.N;
  const float* xb = static_cast<const float*>(p.x) + bz * p.M * p.K;
  const float* wb = static_cast<const float*>(p.w) + bz * p.N * p.K;
  const float* planes = p.ws + 3 * p.batch * MN + bz * 3 * MN;   // [n][m] planes
  const float L = kLog2e / p.tau;
  const bool rows_ok = r0 + 4 * ty < p.M;                // M % 4 == 0: all four or none
  const int64_t mt = gridDim.y;
  float* gpart = p.part + (bz * mt + blockIdx.y) * p.N * p.K;

  float2 own[4][2], acc[4][2];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int64_t r = r0 + 4 * ty + i;
    float v[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int64_t k = k0 + 4 * tx + j;
      v[j] = (r < p.M && k < p.K) ? __ldg(xb + r * p.K + k) * L : 0.0f;
    }
    own[i][0] = make_float2(v[0], v[1]);
    own[i][1] = make_float2(v[2], v[3]);
    acc[i][0] = make_float2(0.0f, 0.0f);
    acc[i][1] = make_float2(0.0f, 0.0f);
  }

  auto issue = [&](int b, int64_t q0) {
    {
      const int qq = threadIdx.x / 16, kv = threadIdx.x % 16;
      const int64_t q = q0 + qq, k = k0 + 4 * kv;
      const bool ok = q < p.N && k < p.K;
      tp_cp_async16(&os[b][qq][4 * kv], ok ? wb + q * p.K + k : wb, ok ? 16 : 0);
    }
#pragma unroll
    for (int c = 0; c < 3; ++c) {
      const int e = threadIdx.x + c * G_THREADS;
      const int pl = e / (QS * 16), rem = e % (QS * 16);
      const int qq = rem / 16, rv = rem % 16;
      const int64_t q = q0 + qq, r = r0 + 4 * rv;
      const bool ok = q < p.N && r < p.M;
      tp_cp_async16(&st[b][pl][qq][4 * rv], ok ? planes + pl * MN + q * p.M + r : planes,
                    ok ? 16 : 0);
    }
    tp_cp_async_commit();
  };

  const float2 Lp = make_float2(L, L);
  const float2 zero2 = make_float2(0.0f, 0.0f);
  int b = 0;
  issue(0, 0);
  for (int64_t q0 = 0; q0 < p.N; q0 += QS, b ^= 1) {
    if (q0 + QS < p.N) {
      issue(b ^ 1, q0 + QS);
      tp_cp_async_wait<1>();
    } else {
      tp_cp_async_wait<0>();
    }
    __syncthreads();
    const int qmax = (int)((p.N - q0) < QS ? (p.N - q0) : QS);
#pragma unroll 2
    for (int qq = 0; qq < qmax; ++qq) {
      const float4 o4 = *reinterpret_cast<const float4*>(&os[b][qq][4 * tx]);
      const float2 ob[2] = {make_float2(o4.x, o4.y), make_float2(o4.z, o4.w)};
      const float4 rf = *reinterpret_cast<const float4*>(&st[b][0][qq][4 * ty]);
      const float4 aa = *reinterpret_cast<const float4*>(&st[b][1][qq][4 * ty]);
      const float4 bb = *reinterpret_cast<const float4*>(&st[b][2][qq][4 * ty]);
      const float rfv[4] = {rf.x, rf.y, rf.z, rf.w};
      const float av[4] = {aa.x, aa.y, aa.z, aa.w};
      const float bv[4] = {bb.x, bb.y, bb.z, bb.w};
      float2 gs[2] = {zero2, zero2};
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float2 nref = make_float2(-rfv[i], -rfv[i]);
        const float2 A = make_float2(av[i], av[i]);
        const float2 Bp = make_float2(bv[i], bv[i]);
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          float2 t = tp_add2(tp_fma2(Lp, ob[h], own[i][h]), nref);
          t.x = tp_max_nan(t.x, kClampL);
          t.y = tp_max_nan(t.y, kClampL);
          const float2 e = make_float2(tp_ex2(t.x), tp_ex2(t.y));
          const float2 d = tp_mul2(e, tp_fma2(Bp, t, A));
          acc[i][h] = tp_add2(acc[i][h], d);
          gs[h] = tp_add2(gs[h], d);
        }
      }
      // sum over the warp's four row groups, then one store per k quad
      float g4[4] = {rows_ok ? gs[0].x : 0.0f, rows_ok ? gs[0].y : 0.0f,
                     rows_ok ? gs[1].x : 0.0f, rows_ok ? gs[1].y : 0.0f};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        g4[j] += __shfl_xor_sync(0xffffffffu, g4[j], 8);
        g4[j] += __shfl_xor_sync(0xffffffffu, g4[j], 16);
      }
      if (lane < 8)
        *reinterpret_cast<float4*>(&gws[wg][qq][4 * tx]) = make_float4(g4[0], g4[1], g4[2], g4[3]);
    }
    __syncthreads();
    // gW partial of this chunk: add the four warp groups, store k quads
    {
      const int qq = threadIdx.x / 16, kv = threadIdx.x % 16;
      const int64_t q = q0 + qq, k = k0 + 4 * kv;
      if (qq < qmax && k < p.K) {
        float4 sum = *reinterpret_cast<const float4*>(&gws[0][qq][4 * kv]);
#pragma unroll
        for (int g = 1; g < 4; ++g) {
          const float4 v = *reinterpret_cast<const float4*>(&gws[g][qq][4 * kv]);
          sum.x += v.x;
          sum.y += v.y;
          sum.z += v.z;
          sum.w += v.w;
        }
        *reinterpret_cast<float4*>(gpart + q * p.K + k) = sum;
      }
    }
    __syncthreads();   // buffer b and gws are rewritten by the next iteration
  }
  float* out = p.gx + bz * p.M * p.K;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int64_t r = r0 + 4 * ty + i;
    if (r >= p.M) continue;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int64_t k = k0 + 4 * tx + j;
      const float v = j & 1 ? acc[i][j >> 1].y : acc[i][j >> 1].x;
      if (k < p.K) out[r * p.K + k] = v;
    }
  }
}

// out[b][i] = sum_s part[b][s][i], s in increasing order (deterministic).
__global__ void split_sum_kernel(const float* __restrict__ part, int64_t batch, int64_t S,
                                 int64_t n, float* __restrict__ out) {
  const int64_t total = batch * n;
  for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < total;
       e += (int64_t)gridDim.x * blockDim.x) {
    const int64_t b = e / n, i = e % n;
    const float* src = part + b * S * n + i;
    float acc = 0.0f;
    for (int64_t s = 0; s < S; ++s) acc += src[s * n];
    out[e] = acc;
  }
}

inline dim3 generic_grid(int64_t M, int64_t N, int64_t batches) {
  int64_t gz = batches < 65535 ? batches : 65535;
  return dim3((unsigned)ceil_div(N, GB_N), (unsigned)ceil_div(M, GB_M), (unsigned)gz);
}

inline unsigned flat_grid(int64_t total, int threads) {
  int64_t b = ceil_div(total, threads);
  int64_t cap = (int64_t)num_sms() * 32;
  if (b > cap) b = cap;
  if (b < 1) b = 1;
  return (unsigned)b;
}

}  // namespace

template <int TYR>
void launch_fwd_generic_tyr(const StridedMaxPlus& p, dim3 grid, cudaStream_t stream) {
  const bool am = p.am != nullptr;
  const int t = 16 * TYR;
  if (p.dtype == TP_DTYPE_F32) {
    if (am)
      maxplus_fwd_generic_kernel<float, true, false, TYR><<<grid, t, 0, stream>>>(p);
    else
      maxplus_fwd_generic_kernel<float, false, false, TYR><<<grid, t, 0, stream>>>(p);
  } else if (p.dtype == TP_DTYPE_BF16) {
    if (am)
      maxplus_fwd_generic_kernel<uint16_t, true, false, TYR><<<grid, t, 0, stream>>>(p);
    else
      maxplus_fwd_generic_kernel<uint16_t, false, false, TYR><<<grid, t, 0, stream>>>(p);
  } else {
    if (am)
      maxplus_fwd_generic_kernel<uint16_t, true, true, TYR><<<grid, t, 0, stream>>>(p);
    else
      maxplus_fwd_generic_kernel<uint16_t, false, true, TYR><<<grid, t, 0, stream>>>(p);
  }
}

int launch_maxplus_fwd_generic(const StridedMaxPlus& p, cudaStream_t stream) {
  // the tallest tile that still gives every SM two CTAs (16-row tiles at least)
  const int64_t batches = p.B1 * p.B2;
  const int64_t want = 2 * (int64_t)num_sms();
  int tyr = 16;
  while (tyr > 4 && ceil_div(p.M, (int64_t)(4 * tyr)) * ceil_div(p.N, (int64_t)GB_N) *
                            (batches < 65535 ? batches : 65535) < want)
    tyr /= 2;
  dim3 grid = generic_grid(p.M, p.N, batches);
  grid.y = (unsigned)ceil_div(p.M, (int64_t)(4 * tyr));
  if (grid.x > 2147483647u || ceil_div(p.M, (int64_t)(4 * tyr)) > 65535) return TP_ERR_TOO_LARGE;
  if (tyr == 16) launch_fwd_generic_tyr<16>(p, grid, stream);
  else if (tyr == 8) launch_fwd_generic_tyr<8>(p, grid, stream);
  else {
    launch_fwd_generic_tyr<4>(p, grid, stream);
  }
  return launch_status();
}

int launch_maxplus_lse_fwd_generic(const StridedMaxPlus& p, cudaStream_t stream) {
  dim3 grid = generic_grid(p.M, p.N, p.B1 * p.B2);
  if (grid.y > 65535u) return TP_ERR_TOO_LARGE;
  if (p.dtype == TP_DTYPE_F32)
    maxplus_lse_fwd_generic_kernel<float><<<grid, G_THREADS, 0, stream>>>(p);
  else
    maxplus_lse_fwd_generic_kernel<uint16_t><<<grid, G_THREADS, 0, stream>>>(p);
  return launch_status();
}

int launch_strided_zero(float* base, int64_t B1, int64_t B2, int64_t R, int64_t C, int64_t s_b1,
                        int64_t s_b2, int64_t s_r, int64_t s_c, cudaStream_t stream) {
  const int64_t total = B1 * B2 * R * C;
  if (total == 0) return TP_OK;
  // contiguous fast path
  if (s_c == 1 && s_r == C && s_b2 == R * C && s_b1 == B2 * R * C)
    return cuda_status(cudaMemsetAsync(base, 0, (size_t)total * sizeof(float), stream));
  strided_zero_kernel<<<flat_grid(total, 256), 256, 0, stream>>>(base, B1, B2, R, C, s_b1, s_b2,
                                                                  s_r, s_c);
  return launch_status();
}

int launch_maxplus_bwd_argmax(const ScatterArgs& p, cudaStream_t stream) {
  int s = launch_strided_zero(p.gx, p.B1, p.B2, p.M, p.K, p.sgx_b1, p.sgx_b2, p.sgx_m, p.sgx_k,
                              stream);
  if (s != TP_OK) return s;
  if (p.gw) {
    s = launch_strided_zero(p.gw, p.B1, p.B2, p.N, p.K, p.sgw_b1, p.sgw_b2, p.sgw_n, p.sgw_k,
                            stream);
    if (s != TP_OK) return s;
  }
  const int64_t total = p.B1 * p.B2 * p.M * p.N;
  if (total > 0 && p.K > 0) {
    maxplus_bwd_scatter_kernel<<<flat_grid(total, 256), 256, 0, stream>>>(p);
    s = launch_status();
    if (s != TP_OK) return s;
  }
  if (p.gbias) return launch_column_sum(p.gy, p.B1, p.B2, p.M, p.N, p.sg_b1, p.sg_b2, p.sg_m,
                                        p.sg_n, p.scale, p.gbias, stream);
  return TP_OK;
}

int launch_column_sum(const float* g, int64_t B1, int64_t B2, int64_t M, int64_t N, int64_t s_b1,
                      int64_t s_b2, int64_t s_m, int64_t s_n, float scale, float* out,
                      cudaStream_t stream) {
  if (N == 0) return TP_OK;
  column_sum_kernel<<<(unsigned)ceil_div(N, 32), CS_WARPS * 32, 0, stream>>>(
      g, B1, B2, M, N, s_b1, s_b2, s_m, s_n, scale, out);
  return launch_status();
}

// Split the reduced index when the output tiles (64 x 64) give fewer blocks
// than two per SM of a B200 (148 SMs); aim for about four per SM, with at
// least 256 reduced elements per slice.
int64_t smooth_splits(int64_t batch, int64_t rows, int64_t Q, int64_t K) {
  constexpr int64_t kFewBlocks = 2 * 148, kTargetBlocks = 4 * 148, kMinSlice = 256;
  if (batch <= 0 || rows <= 0 || K <= 0 || Q < 2 * kMinSlice) return 1;
  const int64_t tiles = batch * ceil_div(rows, (int64_t)GB_M) * ceil_div(K, (int64_t)GB_N);
  if (tiles >= kFewBlocks) return 1;
  int64_t s = ceil_div(kTargetBlocks, tiles);
  const int64_t by_len = ceil_div(Q, kMinSlice);
  if (s > by_len) s = by_len;
  if (s > 65535 / batch) s = 65535 / batch;
  return s < 1 ? 1 : s;
}

// The one-pass gradient kernel: fp32 staging shapes, gx tiles that fill the
// GPU without splits, and gW partials ([batch][ceil(M/64)][N][K]) of at most
// 16M floats (64 MiB; their write and read cost far less than the pass saved).
bool smooth_fused_ok(int64_t batch, int64_t M, int64_t N, int64_t K) {
  if (batch <= 0 || M <= 0 || N <= 0 || K <= 0) return false;
  if (M % 4 || N % 4 || K % 4) return false;
  if (smooth_splits(batch, M, N, K) != 1) return false;
  const int64_t mt = ceil_div(M, (int64_t)GB_M);
  return mt <= 65535 && batch * mt * N * K <= ((int64_t)1 << 24);
}

int64_t smooth_workspace_floats(int64_t batch, int64_t M, int64_t N, int64_t K) {
  const int64_t sx = smooth_splits(batch, M, N, K), sw = smooth_splits(batch, N, M, K);
  int64_t part = 0;
  if (sx > 1) part = batch * sx * M * K;
  if (sw > 1 && batch * sw * N * K > part) part = batch * sw * N * K;
  if (smooth_fused_ok(batch, M, N, K)) {
    const int64_t f = batch * ceil_div(M, (int64_t)GB_M) * N * K;
    if (f > part) part = f;
  }
  return 6 * batch * M * N + part;
}

int launch_maxplus_bwd_smooth(const SmoothArgs& p, cudaStream_t stream) {
  if (p.batch == 0) return TP_OK;
  if (p.M == 0 || p.N == 0) {
    int s = TP_OK;
    if (p.M > 0 && p.K > 0)
      s = cuda_status(cudaMemsetAsync(p.gx, 0, p.batch * p.M * p.K * 4, stream));
    if (s == TP_OK && p.N > 0 && p.K > 0 && p.gw)
      s = cuda_status(cudaMemsetAsync(p.gw, 0, p.batch * p.N * p.K * 4, stream));
    if (s == TP_OK && p.gbias && p.N > 0)
      s = cuda_status(cudaMemsetAsync(p.gbias, 0, p.N * 4, stream));
    return s;
  }
  if (p.batch > 65535) return TP_ERR_TOO_LARGE;
  const unsigned nb = (unsigned)p.batch;
  dim3 g1((unsigned)ceil_div(p.N, GB_N), (unsigned)ceil_div(p.M, GB_M), nb);
  if (g1.y > 65535u) return TP_ERR_TOO_LARGE;
  if (p.async_stage)
    smooth_stats_async_kernel<<<g1, G_THREADS, 0, stream>>>(p);
  else if (p.dtype == TP_DTYPE_F32)
    smooth_stats_kernel<float><<<g1, G_THREADS, 0, stream>>>(p);
  else
    smooth_stats_kernel<uint16_t><<<g1, G_THREADS, 0, stream>>>(p);
  int s = launch_status();
  if (s != TP_OK) return s;
  if (p.K > 0) {
    const int64_t sx = p.splits_x, sw = p.splits_w;
    if (sx < 1 || sw < 1 || nb * sx > 65535 || nb * sw > 65535) return TP_ERR_INVALID_ARG;
    dim3 gx((unsigned)ceil_div(p.K, GB_N), (unsigned)ceil_div(p.M, GB_M), (unsigned)(nb * sx));
    dim3 gw((unsigned)ceil_div(p.K, GB_N), (unsigned)ceil_div(p.N, GB_M), (unsigned)(nb * sw));
    if (gx.y > 65535u || gw.y > 65535u) return TP_ERR_TOO_LARGE;
    if (p.fused_gw && p.gw && p.async_stage && sx == 1) {
      // one pass for both gradients, then the row tiles' gW partials added
      dim3 gf((unsigned)ceil_div(p.K, GB_N), (unsigned)ceil_div(p.M, GB_M), nb);
      smooth_grad_fused_kernel<<<gf, G_THREADS, 0, stream>>>(p);
      split_sum_kernel<<<flat_grid(p.batch * p.N * p.K, 256), 256, 0, stream>>>(
          p.part, p.batch, (int64_t)gf.y, p.N * p.K, p.gw);
      s = launch_status();
      if (s != TP_OK) return s;
    } else {
    if (p.async_stage)
      smooth_grad_async_kernel<0><<<gx, G_THREADS, 0, stream>>>(p);
    else if (p.dtype == TP_DTYPE_F32)
      smooth_grad_kernel<float, 0><<<gx, G_THREADS, 0, stream>>>(p);
    else
      smooth_grad_kernel<uint16_t, 0><<<gx, G_THREADS, 0, stream>>>(p);
    if (sx > 1)
      split_sum_kernel<<<flat_grid(p.batch * p.M * p.K, 256), 256, 0, stream>>>(
          p.part, p.batch, sx, p.M * p.K, p.gx);
    s = launch_status();
    if (s != TP_OK) return s;
    if (p.gw) {
      if (p.async_stage)
        smooth_grad_async_kernel<1><<<gw, G_THREADS, 0, stream>>>(p);
      else if (p.dtype == TP_DTYPE_F32)
        smooth_grad_kernel<float, 1><<<gw, G_THREADS, 0, stream>>>(p);
      else
        smooth_grad_kernel<uint16_t, 1><<<gw, G_THREADS, 0, stream>>>(p);
      if (sw > 1)
        split_sum_kernel<<<flat_grid(p.batch * p.N * p.K, 256), 256, 0, stream>>>(
            p.part, p.batch, sw, p.N * p.K, p.gw);
      s = launch_status();
      if (s != TP_OK) return s;
    }
    }
  }
  if (p.gbias)
    return launch_column_sum(p.gy, p.batch, 1, p.M, p.N, p.M * p.N, 0, p.N, 1, 1.0f, p.gbias,
                             stream);
  return TP_OK;
}

}  // namespace tp

// ---------------------------------------------------------------------------
// bf16 -> fp32 widening (exact): 8 elements (16 bytes in, 32 bytes out) per
// thread step when both pointers allow it, scalar otherwise.
// ---------------------------------------------------------------------------
namespace tp {
namespace {
__global__ void bf16_to_f32_kernel(const uint16_t* __restrict__ src, float* __restrict__ dst,
                                   int64_t n, bool vec) {
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  const int64_t tid = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  int64_t done = 0;
  if (vec) {
    const int64_t n8 = n / 8;
    const uint4* s4 = reinterpret_cast<const uint4*>(src);
    float4* d4 = reinterpret_cast<float4*>(dst);
    for (int64_t i = tid; i < n8; i += stride) {
      const uint4 v = __ldg(s4 + i);
      const uint32_t w[4] = {v.x, v.y, v.z, v.w};
      float f[8];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        f[2 * j] = __uint_as_float(w[j] << 16);
        f[2 * j + 1] = __uint_as_float(w[j] & 0xffff0000u);
      }
      d4[2 * i] = make_float4(f[0], f[1], f[2], f[3]);
      d4[2 * i + 1] = make_float4(f[4], f[5], f[6], f[7]);
    }
    done = n8 * 8;
  }
  for (int64_t i = done + tid; i < n; i += stride) dst[i] = tp_bf16_to_f32(src[i]);
}
}  // namespace

int launch_bf16_to_f32(const void* src, float* dst, int64_t n, cudaStream_t stream) {
  if (n == 0) return TP_OK;
  const bool vec = aligned16(src) && aligned16(dst);
  int64_t blocks = ceil_div(n, 256 * 8);
  const int64_t cap = (int64_t)num_sms() * 16;
  if (blocks > cap) blocks = cap;
  bf16_to_f32_kernel<<<(unsigned)blocks, 256, 0, stream>>>((const uint16_t*)src, dst, n, vec);
  return launch_status();
}
}  // namespace tp
