// split_tf32.cu -- x = hi + lo with hi exactly representable in TF32 (the low 13
// mantissa bits of x cleared) and lo = x - hi (exact in fp32).  Three TF32
// tensor-core products hi.hi + hi.lo + lo.hi then give an fp32-accurate
// product (the dropped lo.lo term is below 2^-22 of it; lo's own TF32
// rounding adds ~2^-21): the projections around the tropical kernels run on
// the tensor cores at fp32-level accuracy.  One read, two writes, 16 bytes
// per thread and step.
#include "maxplus_internal.cuh"

namespace tp {

namespace {

__device__ __forceinline__ void split1(float x, float& hi, float& lo) {
  hi = __uint_as_float(__float_as_uint(x) & 0xffffe000u);
  // a non-finite x keeps its value in hi (lo = 0, not inf - inf)
  lo = isfinite(x) ? x - hi : 0.0f;
}

__global__ void __launch_bounds__(256) split_tf32_kernel(const float* __restrict__ x, int64_t n,
                                                         float* __restrict__ hi,
                                                         float* __restrict__ lo) {
  const int64_t n4 = n >> 2;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n4; i += stride) {
    const float4 v = reinterpret_cast<const float4*>(x)[i];
    float4 h, l;
    split1(v.x, h.x, l.x);
    split1(v.y, h.y, l.y);
    split1(v.z, h.z, l.z);
    split1(v.w, h.w, l.w);
    reinterpret_cast<float4*>(hi)[i] = h;
    reinterpret_cast<float4*>(lo)[i] = l;
  }
  // the tail past the last multiple of 4
  const int64_t t = (n4 << 2) + (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (t < n && t < (n4 << 2) + 4) split1(x[t], hi[t], lo[t]);
}

// Row-concatenated parts: out[r] = [part0 | part1 (| part2)] of x's row r
// (cols values each, row stride nparts cols), part p = lo where bit p of
// lo_mask is set, else hi.  [xh | xl] against [wl | wh] is the two
// correction products hi.lo + lo.hi as ONE GEMM of depth 2 K, accumulated on
// top of hi.hi: the output is read and written once for both.  Four columns
// per thread.
__global__ void __launch_bounds__(256) split_tf32_cat_kernel(const float* __restrict__ x,
                                                             int64_t rows, int64_t cols,
                                                             float* __restrict__ out, int nparts,
                                                             int lo_mask) {
  const int64_t q4 = cols >> 2;
  const int64_t total = rows * q4;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += stride) {
    const int64_t r = i / q4, q = i - r * q4;
    const float4 v = reinterpret_cast<const float4*>(x + r * cols)[q];
    float4 h, l;
    split1(v.x, h.x, l.x);
    split1(v.y, h.y, l.y);
    split1(v.z, h.z, l.z);
    split1(v.w, h.w, l.w);
    float4* o = reinterpret_cast<float4*>(out + r * nparts * cols);
    for (int p = 0; p < nparts; ++p) o[p * q4 + q] = ((lo_mask >> p) & 1) ? l : h;
  }
}

}  // namespace

int launch_split_tf32_cat(const float* x, int64_t rows, int64_t cols, float* out, int nparts,
                          int lo_mask, cudaStream_t stream) {
  if (rows == 0 || cols == 0) return TP_OK;
  const int64_t want = ceil_div(rows * (cols >> 2), (int64_t)256);
  const int64_t cap = (int64_t)num_sms() * 8;
  const int64_t blocks = want < cap ? (want > 0 ? want : 1) : cap;
  split_tf32_cat_kernel<<<(unsigned)blocks, 256, 0, stream>>>(x, rows, cols, out, nparts,
                                                              lo_mask);
  return launch_status();
}

int launch_split_tf32(const float* x, int64_t n, float* hi, float* lo, cudaStream_t stream) {
  if (n == 0) return TP_OK;
  int sms = 148;
  int dev = 0;
  if (cudaGetDevice(&dev) == cudaSuccess)
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int64_t want = ceil_div(n >> 2, (int64_t)256);
  const int64_t blocks = want < (int64_t)sms * 8 ? (want > 0 ? want : 1) : (int64_t)sms * 8;
  split_tf32_kernel<<<(unsigned)blocks, 256, 0, stream>>>(x, n, hi, lo);
  return launch_status();
}

}  // namespace tp
