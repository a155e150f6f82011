// probe.cu -- register-only microbenchmark of the CUDA-core max-plus term rate.
//
// It measures how close a loop of nothing but max-plus arithmetic gets to the
// issue limit of the GEMM kernel's instruction form (one add.f32x2 and one
// 3-input max per two terms: 128 terms per clock per SM).  Each thread keeps
// an 8x8 block of independent accumulators (the GEMM's register tile) and
// folds 128 terms per iteration.  The x operands are advanced by one packed
// add each per iteration (8 extra adds per 128 terms) so that no sum is loop
// invariant -- otherwise the compiler hoists every add out of the loop and
// the loop measures the max instruction alone.
//   form 0: add.rn.f32 + 2-input max.f32 per term (4 instructions / 2 terms)
//   form 1: add.rn.f32x2 + 3-input max.f32 per two terms (2 instructions)
//   form 2: add.rn.f32x2 + 3-input max.NaN.f32
//   form 3: two add.rn.f32 + 3-input max.NaN.f32 per two terms (3 instructions)
//   form 4: forms 2 and 3 alternating over the outputs
//   form 5: add.rn.bf16x2 + 2-input max.bf16x2 per two terms (packed bf16
//           arithmetic; there is no 3-input packed max)
//   form 6: add.rn.bf16x2 + max.NaN.bf16x2
//   form 7: fp32 fused multiply-add (two per accumulator and iteration; one
//           "term" = one FMA = 2 flops), the CUDA-core roofline of dot products
//   form 9: packed fp32 FMA pairs (fma.rn.f32x2; a term is one FMA)
//   form 8: the smooth (STE / LSE) backward's per-term shape: packed adds
//           forming s - max, a clamp, ex2.approx per term, a packed add into
//           the partition sum and a packed FMA into the first moment (one
//           "term" = one exponential): the SFU-bound roofline of those passes
#include "maxplus_internal.cuh"

namespace tp {

namespace {

template <int FORM>
__device__ __forceinline__ void term_pair(float& acc, uint64_t xa, uint64_t wb) {
  if (FORM == 0) {
    asm volatile(
        "{\n\t.reg .f32 x0, x1, w0, w1, s0, s1;\n\t"
        "mov.b64 {x0, x1}, %1;\n\tmov.b64 {w0, w1}, %2;\n\t"
        "add.rn.f32 s0, x0, w0;\n\tadd.rn.f32 s1, x1, w1;\n\t"
        "max.f32 %0, %0, s0;\n\tmax.f32 %0, %0, s1;\n\t}"
        : "+f"(acc)
        : "l"(xa), "l"(wb));
  } else if (FORM == 1) {
    asm volatile(
        "{\n\t.reg .b64 s;\n\t.reg .f32 lo, hi;\n\t"
        "add.rn.f32x2 s, %1, %2;\n\tmov.b64 {lo, hi}, s;\n\t"
        "max.f32 %0, %0, lo, hi;\n\t}"
        : "+f"(acc)
        : "l"(xa), "l"(wb));
  } else if (FORM == 2) {
    asm volatile(
        "{\n\t.reg .b64 s;\n\t.reg .f32 lo, hi;\n\t"
        "add.rn.f32x2 s, %1, %2;\n\tmov.b64 {lo, hi}, s;\n\t"
        "max.NaN.f32 %0, %0, lo, hi;\n\t}"
        : "+f"(acc)
        : "l"(xa), "l"(wb));
  } else {
    asm volatile(
        "{\n\t.reg .f32 x0, x1, w0, w1, s0, s1;\n\t"
        "mov.b64 {x0, x1}, %1;\n\tmov.b64 {w0, w1}, %2;\n\t"
        "add.rn.f32 s0, x0, w0;\n\tadd.rn.f32 s1, x1, w1;\n\t"
        "max.NaN.f32 %0, %0, s0, s1;\n\t}"
        : "+f"(acc)
        : "l"(xa), "l"(wb));
  }
}

template <int FORM>
__global__ void __launch_bounds__(256) probe_kernel(int64_t iters, float* sink) {
  const int t = blockIdx.x * blockDim.x + threadIdx.x;
  uint64_t xa[8], wb[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const float f0 = (float)(t % 97) * 0.01f + (float)i;
    const float f1 = (float)(t % 89) * 0.02f - (float)i;
    xa[i] = ((uint64_t)__float_as_uint(f1) << 32) | __float_as_uint(f0);
    wb[i] = ((uint64_t)__float_as_uint(f0 * 0.5f) << 32) | __float_as_uint(f1 * 0.25f);
  }
  float acc[8][8];
#pragma unroll
  for (int i = 0; i < 8; ++i)
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[i][j] = -1.0e30f;
  const uint64_t step = ((uint64_t)__float_as_uint(1.0e-3f) << 32) | __float_as_uint(-1.0e-3f);
  for (int64_t it = 0; it < iters; ++it) {
#pragma unroll
    for (int i = 0; i < 8; ++i)
      asm volatile("add.rn.f32x2 %0, %0, %1;" : "+l"(xa[i]) : "l"(step));
#pragma unroll
    for (int j = 0; j < 8; ++j)
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        if (FORM == 4) {
          if ((i + j) & 1) term_pair<2>(acc[i][j], xa[i], wb[j]);
          else term_pair<3>(acc[i][j], xa[i], wb[j]);
        } else {
          term_pair<FORM>(acc[i][j], xa[i], wb[j]);
        }
      }
  }
  float r = 0.0f;
#pragma unroll
  for (int i = 0; i < 8; ++i)
#pragma unroll
    for (int j = 0; j < 8; ++j) r += acc[i][j];
  sink[t] = r;
}

// bf16x2 forms: each register holds two bf16 lanes; per pair of terms one
// packed add and one packed max into a two-lane accumulator
template <bool kNaN>
__global__ void __launch_bounds__(256) probe_bf16_kernel(int64_t iters, float* sink) {
  const int t = blockIdx.x * blockDim.x + threadIdx.x;
  uint32_t xa[8], wb[8], acc[8][8];
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const float f0 = (float)(t % 97) * 0.01f + (float)i;
    const float f1 = (float)(t % 89) * 0.02f - (float)i;
    xa[i] = (__float_as_uint(f1) & 0xffff0000u) | (__float_as_uint(f0) >> 16);
    wb[i] = (__float_as_uint(f0 * 0.5f) & 0xffff0000u) | (__float_as_uint(f1 * 0.25f) >> 16);
  }
#pragma unroll
  for (int i = 0; i < 8; ++i)
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[i][j] = 0xff80ff80u;   // two -inf lanes
  const uint32_t step = (__float_as_uint(1.0e-2f) & 0xffff0000u) | (__float_as_uint(-1.0e-2f) >> 16);
  for (int64_t it = 0; it < iters; ++it) {
#pragma unroll
    for (int i = 0; i < 8; ++i) asm volatile("add.rn.bf16x2 %0, %0, %1;" : "+r"(xa[i]) : "r"(step));
#pragma unroll
    for (int j = 0; j < 8; ++j)
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        if (kNaN)
          asm volatile("{\n\t.reg .b32 s;\n\tadd.rn.bf16x2 s, %1, %2;\n\t"
                       "max.NaN.bf16x2 %0, %0, s;\n\t}"
                       : "+r"(acc[i][j]) : "r"(xa[i]), "r"(wb[j]));
        else
          asm volatile("{\n\t.reg .b32 s;\n\tadd.rn.bf16x2 s, %1, %2;\n\t"
                       "max.bf16x2 %0, %0, s;\n\t}"
                       : "+r"(acc[i][j]) : "r"(xa[i]), "r"(wb[j]));
      }
  }
  float r = 0.0f;
#pragma unroll
  for (int i = 0; i < 8; ++i)
#pragma unroll
    for (int j = 0; j < 8; ++j) r += __uint_as_float(acc[i][j] << 16) + __uint_as_float(acc[i][j] & 0xffff0000u);
  sink[t] = r;
}

// packed fp32 FMA pairs (fma.rn.f32x2): 32 accumulator pairs, two sweeps of
// independent instructions per iteration; a "term" is one FMA (2 flops)
__global__ void __launch_bounds__(256) probe_ffma2_kernel(int64_t iters, float* sink) {
  const int t = blockIdx.x * blockDim.x + threadIdx.x;
  float2 a[4], b[8], acc[4][8];
#pragma unroll
  for (int i = 0; i < 4; ++i)
    a[i] = make_float2((float)(t % 97) * 1e-3f + (float)i * 1e-2f,
                       (float)(t % 83) * 1e-3f + (float)i * 2e-2f);
#pragma unroll
  for (int j = 0; j < 8; ++j)
    b[j] = make_float2(1.0f - (float)(t % 89) * 1e-4f - (float)j * 1e-3f,
                       1.0f - (float)(t % 79) * 1e-4f - (float)j * 2e-3f);
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[i][j] = make_float2(0.0f, 0.0f);
  const float2 step = make_float2(1e-3f, 1e-3f);
  for (int64_t it = 0; it < iters; ++it) {
#pragma unroll
    for (int i = 0; i < 4; ++i) a[i] = tp_add2(a[i], step);
#pragma unroll
    for (int sweep = 0; sweep < 2; ++sweep)
#pragma unroll
      for (int j = 0; j < 8; ++j)
#pragma unroll
        for (int i = 0; i < 4; ++i) acc[i][j] = tp_fma2(a[i], b[j], acc[i][j]);
  }
  float r = 0.0f;
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 8; ++j) r += acc[i][j].x + acc[i][j].y;
  sink[t] = r;
}

__global__ void __launch_bounds__(256) probe_ffma_kernel(int64_t iters, float* sink) {
  const int t = blockIdx.x * blockDim.x + threadIdx.x;
  float a[8], b[8], acc[8][8];
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    a[i] = (float)(t % 97) * 1e-3f + (float)i * 1e-2f;
    b[i] = 1.0f - (float)(t % 89) * 1e-4f - (float)i * 1e-3f;
  }
#pragma unroll
  for (int i = 0; i < 8; ++i)
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[i][j] = 0.0f;
  for (int64_t it = 0; it < iters; ++it) {
#pragma unroll
    for (int i = 0; i < 8; ++i) asm volatile("add.rn.f32 %0, %0, 0f3A83126F;" : "+f"(a[i]));
    // two sweeps over the 64 accumulators: consecutive FMAs are independent
    // (volatile asm keeps program order, so a dependent pair issued back to
    // back would wait out the FMA latency every time)
#pragma unroll
    for (int j = 0; j < 8; ++j)
#pragma unroll
      for (int i = 0; i < 8; ++i)
        asm volatile("fma.rn.f32 %0, %1, %2, %0;" : "+f"(acc[i][j]) : "f"(a[i]), "f"(b[j]));
#pragma unroll
    for (int j = 0; j < 8; ++j)
#pragma unroll
      for (int i = 0; i < 8; ++i)
        asm volatile("fma.rn.f32 %0, %1, %2, %0;" : "+f"(acc[i][j]) : "f"(b[j]), "f"(a[i]));
  }
  float r = 0.0f;
#pragma unroll
  for (int i = 0; i < 8; ++i)
#pragma unroll
    for (int j = 0; j < 8; ++j) r += acc[i][j];
  sink[t] = r;
}

__global__ void __launch_bounds__(256) probe_smooth_kernel(int64_t iters, float* sink) {
  const int t = blockIdx.x * blockDim.x + threadIdx.x;
  float2 a[4], n[4], b[8], Z[4][8], S1[4][8];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    a[i] = make_float2(-1.0f - (float)(t % 97) * 1e-3f, -1.5f + (float)i * 1e-2f);
    n[i] = make_float2(-2.0f + (float)i * 1e-3f, -2.5f);
  }
#pragma unroll
  for (int j = 0; j < 8; ++j) b[j] = make_float2(-(float)(t % 89) * 1e-3f, -0.25f * (float)j);
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 8; ++j) Z[i][j] = S1[i][j] = make_float2(0.0f, 0.0f);
  const float2 step = make_float2(1.0e-7f, -1.0e-7f);
  for (int64_t it = 0; it < iters; ++it) {
#pragma unroll
    for (int k = 0; k < 2; ++k) {            // two k steps of 4 x 8 x 2 terms
#pragma unroll
      for (int i = 0; i < 4; ++i) a[i] = tp_add2(a[i], step);
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          float2 s = tp_add2(tp_add2(a[i], b[j]), n[i]);
          s.x = tp_max_nan(s.x, -256.0f);
          s.y = tp_max_nan(s.y, -256.0f);
          const float2 e = make_float2(tp_ex2(s.x), tp_ex2(s.y));
          Z[i][j] = tp_add2(Z[i][j], e);
          S1[i][j] = tp_fma2(e, s, S1[i][j]);
        }
    }
  }
  float r = 0.0f;
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 8; ++j) r += Z[i][j].x + Z[i][j].y + S1[i][j].x + S1[i][j].y;
  sink[t] = r;
}

}  // namespace

int launch_probe_addmax(int form, int64_t blocks, int64_t threads, int64_t iters, float* sink,
                        cudaStream_t stream) {
  if (threads != 256) return TP_ERR_INVALID_ARG;
  if (form == 0)
    probe_kernel<0><<<(unsigned)blocks, 256, 0, stream>>>(iters, sink);
  else if (form == 1)
    probe_kernel<1><<<(unsigned)blocks, 256, 0, stream>>>(iters, sink);
  else if (form == 2)
    probe_kernel<2><<<(unsigned)blocks, 256, 0, stream>>>(iters, sink);
  else if (form == 3)
    probe_kernel<3><<<(unsigned)blocks, 256, 0, stream>>>(iters, sink);
  else if (form == 4)
    probe_kernel<4><<<(unsigned)blocks, 256, 0, stream>>>(iters, sink);
  else if (form == 5)
    probe_bf16_kernel<false><<<(unsigned)blocks, 256, 0, stream>>>(iters, sink);
  else if (form == 6)
    probe_bf16_kernel<true><<<(unsigned)blocks, 256, 0, stream>>>(iters, sink);
  else if (form == 7)
    probe_ffma_kernel<<<(unsigned)blocks, 256, 0, stream>>>(iters, sink);
  else if (form == 8)
    probe_smooth_kernel<<<(unsigned)blocks, 256, 0, stream>>>(iters, sink);
  else if (form == 9)
    probe_ffma2_kernel<<<(unsigned)blocks, 256, 0, stream>>>(iters, sink);
  else
    return TP_ERR_INVALID_ARG;
  return launch_status();
}

}  // namespace tp
