// common.cuh -- shared helpers for the sm_100a tropical kernels.
//
// Host side: status codes, argument validation helpers, a lazily resolved
// cuTensorMapEncodeTiled (through cudaGetDriverEntryPoint, so the library
// needs no -lcuda), and pointer checks.
// Device side: NaN-propagating max, packed f32x2 add, mbarrier and TMA
// wrappers whose waits are bounded by a wall-clock budget.  A wait that runs
// out records an error code in the library's device error word (its address
// is passed to every kernel that waits) and returns false; callers then stop
// issuing work and exit, so the context stays usable.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdint.h>

#include "tropical_b200.h"

// ---------------------------------------------------------------------------
// device status block (module-scope device memory, not a per-call allocation)
// ---------------------------------------------------------------------------
// Kernels that wait receive `int* err`, the address of `error` below; the
// budget of every bounded wait is read from the same block, so the host can
// change it at run time (tp_set_wait_budget_ns).  Error codes
// TP_DEVERR_BARRIER_TIMEOUT / TP_DEVERR_FLAG_TIMEOUT are in tropical_b200.h.
struct TpDeviceStatus {
  int error;                          // 0, or the first TP_DEVERR_* recorded
  int reserved;
  unsigned long long wait_budget_ns;  // %globaltimer budget of one bounded wait
};

// Default bounded-wait budget: 2 seconds of %globaltimer (ns).
#define TP_WAIT_BUDGET_NS 2000000000ull

__device__ __forceinline__ uint64_t tp_globaltimer() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ void tp_record_device_error(int* err, int code) {
  if (err) atomicCAS(err, 0, code);
}

// The wait budget of the status block that `err` belongs to (read when a wait
// first fails to complete, so the fast path never touches it).
__device__ __forceinline__ uint64_t tp_wait_budget(const int* err) {
  if (err == nullptr) return TP_WAIT_BUDGET_NS;
  const TpDeviceStatus* st = reinterpret_cast<const TpDeviceStatus*>(err);
  return *reinterpret_cast<const volatile unsigned long long*>(&st->wait_budget_ns);
}

// ---------------------------------------------------------------------------
// arithmetic helpers
// ---------------------------------------------------------------------------
__device__ __forceinline__ float tp_max_nan(float a, float b) {
  float r;
  asm("max.NaN.f32 %0, %1, %2;" : "=f"(r) : "f"(a), "f"(b));
  return r;
}

// 3-input NaN-propagating max (one instruction on sm_100a)
__device__ __forceinline__ float tp_max3_nan(float a, float b, float c) {
  float r;
  asm("max.NaN.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
  return r;
}

// Packed fp32 pairs (sm_100a add/mul/fma .f32x2): each half is an ordinary
// round-to-nearest fp32 add / multiply / fused multiply-add, two per
// instruction.
__device__ __forceinline__ float2 tp_add2(float2 a, float2 b) {
  float2 r;
  asm("{\n\t.reg .b64 pa, pb, pr;\n\t"
      "mov.b64 pa, {%2, %3};\n\tmov.b64 pb, {%4, %5};\n\t"
      "add.rn.f32x2 pr, pa, pb;\n\tmov.b64 {%0, %1}, pr;\n\t}"
      : "=f"(r.x), "=f"(r.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
  return r;
}

__device__ __forceinline__ float2 tp_mul2(float2 a, float2 b) {
  float2 r;
  asm("{\n\t.reg .b64 pa, pb, pr;\n\t"
      "mov.b64 pa, {%2, %3};\n\tmov.b64 pb, {%4, %5};\n\t"
      "mul.rn.f32x2 pr, pa, pb;\n\tmov.b64 {%0, %1}, pr;\n\t}"
      : "=f"(r.x), "=f"(r.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
  return r;
}

__device__ __forceinline__ float2 tp_fma2(float2 a, float2 b, float2 c) {
  float2 r;
  asm("{\n\t.reg .b64 pa, pb, pc, pr;\n\t"
      "mov.b64 pa, {%2, %3};\n\tmov.b64 pb, {%4, %5};\n\tmov.b64 pc, {%6, %7};\n\t"
      "fma.rn.f32x2 pr, pa, pb, pc;\n\tmov.b64 {%0, %1}, pr;\n\t}"
      : "=f"(r.x), "=f"(r.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y), "f"(c.x), "f"(c.y));
  return r;
}

// 2^x with the hardware approximation (PTX ex2.approx.ftz.f32: relative error
// about 2^-22, subnormal results flushed to zero, 2^-inf = 0).
__device__ __forceinline__ float tp_ex2(float x) {
  float r;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(x));
  return r;
}

__device__ __forceinline__ float tp_bf16_to_f32(uint16_t v) {
  return __uint_as_float(((uint32_t)v) << 16);
}

template <typename T>
__device__ __forceinline__ float tp_load_as_f32(const T* p);
template <>
__device__ __forceinline__ float tp_load_as_f32<float>(const float* p) { return __ldg(p); }
template <>
__device__ __forceinline__ float tp_load_as_f32<uint16_t>(const uint16_t* p) {
  return tp_bf16_to_f32(__ldg(p));
}

// ---------------------------------------------------------------------------
// shared-memory / mbarrier / TMA wrappers (sm_90+ PTX, used on sm_100a)
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t tp_smem_addr(const void* p) {
  return (uint32_t)__cvta_generic_to_shared(p);
}

__device__ __forceinline__ void tp_mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(tp_smem_addr(bar)), "r"(count));
}

__device__ __forceinline__ void tp_fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void tp_fence_proxy_async() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void tp_mbar_arrive(uint64_t* bar) {
  asm volatile(
      "{\n\t.reg .b64 st;\n\t"
      "mbarrier.arrive.shared::cta.b64 st, [%0];\n\t}" ::"r"(tp_smem_addr(bar))
      : "memory");
}

__device__ __forceinline__ void tp_mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile(
      "{\n\t.reg .b64 st;\n\t"
      "mbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n\t}" ::"r"(tp_smem_addr(bar)),
      "r"(bytes)
      : "memory");
}

__device__ __forceinline__ bool tp_mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(tp_smem_addr(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Wait until the phase with the given parity completes.  Returns false (and
// records TP_DEVERR_BARRIER_TIMEOUT) if the budget runs out.
__device__ __forceinline__ bool tp_mbar_wait(uint64_t* bar, uint32_t parity, int* err) {
  if (tp_mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = tp_globaltimer();
  const uint64_t budget = tp_wait_budget(err);
  uint32_t polls = 0;
  while (!tp_mbar_try_wait(bar, parity)) {
    if (((++polls) & 255u) == 0u) {
      if (tp_globaltimer() - t0 > budget) {
        tp_record_device_error(err, TP_DEVERR_BARRIER_TIMEOUT);
        return false;
      }
    }
  }
  return true;
}

// Wait until the global flag word reads 1 (acquire load, GPU scope: the
// writer releases it after storing the data it guards).  Returns false (and
// records TP_DEVERR_FLAG_TIMEOUT) if the budget runs out.
__device__ __forceinline__ bool tp_flag_wait(const unsigned* flag, int* err) {
  uint64_t t0 = 0, budget = 0;
  uint32_t polls = 0;
  while (true) {
    unsigned f;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(f) : "l"(flag) : "memory");
    if (f == 1u) return true;
    if (polls == 0) {
      t0 = tp_globaltimer();
      budget = tp_wait_budget(err);
    }
    if (((++polls) & 63u) == 0u && tp_globaltimer() - t0 > budget) {
      tp_record_device_error(err, TP_DEVERR_FLAG_TIMEOUT);
      return false;
    }
  }
}

// Asynchronous 16-byte global -> shared copy (L2 only); bytes past
// src_bytes (0 or 16) are zero-filled and not read.
__device__ __forceinline__ void tp_cp_async16(void* smem_dst, const void* gsrc, int src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(tp_smem_addr(smem_dst)),
               "l"(gsrc), "r"(src_bytes)
               : "memory");
}
// 4-byte variant (through L1); src_bytes 0 zero-fills without reading
__device__ __forceinline__ void tp_cp_async4(void* smem_dst, const void* gsrc, int src_bytes) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;" ::"r"(tp_smem_addr(smem_dst)),
               "l"(gsrc), "r"(src_bytes)
               : "memory");
}
__device__ __forceinline__ void tp_cp_async_commit() {
  asm volatile("cp.async.commit_group;" ::: "memory");
}
// wait until at most `N` of this thread's committed copy groups are pending
template <int N>
__device__ __forceinline__ void tp_cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// 2-D tiled TMA load (no multicast) into shared memory, completing on `bar`.
__device__ __forceinline__ void tp_tma_load_2d(void* smem_dst, const CUtensorMap* map,
                                               int32_t c0, int32_t c1, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3}], [%4];" ::"r"(tp_smem_addr(smem_dst)),
      "l"((uint64_t)map), "r"(c0), "r"(c1), "r"(tp_smem_addr(bar))
      : "memory");
}

__device__ __forceinline__ void tp_prefetch_tensormap(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"((uint64_t)map) : "memory");
}

// ---------------------------------------------------------------------------
// host helpers
// ---------------------------------------------------------------------------
namespace tp {

int check_device_pointer(const void* p);   // TP_OK or TP_ERR_BAD_POINTER
bool pointer_checks_enabled();

// Resolve cuTensorMapEncodeTiled through the runtime (no -lcuda).  Returns
// nullptr if the driver does not provide it.
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                  const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                  const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);
EncodeTiledFn encode_tiled();

inline int cuda_status(cudaError_t e) { return e == cudaSuccess ? TP_OK : (int)e; }

inline int launch_status() { return cuda_status(cudaGetLastError()); }

inline bool aligned16(const void* p) { return (((uintptr_t)p) & 15u) == 0; }

__host__ __device__ inline int64_t ceil_div(int64_t a, int64_t b) { return (a + b - 1) / b; }

int num_sms();

// Device address of the library's error word on the current device (resolved
// once per device with cudaGetSymbolAddress); nullptr if unavailable.
int* device_error_ptr();

}  // namespace tp

#define TP_RETURN_IF(cond, code) \
  do {                           \
    if (cond) return (code);     \
  } while (0)

#define TP_CHECK_PTR(p)                                     \
  do {                                                      \
    if ((p) == nullptr) return TP_ERR_NULL_POINTER;         \
    if (tp::pointer_checks_enabled()) {                     \
      int _s = tp::check_device_pointer((const void*)(p));  \
      if (_s != TP_OK) return _s;                           \
    }                                                       \
  } while (0)

#define TP_CHECK_OPT_PTR(p)                                 \
  do {                                                      \
    if ((p) != nullptr && tp::pointer_checks_enabled()) {   \
      int _s = tp::check_device_pointer((const void*)(p));  \
      if (_s != TP_OK) return _s;                           \
    }                                                       \
  } while (0)
