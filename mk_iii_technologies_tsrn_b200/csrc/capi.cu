// capi.cu -- the extern "C" boundary (include/tropical_b200.h).
//
// Every entry point validates its arguments on the host, then launches on the
// caller's stream and returns a status code.  No entry point allocates device
// memory or synchronises.  Reference interface replaced:
// cuda/maxplus_gemm.cu:297-341 (launchers) and cuda/maxplus_binding.py:42-97
// (the ctypes calls that fed them).
#include <atomic>
#include <mutex>

#include "maxplus_internal.cuh"

// One per GPU that loads the library: the device error word and the budget
// of every bounded wait (TpDeviceStatus, common.cuh).
__device__ TpDeviceStatus g_tp_status = {0, 0, TP_WAIT_BUDGET_NS};

namespace tp {

namespace {
std::atomic<int> g_pointer_checks{1};
std::atomic<int> g_smooth_fused{1};
thread_local int g_last_error = TP_OK;
}  // namespace

bool pointer_checks_enabled() { return g_pointer_checks.load(std::memory_order_relaxed) != 0; }

int check_device_pointer(const void* p) {
  cudaPointerAttributes attr;
  cudaError_t e = cudaPointerGetAttributes(&attr, p);
  if (e != cudaSuccess) {
    cudaGetLastError();  // clear the sticky-free error state
    return TP_ERR_BAD_POINTER;
  }
  if (attr.type != cudaMemoryTypeDevice && attr.type != cudaMemoryTypeManaged)
    return TP_ERR_BAD_POINTER;
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess) return TP_ERR_BAD_POINTER;
  if (attr.type == cudaMemoryTypeDevice && attr.device != dev) return TP_ERR_BAD_POINTER;
  return TP_OK;
}

EncodeTiledFn encode_tiled() {
  static std::once_flag once;
  static EncodeTiledFn fn = nullptr;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(ptr);
  });
  return fn;
}

int* device_error_ptr() {
  static std::mutex mu;
  static int* ptrs[64] = {nullptr};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
  std::lock_guard<std::mutex> lock(mu);
  if (ptrs[dev] == nullptr) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_tp_status) == cudaSuccess)
      ptrs[dev] = &static_cast<TpDeviceStatus*>(p)->error;
    else
      cudaGetLastError();
  }
  return ptrs[dev];
}

int num_sms() {
  int dev = 0, n = 148;
  if (cudaGetDevice(&dev) == cudaSuccess)
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  return n > 0 ? n : 148;
}

int check_scan_bwd_pointers(int64_t T, const float* gh, const float* bb, const float* xx,
                            const float* a, const float* h0, const float* h,
                            const uint32_t* win_mask, const float* gu, const float* ga,
                            const float* gh0) {
  TP_CHECK_PTR(a);
  TP_CHECK_OPT_PTR(h0);
  TP_CHECK_OPT_PTR(ga);
  TP_CHECK_OPT_PTR(gh0);
  if (T > 0) {
    TP_CHECK_PTR(gh);
    TP_CHECK_PTR(gu);
    if (win_mask) {
      TP_CHECK_PTR(win_mask);
    } else {
      TP_CHECK_PTR(bb);
      TP_CHECK_OPT_PTR(xx);
      TP_CHECK_PTR(h);
    }
  }
  return TP_OK;
}

// One warp; lane 0 runs a bounded wait that nothing can satisfy (see
// tp_selftest_bounded_wait).  The mbarrier expects two arrivals and gets one.
__global__ void selftest_wait_kernel(int kind, const unsigned* flag, int* err) {
  __shared__ __align__(8) uint64_t bar;
  if (threadIdx.x != 0) return;
  if (kind == 0) {
    tp_mbar_init(&bar, 2);
    tp_fence_mbar_init();
    tp_mbar_arrive(&bar);
    (void)tp_mbar_wait(&bar, 0u, err);
  } else {
    (void)tp_flag_wait(flag, err);
  }
}

int launch_selftest_wait(int kind, const unsigned* flag, cudaStream_t stream) {
  int* err = device_error_ptr();
  if (err == nullptr) return TP_ERR_UNSUPPORTED;
  selftest_wait_kernel<<<1, 32, 0, stream>>>(kind, flag, err);
  return launch_status();
}

static void set_last_error(int s) { g_last_error = s; }
static int last_error() { return g_last_error; }

}  // namespace tp

using namespace tp;

static inline cudaStream_t as_stream(void* s) { return reinterpret_cast<cudaStream_t>(s); }

static int validate_strided(const StridedMaxPlus& p) {
  TP_RETURN_IF(p.dtype != TP_DTYPE_F32 && p.dtype != TP_DTYPE_BF16 &&
                   p.dtype != TP_DTYPE_BF16_ARITH,
               TP_ERR_UNSUPPORTED);
  TP_RETURN_IF(p.B1 < 0 || p.B2 < 0 || p.M < 0 || p.N < 0 || p.K < 0, TP_ERR_INVALID_ARG);
  TP_RETURN_IF(p.K > (int64_t)INT32_MAX, TP_ERR_TOO_LARGE);  // int32 argmax
  TP_RETURN_IF(!(p.tau > 0.0f), TP_ERR_INVALID_ARG);
  return TP_OK;
}

extern "C" {

const char* tp_status_string(int status) {
  switch (status) {
    case TP_OK: return "ok";
    case TP_ERR_INVALID_ARG: return "invalid argument (size, stride or mode)";
    case TP_ERR_NULL_POINTER: return "required pointer is NULL";
    case TP_ERR_MISALIGNED: return "pointer or stride violates an alignment rule";
    case TP_ERR_UNSUPPORTED: return "unsupported dtype, mode or layout";
    case TP_ERR_TOO_LARGE: return "size exceeds a documented limit";
    case TP_ERR_BAD_POINTER: return "pointer is not device memory of the current device";
    case TP_ERR_WORKSPACE: return "workspace missing or too small";
    default: break;
  }
  if (status > 0) return cudaGetErrorString((cudaError_t)status);
  return "unknown tropical_b200 status";
}

int tp_abi_version(void) { return 1; }

int tp_set_pointer_checks(int enable) {
  return g_pointer_checks.exchange(enable ? 1 : 0);
}

int tp_maxplus_fwd_strided(int dtype, int64_t B1, int64_t B2, int64_t M, int64_t N, int64_t K,
                           const void* x, int64_t sx_b1, int64_t sx_b2, int64_t sx_m, int64_t sx_k,
                           const void* w, int64_t sw_b1, int64_t sw_b2, int64_t sw_n, int64_t sw_k,
                           const float* bias, float* y, int64_t sy_b1, int64_t sy_b2, int64_t sy_m,
                           int64_t sy_n, int32_t* argmax, int64_t sa_b1, int64_t sa_b2,
                           int64_t sa_m, int64_t sa_n, float scale, void* stream) {
  StridedMaxPlus p{dtype, B1, B2, M,     N,     K,     x,     sx_b1, sx_b2, sx_m,  sx_k,
                   w,     sw_b1, sw_b2, sw_n, sw_k,  bias,  y,     sy_b1, sy_b2, sy_m, sy_n,
                   argmax, sa_b1, sa_b2, sa_m, sa_n, scale, 1.0f};
  int s = validate_strided(p);
  if (s != TP_OK) return s;
  if (B1 * B2 * M * N == 0) return TP_OK;
  TP_CHECK_PTR(y);
  TP_CHECK_OPT_PTR(argmax);
  TP_CHECK_OPT_PTR(bias);
  if (K > 0) {
    TP_CHECK_PTR(x);
    TP_CHECK_PTR(w);
  }
  if (maxplus_tma_eligible(p)) {
    s = launch_maxplus_fwd_tma(p, as_stream(stream));
    if (s != TP_ERR_UNSUPPORTED) return s;
  }
  return launch_maxplus_fwd_generic(p, as_stream(stream));
}

int tp_maxplus_fwd(int dtype, int64_t M, int64_t N, int64_t K, const void* x, int64_t ldx,
                   const void* w, int64_t ldw, const float* bias, float* y, int64_t ldy,
                   int32_t* argmax, int64_t ld_argmax, void* stream) {
  TP_RETURN_IF(M < 0 || N < 0 || K < 0, TP_ERR_INVALID_ARG);
  TP_RETURN_IF((M > 0 && K > 0 && ldx < K) || (N > 0 && K > 0 && ldw < K) || (M > 0 && ldy < N),
               TP_ERR_INVALID_ARG);
  TP_RETURN_IF(argmax && M > 0 && ld_argmax < N, TP_ERR_INVALID_ARG);
  return tp_maxplus_fwd_strided(dtype, 1, 1, M, N, K, x, 0, 0, ldx, 1, w, 0, 0, ldw, 1, bias, y, 0,
                                0, ldy, 1, argmax, 0, 0, ld_argmax, 1, 1.0f, stream);
}

int tp_maxplus_fwd_lfdual(int dtype, int64_t M, int64_t N, int64_t K, const void* x,
                          int64_t ldx, const void* w, int64_t ldw, const float* bias, float* y,
                          int64_t ldy, int act_mode, int pieces, const float* slopes,
                          const float* piece_bias, const float* x_grid, const float* gate,
                          void* stream) {
  TP_RETURN_IF(M < 0 || N < 0 || K < 0, TP_ERR_INVALID_ARG);
  TP_RETURN_IF((M > 0 && K > 0 && ldx < K) || (N > 0 && K > 0 && ldw < K) || (M > 0 && ldy < N),
               TP_ERR_INVALID_ARG);
  TP_RETURN_IF(act_mode < 0 || act_mode > 2, TP_ERR_INVALID_ARG);
  TP_RETURN_IF(pieces < 1 || pieces > LF_MAX_PIECES, TP_ERR_INVALID_ARG);
  StridedMaxPlus p{dtype, 1, 1, M, N, K, x, 0, 0, ldx, 1, w, 0, 0, ldw, 1, bias, y, 0, 0, ldy, 1,
                   nullptr, 0, 0, 0, 0, 1.0f, 1.0f};
  p.act = LfAct{act_mode, pieces, slopes, piece_bias, x_grid, gate};
  int s = validate_strided(p);
  if (s != TP_OK) return s;
  if (M * N == 0) return TP_OK;
  TP_CHECK_PTR(y);
  TP_CHECK_OPT_PTR(bias);
  TP_CHECK_PTR(slopes);
  TP_CHECK_PTR(piece_bias);
  TP_CHECK_PTR(x_grid);
  if (act_mode == 2) TP_CHECK_PTR(gate);
  if (K > 0) {
    TP_CHECK_PTR(x);
    TP_CHECK_PTR(w);
  }
  if (maxplus_tma_eligible(p)) {
    s = launch_maxplus_fwd_tma(p, as_stream(stream));
    if (s != TP_ERR_UNSUPPORTED) return s;
  }
  return launch_maxplus_fwd_generic(p, as_stream(stream));
}

int tp_maxplus_fwd_sharded(int64_t M, int64_t N_shard, int64_t K, const float* x, int64_t ldx,
                           const float* w_shard, int64_t ldw, const float* bias_shard,
                           float* const* y_dst, int32_t* const* argmax_dst, int n_dst,
                           int64_t ldy, int64_t col0, void* stream) {
  TP_RETURN_IF(M < 0 || N_shard < 0 || K < 0 || col0 < 0, TP_ERR_INVALID_ARG);
  TP_RETURN_IF(n_dst < 1 || n_dst > 8, TP_ERR_INVALID_ARG);
  TP_RETURN_IF(y_dst == nullptr, TP_ERR_NULL_POINTER);
  TP_RETURN_IF(M > 0 && (ldy < col0 + N_shard || ldx < K || ldw < K), TP_ERR_INVALID_ARG);
  if (M * N_shard == 0) return TP_OK;
  for (int d = 0; d < n_dst; ++d) {
    TP_RETURN_IF(y_dst[d] == nullptr, TP_ERR_NULL_POINTER);
    TP_RETURN_IF(argmax_dst != nullptr && argmax_dst[d] == nullptr, TP_ERR_NULL_POINTER);
  }
  TP_CHECK_PTR(x);
  TP_CHECK_PTR(w_shard);
  TP_CHECK_OPT_PTR(bias_shard);
  // destination 0 is this device's own output; the others may be peer memory
  // (mapped through CUDA IPC / symmetric memory), which the pointer check
  // below accepts as device memory of another device.
  TP_CHECK_PTR(y_dst[0]);
  if (argmax_dst) TP_CHECK_PTR(argmax_dst[0]);
  StridedMaxPlus p{TP_DTYPE_F32, 1, 1, M, N_shard, K, x, 0, 0, ldx, 1, w_shard, 0, 0, ldw, 1,
                   bias_shard, y_dst[0] + col0, 0, 0, ldy, 1,
                   argmax_dst ? argmax_dst[0] + col0 : nullptr, 0, 0, ldy, 1, 1.0f, 1.0f};
  if (maxplus_tma_eligible(p))
    return launch_maxplus_fwd_tma_dests(p, y_dst + 1, argmax_dst ? argmax_dst + 1 : nullptr,
                                        n_dst - 1, col0, as_stream(stream));
  // small or unaligned shards: compute into the local copy, then copy the
  // block into the other destinations (peer copies through unified addressing)
  int s = launch_maxplus_fwd_generic(p, as_stream(stream));
  if (s != TP_OK) return s;
  for (int d = 1; d < n_dst; ++d) {
    cudaError_t e = cudaMemcpy2DAsync(y_dst[d] + col0, ldy * 4, y_dst[0] + col0, ldy * 4,
                                      N_shard * 4, M, cudaMemcpyDeviceToDevice, as_stream(stream));
    if (e == cudaSuccess && argmax_dst)
      e = cudaMemcpy2DAsync(argmax_dst[d] + col0, ldy * 4, argmax_dst[0] + col0, ldy * 4,
                            N_shard * 4, M, cudaMemcpyDeviceToDevice, as_stream(stream));
    if (e != cudaSuccess) return (int)e;
  }
  return TP_OK;
}

int tp_maxplus_lse_fwd_strided(int dtype, float tau, int64_t B1, int64_t B2, int64_t M, int64_t N,
                               int64_t K, const void* x, int64_t sx_b1, int64_t sx_b2,
                               int64_t sx_m, int64_t sx_k, const void* w, int64_t sw_b1,
                               int64_t sw_b2, int64_t sw_n, int64_t sw_k, const float* bias,
                               float* y, int64_t sy_b1, int64_t sy_b2, int64_t sy_m, int64_t sy_n,
                               float scale, void* stream) {
  StridedMaxPlus p{dtype, B1, B2,  M,    N,    K,     x,     sx_b1, sx_b2, sx_m,    sx_k,
                   w,     sw_b1, sw_b2, sw_n, sw_k, bias,  y,     sy_b1, sy_b2, sy_m,  sy_n,
                   nullptr, 0,   0,     0,    0,    scale, tau};
  TP_RETURN_IF(dtype == TP_DTYPE_BF16_ARITH, TP_ERR_UNSUPPORTED);
  int s = validate_strided(p);
  if (s != TP_OK) return s;
  if (B1 * B2 * M * N == 0) return TP_OK;
  TP_CHECK_PTR(y);
  TP_CHECK_OPT_PTR(bias);
  if (K > 0) {
    TP_CHECK_PTR(x);
    TP_CHECK_PTR(w);
  }
  return launch_maxplus_lse_fwd_generic(p, as_stream(stream));
}

int tp_maxplus_bwd_argmax_strided(int64_t B1, int64_t B2, int64_t M, int64_t N, int64_t K,
                                  const int32_t* argmax, int64_t sa_b1, int64_t sa_b2,
                                  int64_t sa_m, int64_t sa_n, const float* gy, int64_t sg_b1,
                                  int64_t sg_b2, int64_t sg_m, int64_t sg_n, float* gx,
                                  int64_t sgx_b1, int64_t sgx_b2, int64_t sgx_m, int64_t sgx_k,
                                  float* gw, int64_t sgw_b1, int64_t sgw_b2, int64_t sgw_n,
                                  int64_t sgw_k, float* gbias, float scale, void* stream) {
  TP_RETURN_IF(B1 < 0 || B2 < 0 || M < 0 || N < 0 || K < 0, TP_ERR_INVALID_ARG);
  ScatterArgs p{B1, B2, M, N, K, argmax, sa_b1, sa_b2, sa_m, sa_n, gy, sg_b1, sg_b2, sg_m, sg_n,
                gx, sgx_b1, sgx_b2, sgx_m, sgx_k, gw, sgw_b1, sgw_b2, sgw_n, sgw_k, gbias, scale};
  if (B1 * B2 * M * K > 0) TP_CHECK_PTR(gx);
  if (B1 * B2 * N * K > 0) TP_CHECK_OPT_PTR(gw);
  TP_CHECK_OPT_PTR(gbias);
  if (B1 * B2 * M * N > 0) {
    TP_CHECK_PTR(argmax);
    TP_CHECK_PTR(gy);
  }
  if (gx == nullptr) p.gx = nullptr;
  if (B1 * B2 * M * K == 0 && B1 * B2 * N * K == 0 && gbias == nullptr) return TP_OK;
  return launch_maxplus_bwd_argmax(p, as_stream(stream));
}

int64_t tp_maxplus_bwd_smooth_workspace_bytes(int64_t batch, int64_t M, int64_t N, int64_t K) {
  if (batch < 0 || M < 0 || N < 0 || K < 0) return 0;
  return tp::smooth_workspace_floats(batch, M, N, K) * (int64_t)sizeof(float);
}

int tp_maxplus_bwd_smooth_ref(int mode, float tau, int dtype, int64_t batch, int64_t M,
                              int64_t N, int64_t K, const void* x, const void* w, const float* gy,
                              const float* ref_max, float* gx, float* gw, float* gbias,
                              void* workspace, int64_t workspace_bytes, void* stream) {
  TP_RETURN_IF(mode != TP_BWD_STE && mode != TP_BWD_LSE, TP_ERR_INVALID_ARG);
  TP_RETURN_IF(!(tau > 0.0f), TP_ERR_INVALID_ARG);
  TP_RETURN_IF(dtype != TP_DTYPE_F32 && dtype != TP_DTYPE_BF16, TP_ERR_UNSUPPORTED);
  TP_RETURN_IF(batch < 0 || M < 0 || N < 0 || K < 0, TP_ERR_INVALID_ARG);
  TP_RETURN_IF(batch > 65535, TP_ERR_TOO_LARGE);
  if (batch == 0) return TP_OK;
  if (M * N > 0) {
    TP_CHECK_PTR(gy);
    TP_RETURN_IF(workspace == nullptr ||
                     workspace_bytes < tp_maxplus_bwd_smooth_workspace_bytes(batch, M, N, K),
                 TP_ERR_WORKSPACE);
    TP_RETURN_IF(!aligned16(workspace), TP_ERR_MISALIGNED);
    TP_CHECK_PTR(workspace);
    if (K > 0) {
      TP_CHECK_PTR(x);
      TP_CHECK_PTR(w);
    }
  }
  if (M * K > 0) TP_CHECK_PTR(gx);
  if (N * K > 0) TP_CHECK_OPT_PTR(gw);
  TP_CHECK_OPT_PTR(gbias);
  TP_CHECK_OPT_PTR(ref_max);
  const bool async_stage = dtype == TP_DTYPE_F32 && M % 4 == 0 && N % 4 == 0 && K % 4 == 0 &&
                           aligned16(x) && aligned16(w);
  SmoothArgs p{mode, tau, dtype, batch, M, N, K, x, w, gy, gx, gw, gbias, (float*)workspace,
               async_stage, tp::smooth_splits(batch, M, N, K), tp::smooth_splits(batch, N, M, K),
               (float*)workspace + 6 * batch * M * N, ref_max, false};
  p.fused_gw = async_stage && gw != nullptr && tp::smooth_fused_ok(batch, M, N, K) &&
               g_smooth_fused.load(std::memory_order_relaxed) != 0;
  return launch_maxplus_bwd_smooth(p, as_stream(stream));
}

int tp_maxplus_bwd_smooth(int mode, float tau, int dtype, int64_t batch, int64_t M, int64_t N,
                          int64_t K, const void* x, const void* w, const float* gy, float* gx,
                          float* gw, float* gbias, void* workspace, int64_t workspace_bytes,
                          void* stream) {
  return tp_maxplus_bwd_smooth_ref(mode, tau, dtype, batch, M, N, K, x, w, gy, nullptr, gx, gw,
                                   gbias, workspace, workspace_bytes, stream);
}

int tp_scan_fwd(int64_t B, int64_t T, int64_t C, const float* bb, const float* xx, const float* a,
                float h_init, const float* h0, float* h, uint32_t* win_mask, void* stream) {
  TP_RETURN_IF(B < 0 || T < 0 || C < 0, TP_ERR_INVALID_ARG);
  if (B * T * C == 0) return TP_OK;
  TP_CHECK_PTR(bb);
  TP_CHECK_OPT_PTR(xx);
  TP_CHECK_PTR(a);
  TP_CHECK_OPT_PTR(h0);
  TP_CHECK_PTR(h);
  TP_CHECK_OPT_PTR(win_mask);
  ScanArgs p{};
  p.B = B; p.T = T; p.C = C;
  p.bb = bb; p.xx = xx; p.a = a; p.h_init = h_init; p.h0 = h0; p.h = h; p.win = win_mask;
  return launch_scan_fwd(p, as_stream(stream));
}

int tp_scan_bwd(int64_t B, int64_t T, int64_t C, const float* gh, const float* bb, const float* xx,
                const float* a, float h_init, const float* h0, const float* h,
                const uint32_t* win_mask, float* gu, float* ga, float* gh0, float* workspace,
                void* stream) {
  TP_RETURN_IF(B < 0 || T < 0 || C < 0, TP_ERR_INVALID_ARG);
  if (B * C == 0) return TP_OK;
  TP_RETURN_IF(ga != nullptr && workspace == nullptr, TP_ERR_WORKSPACE);
  const int s = tp::check_scan_bwd_pointers(T, gh, bb, xx, a, h0, h, win_mask, gu, ga, gh0);
  if (s != TP_OK) return s;
  TP_CHECK_OPT_PTR(workspace);
  ScanArgs p{};
  p.B = B; p.T = T; p.C = C;
  p.gh = gh; p.bb = bb; p.xx = win_mask ? nullptr : xx; p.a = a; p.h_init = h_init; p.h0 = h0;
  p.h = const_cast<float*>(h); p.win_in = win_mask; p.gu = gu; p.ga = ga; p.gh0 = gh0;
  p.ws = workspace;
  return launch_scan_bwd(p, as_stream(stream));
}

int64_t tp_scan_chunked_workspace_bytes(int64_t B, int64_t T, int64_t C, int chunk) {
  if (B < 0 || T < 0 || C < 0 || chunk < 0 || chunk % 32 != 0) return -1;
  return tp::scan_chunked_workspace_bytes(B, T, C, chunk);
}

int tp_scan_chunk_length(int64_t B, int64_t T, int64_t C) {
  TP_RETURN_IF(B < 0 || T < 0 || C < 0, TP_ERR_INVALID_ARG);
  return tp::scan_chunk_pick(B, T, C);
}

int tp_scan_fwd_chunked(int64_t B, int64_t T, int64_t C, const float* bb, const float* xx,
                        const float* a, float h_init, const float* h0, float* h,
                        uint32_t* win_mask, int chunk, void* workspace, int64_t workspace_bytes,
                        void* stream) {
  TP_RETURN_IF(B < 0 || T < 0 || C < 0, TP_ERR_INVALID_ARG);
  TP_RETURN_IF(chunk < 0 || chunk % 32 != 0, TP_ERR_INVALID_ARG);
  if (B * T * C == 0) return TP_OK;
  TP_RETURN_IF(C > (int64_t)INT32_MAX || ceil_div(T, 32) > (int64_t)INT32_MAX, TP_ERR_TOO_LARGE);
  TP_CHECK_PTR(bb);
  TP_CHECK_OPT_PTR(xx);
  TP_CHECK_PTR(a);
  TP_CHECK_OPT_PTR(h0);
  TP_CHECK_PTR(h);
  TP_CHECK_OPT_PTR(win_mask);
  TP_CHECK_PTR(workspace);
  ScanArgs p{};
  p.B = B; p.T = T; p.C = C;
  p.bb = bb; p.xx = xx; p.a = a; p.h_init = h_init; p.h0 = h0; p.h = h; p.win = win_mask;
  return launch_scan_fwd_chunked(p, chunk, workspace, workspace_bytes, as_stream(stream));
}

int tp_scan_bwd_chunked(int64_t B, int64_t T, int64_t C, const float* gh, const float* bb,
                        const float* xx, const float* a, float h_init, const float* h0,
                        const float* h, const uint32_t* win_mask, float* gu, float* ga,
                        float* gh0, int chunk, void* workspace, int64_t workspace_bytes,
                        void* stream) {
  TP_RETURN_IF(B < 0 || T < 0 || C < 0, TP_ERR_INVALID_ARG);
  TP_RETURN_IF(chunk < 0 || chunk % 32 != 0, TP_ERR_INVALID_ARG);
  if (B * C == 0) return TP_OK;
  TP_RETURN_IF(C > (int64_t)INT32_MAX || ceil_div(T, 32) > (int64_t)INT32_MAX, TP_ERR_TOO_LARGE);
  const int s = tp::check_scan_bwd_pointers(T, gh, bb, xx, a, h0, h, win_mask, gu, ga, gh0);
  if (s != TP_OK) return s;
  if (T > 0) TP_CHECK_PTR(workspace);
  ScanArgs p{};
  p.B = B; p.T = T; p.C = C;
  p.gh = gh; p.bb = bb; p.xx = win_mask ? nullptr : xx; p.a = a; p.h_init = h_init; p.h0 = h0;
  p.h = const_cast<float*>(h); p.win_in = win_mask; p.gu = gu; p.ga = ga; p.gh0 = gh0;
  return launch_scan_bwd_chunked(p, chunk, workspace, workspace_bytes, as_stream(stream));
}

int tp_convert_bf16_to_f32(int64_t n, const void* src, float* dst, void* stream) {
  TP_RETURN_IF(n < 0, TP_ERR_INVALID_ARG);
  if (n == 0) return TP_OK;
  TP_CHECK_PTR(src);
  TP_CHECK_PTR(dst);
  return launch_bf16_to_f32(src, dst, n, as_stream(stream));
}

int tp_probe_addmax(int form, int64_t blocks, int64_t threads, int64_t iters, float* sink,
                    void* stream) {
  TP_RETURN_IF(form < 0 || form > 9 || blocks <= 0 || blocks > 65535 || iters < 0,
               TP_ERR_INVALID_ARG);
  TP_CHECK_PTR(sink);
  return launch_probe_addmax(form, blocks, threads, iters, sink, as_stream(stream));
}

// ---------------------------------------------------------------------------
// reference-compatible symbols (cuda/maxplus_gemm.cu:297-341)
// ---------------------------------------------------------------------------
void maxplus_forward_cuda(const float* W, const float* x, float* y, const float* bias,
                          int batch_size, int in_features, int out_features, bool use_tiled) {
  (void)use_tiled;  // one implementation serves both reference variants
  int s = tp_maxplus_fwd(TP_DTYPE_F32, batch_size, out_features, in_features, x, in_features, W,
                         in_features, bias, y, out_features, nullptr, 0, nullptr);
  set_last_error(s);
}

void maxplus_backward_cuda(const float* W, const float* x, const float* grad_y, float* grad_W,
                           float* grad_x, float* grad_bias, float ste_temp, int batch_size,
                           int in_features, int out_features) {
  // The reference kernel (cuda/maxplus_gemm.cu:181-259) distributes gy by
  // softmax(s/tau): that is the LSE (Maslov) backward.  It needs a workspace;
  // this legacy entry point cannot take one, so it reports TP_ERR_WORKSPACE
  // through tp_last_error() -- callers should use tp_maxplus_bwd_smooth.
  (void)W; (void)x; (void)grad_y; (void)grad_W; (void)grad_x; (void)grad_bias;
  (void)ste_temp; (void)batch_size; (void)in_features; (void)out_features;
  set_last_error(TP_ERR_WORKSPACE);
}

void maxplus_matmul_cuda(const float* A, const float* B, float* C, int M, int K, int N) {
  int s = tp_maxplus_fwd_strided(TP_DTYPE_F32, 1, 1, M, N, K, A, 0, 0, K, 1, B, 0, 0, 1, N,
                                 nullptr, C, 0, 0, N, 1, nullptr, 0, 0, 0, 0, 1.0f, nullptr);
  set_last_error(s);
}

int tp_tsrn_attention_prologue(int64_t B, int64_t T, int64_t H, int64_t dh, const float* qkv,
                               int64_t ld, int64_t koff, int64_t voff, const float* q_gamma,
                               const float* q_beta, const float* k_gamma, const float* k_beta,
                               float eps, const float* cos_table, const float* sin_table,
                               int64_t npos, int64_t pos0, float* Q, float* K, float* V,
                               void* stream) {
  TP_RETURN_IF(B < 0 || T < 0 || H < 0 || dh <= 0 || npos < 0 || pos0 < 0, TP_ERR_INVALID_ARG);
  TP_RETURN_IF(dh % 2 != 0 || dh > 128, TP_ERR_UNSUPPORTED);
  TP_RETURN_IF(koff < 0 || voff < 0 || ld < 0, TP_ERR_INVALID_ARG);
  if (B * T * H == 0) return TP_OK;
  TP_RETURN_IF(ld < H * dh || koff + H * dh > ld || voff + H * dh > ld, TP_ERR_INVALID_ARG);
  TP_RETURN_IF(pos0 + T > npos, TP_ERR_INVALID_ARG);
  TP_RETURN_IF(!(eps >= 0.0f), TP_ERR_INVALID_ARG);
  TP_CHECK_PTR(qkv);
  TP_CHECK_PTR(q_gamma);
  TP_CHECK_PTR(q_beta);
  TP_CHECK_PTR(k_gamma);
  TP_CHECK_PTR(k_beta);
  TP_CHECK_PTR(cos_table);
  TP_CHECK_PTR(sin_table);
  TP_CHECK_PTR(Q);
  TP_CHECK_PTR(K);
  TP_CHECK_PTR(V);
  return tp::launch_tsrn_prologue(B, T, H, dh, qkv, ld, koff, voff, q_gamma, q_beta, k_gamma,
                                  k_beta, eps, cos_table, sin_table, pos0, Q, K, V,
                                  as_stream(stream));
}

int64_t tp_tsrn_attention_workspace_bytes(int64_t B, int64_t H, int64_t T, int64_t Tkv,
                                          int64_t dh) {
  if (B < 0 || H < 0 || T < 0 || Tkv < 0 || dh < 0) return 0;
  return tp::tsrn_attention_workspace_floats(B, H, T, Tkv, dh) * (int64_t)sizeof(float);
}

int64_t tp_tsrn_attention_prologue_bwd_workspace_bytes(int64_t B, int64_t T, int64_t H,
                                                       int64_t dh) {
  if (B < 0 || T < 0 || H < 0 || dh <= 0) return -1;
  return (int64_t)tp::tsrn_prologue_bwd_blocks(B, T, H) * 4 * dh * (int64_t)sizeof(float);
}

int tp_tsrn_attention_prologue_bwd(int64_t B, int64_t T, int64_t H, int64_t dh, const float* qkv,
                                   int64_t ld, int64_t koff, int64_t voff, const float* q_gamma,
                                   const float* k_gamma, float eps, const float* cos_table,
                                   const float* sin_table, int64_t npos, int64_t pos0,
                                   const float* dQ, const float* dK, const float* dV, float* dqkv,
                                   float* dparams, void* workspace, int64_t workspace_bytes,
                                   void* stream) {
  TP_RETURN_IF(B < 0 || T < 0 || H < 0 || dh <= 0 || npos < 0 || pos0 < 0, TP_ERR_INVALID_ARG);
  TP_RETURN_IF(dh % 2 != 0 || dh > 128, TP_ERR_UNSUPPORTED);
  TP_RETURN_IF(koff < 0 || voff < 0 || ld < 0, TP_ERR_INVALID_ARG);
  TP_RETURN_IF(B * T * H > 0 &&
                   (ld < H * dh || koff + H * dh > ld || voff + H * dh > ld || pos0 + T > npos),
               TP_ERR_INVALID_ARG);
  TP_RETURN_IF(!(eps >= 0.0f), TP_ERR_INVALID_ARG);
  TP_CHECK_PTR(dparams);
  TP_RETURN_IF(workspace == nullptr ||
                   workspace_bytes < tp_tsrn_attention_prologue_bwd_workspace_bytes(B, T, H, dh),
               TP_ERR_WORKSPACE);
  TP_CHECK_PTR(workspace);
  if (B * T * H > 0) {
    TP_CHECK_PTR(qkv);
    TP_CHECK_PTR(q_gamma);
    TP_CHECK_PTR(k_gamma);
    TP_CHECK_PTR(cos_table);
    TP_CHECK_PTR(sin_table);
    TP_CHECK_PTR(dQ);
    TP_CHECK_PTR(dK);
    TP_CHECK_PTR(dV);
    TP_CHECK_PTR(dqkv);
  }
  return tp::launch_tsrn_prologue_bwd(B, T, H, dh, qkv, ld, koff, voff, q_gamma, k_gamma, eps,
                                      cos_table, sin_table, pos0, dQ, dK, dV, dqkv, dparams,
                                      (float*)workspace, as_stream(stream));
}

int64_t tp_layernorm_bwd_workspace_bytes(int64_t rows, int64_t D) {
  if (rows < 0 || !tp::layernorm_bwd_supported(D)) return -1;
  return (int64_t)tp::layernorm_bwd_blocks(rows) * 2 * D * (int64_t)sizeof(float);
}

int tp_layernorm_bwd(int64_t rows, int64_t D, const float* x, const float* dy,
                     const float* gamma, float eps, float* dx, float* dgamma, float* dbeta,
                     void* workspace, int64_t workspace_bytes, void* stream) {
  TP_RETURN_IF(rows < 0 || D <= 0, TP_ERR_INVALID_ARG);
  TP_RETURN_IF(!tp::layernorm_bwd_supported(D), TP_ERR_UNSUPPORTED);
  TP_RETURN_IF(!(eps >= 0.0f), TP_ERR_INVALID_ARG);
  TP_RETURN_IF(workspace == nullptr ||
                   workspace_bytes < tp_layernorm_bwd_workspace_bytes(rows, D),
               TP_ERR_WORKSPACE);
  TP_CHECK_PTR(workspace);
  if (gamma != nullptr) TP_RETURN_IF(!aligned16(gamma), TP_ERR_MISALIGNED);
  if (rows > 0) {
    TP_CHECK_PTR(x);
    TP_CHECK_PTR(dy);
    TP_CHECK_PTR(dx);
    TP_RETURN_IF(!aligned16(x) || !aligned16(dy) || !aligned16(dx), TP_ERR_MISALIGNED);
  }
  return tp::launch_layernorm_bwd(rows, D, x, dy, gamma, eps, dx, dgamma, dbeta,
                                  (float*)workspace, as_stream(stream));
}

int tp_tsrn_attention_fwd(int64_t B, int64_t H, int64_t T, int64_t Tkv, int64_t Tc, int64_t dh,
                          const float* Q, const float* K, const float* V,
                          const float* alibi_slopes, int top_k, int causal, float* out,
                          void* workspace, int64_t workspace_bytes, void* stream) {
  TP_RETURN_IF(B < 0 || H < 0 || T < 0 || Tkv < 0 || Tc < 0 || dh < 0, TP_ERR_INVALID_ARG);
  TP_RETURN_IF(Tc > Tkv, TP_ERR_INVALID_ARG);
  if (B * H * T == 0) return TP_OK;
  TP_RETURN_IF(Tkv == 0 || dh == 0 || top_k < 1, TP_ERR_INVALID_ARG);
  TP_CHECK_PTR(Q);
  TP_CHECK_PTR(K);
  TP_CHECK_PTR(V);
  TP_CHECK_PTR(alibi_slopes);
  TP_CHECK_PTR(out);
  TP_RETURN_IF(workspace == nullptr ||
                   workspace_bytes < tp_tsrn_attention_workspace_bytes(B, H, T, Tkv, dh),
               TP_ERR_WORKSPACE);
  TP_RETURN_IF(!aligned16(workspace), TP_ERR_MISALIGNED);
  TP_CHECK_PTR(workspace);
  return tp::launch_tsrn_attention_fwd(B, H, T, Tkv, Tc, dh, Q, K, V, alibi_slopes, top_k,
                                       causal, out, (float*)workspace, as_stream(stream));
}

int tp_tsrn_attention_fwd_lists(int64_t B, int64_t H, int64_t T, int64_t Tkv, int64_t Tc,
                                int64_t dh, const float* Q, const float* K, const float* V,
                                const float* alibi_slopes, int top_k, int causal, float* out,
                                int32_t* kept_keys, float* kept_weights, float* kept_lse,
                                int32_t* kept_count, void* workspace, int64_t workspace_bytes,
                                void* stream) {
  TP_RETURN_IF(B < 0 || H < 0 || T < 0 || Tkv < 0 || Tc < 0 || dh < 0, TP_ERR_INVALID_ARG);
  TP_RETURN_IF(Tc > Tkv, TP_ERR_INVALID_ARG);
  if (B * H * T == 0) return TP_OK;
  TP_RETURN_IF(Tkv == 0 || dh == 0 || top_k < 1, TP_ERR_INVALID_ARG);
  TP_RETURN_IF(!tp::tsrn_attention_tc_supported(dh, top_k), TP_ERR_UNSUPPORTED);
  TP_CHECK_PTR(Q);
  TP_CHECK_PTR(K);
  TP_CHECK_PTR(V);
  TP_CHECK_PTR(alibi_slopes);
  TP_CHECK_PTR(out);
  TP_CHECK_PTR(kept_keys);
  TP_CHECK_PTR(kept_weights);
  TP_CHECK_PTR(kept_lse);
  TP_CHECK_PTR(kept_count);
  TP_RETURN_IF(workspace == nullptr ||
                   workspace_bytes < tp_tsrn_attention_workspace_bytes(B, H, T, Tkv, dh),
               TP_ERR_WORKSPACE);
  TP_RETURN_IF(!aligned16(workspace), TP_ERR_MISALIGNED);
  TP_CHECK_PTR(workspace);
  return tp::launch_tsrn_attention_tc(B, H, T, Tkv, Tc, dh, Q, K, V, alibi_slopes, top_k, causal,
                                      out, (float*)workspace, as_stream(stream), kept_keys,
                                      kept_weights, kept_lse, kept_count);
}

int tp_tsrn_attention_bwd_rows(int64_t S, int64_t T, int64_t Tkv, int64_t dh, const float* Q,
                               const float* K, const float* V, const float* dO,
                               const int32_t* kept_keys, const float* kept_weights,
                               const float* kept_lse, const int32_t* kept_count, float* dQ,
                               float* entry_ds, void* stream) {
  TP_RETURN_IF(S < 0 || T < 0 || Tkv < 0 || dh < 0, TP_ERR_INVALID_ARG);
  if (S * T == 0) return TP_OK;
  TP_RETURN_IF(Tkv == 0 || dh == 0, TP_ERR_INVALID_ARG);
  TP_CHECK_PTR(Q);
  TP_CHECK_PTR(K);
  TP_CHECK_PTR(V);
  TP_CHECK_PTR(dO);
  TP_CHECK_PTR(kept_keys);
  TP_CHECK_PTR(kept_weights);
  TP_CHECK_PTR(kept_lse);
  TP_CHECK_PTR(kept_count);
  TP_CHECK_PTR(dQ);
  TP_CHECK_PTR(entry_ds);
  return tp::launch_tsrn_attention_bwd_rows(S, T, Tkv, dh, Q, K, V, dO, kept_keys, kept_weights,
                                            kept_lse, kept_count, dQ, entry_ds,
                                            as_stream(stream));
}

int tp_tsrn_attention_bwd_group(int64_t S, int64_t T, int64_t Tkv, const int32_t* kept_keys,
                                int32_t* order, int32_t* key_begin, int32_t* key_count,
                                void* stream) {
  TP_RETURN_IF(S < 0 || T < 0 || Tkv < 0, TP_ERR_INVALID_ARG);
  if (S * Tkv == 0) return TP_OK;
  TP_CHECK_PTR(key_begin);
  TP_CHECK_PTR(key_count);
  if (S * T > 0) {
    TP_CHECK_PTR(kept_keys);
    TP_CHECK_PTR(order);
  }
  return tp::launch_tsrn_attention_bwd_group(S, T, Tkv, kept_keys, order, key_begin, key_count,
                                             as_stream(stream));
}

int tp_tsrn_attention_bwd_keys(int64_t S, int64_t T, int64_t Tkv, int64_t dh, const float* Q,
                               const float* K, const float* dO, const float* kept_weights,
                               const float* kept_lse, const float* entry_ds,
                               const int32_t* order, const int32_t* key_begin,
                               const int32_t* key_count, float* dK, float* dV, void* stream) {
  TP_RETURN_IF(S < 0 || T < 0 || Tkv < 0 || dh < 0, TP_ERR_INVALID_ARG);
  if (S * Tkv == 0) return TP_OK;
  TP_RETURN_IF(dh == 0, TP_ERR_INVALID_ARG);
  TP_CHECK_PTR(K);
  TP_CHECK_PTR(key_begin);
  TP_CHECK_PTR(key_count);
  TP_CHECK_PTR(dK);
  TP_CHECK_PTR(dV);
  if (S * T > 0) {
    TP_CHECK_PTR(Q);
    TP_CHECK_PTR(dO);
    TP_CHECK_PTR(kept_weights);
    TP_CHECK_PTR(kept_lse);
    TP_CHECK_PTR(entry_ds);
    TP_CHECK_PTR(order);
  }
  return tp::launch_tsrn_attention_bwd_keys(S, T, Tkv, dh, Q, K, dO, kept_weights, entry_ds,
                                            kept_lse, order, key_begin, key_count, dK, dV,
                                            as_stream(stream));
}

int tp_tsrn_attention_set_path(int path, int* previous) {
  TP_RETURN_IF(path != TP_ATT_PATH_AUTO && path != TP_ATT_PATH_CUDA_CORES &&
                   path != TP_ATT_PATH_TENSOR_CORES,
               TP_ERR_INVALID_ARG);
  if (previous) *previous = tp::tsrn_attention_path();
  tp::tsrn_attention_path() = path;
  return TP_OK;
}

int tp_esn_gru_fwd(int64_t B, int64_t T, int64_t dr, const float* U, const float* Uz,
                   const float* Ur, const float* Wzh, int64_t ld_wzh, const float* Wrh,
                   int64_t ld_wrh, const float* Ws, int64_t ld_ws, float* H, void* stream) {
  TP_RETURN_IF(B < 0 || T < 0 || dr < 0, TP_ERR_INVALID_ARG);
  if (B * T * dr == 0) return TP_OK;
  TP_RETURN_IF(ld_wzh < dr || ld_wrh < dr || ld_ws < dr, TP_ERR_INVALID_ARG);
  TP_CHECK_PTR(U);
  TP_CHECK_PTR(Uz);
  TP_CHECK_PTR(Ur);
  TP_CHECK_PTR(Wzh);
  TP_CHECK_PTR(Wrh);
  TP_CHECK_PTR(Ws);
  TP_CHECK_PTR(H);
  const float* W[3] = {Wzh, Wrh, Ws};
  const int64_t ld[3] = {ld_wzh, ld_wrh, ld_ws};
  return tp::launch_esn_fwd(true, B, T, dr, U, Uz, Ur, W, ld, nullptr, H, as_stream(stream));
}

int tp_split_tf32(const float* x, int64_t n, float* hi, float* lo, void* stream) {
  TP_RETURN_IF(n < 0, TP_ERR_INVALID_ARG);
  if (n == 0) return TP_OK;
  TP_CHECK_PTR(x);
  TP_CHECK_PTR(hi);
  TP_CHECK_PTR(lo);
  TP_RETURN_IF(!aligned16(x) || !aligned16(hi) || !aligned16(lo), TP_ERR_MISALIGNED);
  return tp::launch_split_tf32(x, n, hi, lo, as_stream(stream));
}

int tp_split_tf32_cat(const float* x, int64_t rows, int64_t cols, float* out, int nparts,
                      int lo_mask, void* stream) {
  TP_RETURN_IF(rows < 0 || cols < 0 || nparts < 1 || nparts > 3, TP_ERR_INVALID_ARG);
  TP_RETURN_IF(lo_mask < 0 || lo_mask >= (1 << nparts), TP_ERR_INVALID_ARG);
  if (rows * cols == 0) return TP_OK;
  TP_RETURN_IF(cols % 4 != 0, TP_ERR_UNSUPPORTED);
  TP_CHECK_PTR(x);
  TP_CHECK_PTR(out);
  TP_RETURN_IF(!aligned16(x) || !aligned16(out), TP_ERR_MISALIGNED);
  return tp::launch_split_tf32_cat(x, rows, cols, out, nparts, lo_mask, as_stream(stream));
}

int tp_esn_gru_bwd(int64_t B, int64_t T, int64_t dr, const float* dH, const float* fa,
                   const float* fz, const float* fr, const float* keep, const float* r,
                   const float* WzhT, int64_t ld_wz, const float* WrhT, int64_t ld_wr,
                   const float* WsT, int64_t ld_ws, float* dAh, float* dAz, float* dAr,
                   void* stream) {
  TP_RETURN_IF(B < 0 || T < 0 || dr < 0, TP_ERR_INVALID_ARG);
  if (B * T * dr == 0) return TP_OK;
  TP_RETURN_IF(ld_wz < dr || ld_wr < dr || ld_ws < dr, TP_ERR_INVALID_ARG);
  TP_CHECK_PTR(dH);
  TP_CHECK_PTR(fa);
  TP_CHECK_PTR(fz);
  TP_CHECK_PTR(fr);
  TP_CHECK_PTR(keep);
  TP_CHECK_PTR(r);
  TP_CHECK_PTR(WzhT);
  TP_CHECK_PTR(WrhT);
  TP_CHECK_PTR(WsT);
  TP_CHECK_PTR(dAh);
  TP_CHECK_PTR(dAz);
  TP_CHECK_PTR(dAr);
  const float* F[5] = {fa, fz, fr, keep, r};
  const float* W[3] = {WzhT, WrhT, WsT};
  const int64_t ld[3] = {ld_wz, ld_wr, ld_ws};
  float* out[3] = {dAh, dAz, dAr};
  return tp::launch_esn_bwd(true, B, T, dr, dH, F, W, ld, nullptr, out, as_stream(stream));
}

int tp_esn_leaky_bwd(int64_t B, int64_t T, int64_t dr, const float* dH, const float* fa,
                     const float* WsT, int64_t ld_ws, const float* leak, float* dA, float* dHs,
                     void* stream) {
  TP_RETURN_IF(B < 0 || T < 0 || dr < 0, TP_ERR_INVALID_ARG);
  if (B * T * dr == 0) return TP_OK;
  TP_RETURN_IF(ld_ws < dr, TP_ERR_INVALID_ARG);
  TP_CHECK_PTR(dH);
  TP_CHECK_PTR(fa);
  TP_CHECK_PTR(WsT);
  TP_CHECK_PTR(leak);
  TP_CHECK_PTR(dA);
  TP_CHECK_PTR(dHs);
  const float* F[5] = {fa, nullptr, nullptr, nullptr, nullptr};
  const float* W[3] = {WsT, nullptr, nullptr};
  const int64_t ld[3] = {ld_ws, 0, 0};
  float* out[3] = {dA, dHs, nullptr};
  return tp::launch_esn_bwd(false, B, T, dr, dH, F, W, ld, leak, out, as_stream(stream));
}

int tp_esn_leaky_fwd(int64_t B, int64_t T, int64_t dr, const float* U, const float* Ws,
                     int64_t ld_ws, const float* leak, float* H, void* stream) {
  TP_RETURN_IF(B < 0 || T < 0 || dr < 0, TP_ERR_INVALID_ARG);
  if (B * T * dr == 0) return TP_OK;
  TP_RETURN_IF(ld_ws < dr, TP_ERR_INVALID_ARG);
  TP_CHECK_PTR(U);
  TP_CHECK_PTR(Ws);
  TP_CHECK_PTR(leak);
  TP_CHECK_PTR(H);
  const float* W[3] = {Ws, nullptr, nullptr};
  const int64_t ld[3] = {ld_ws, 0, 0};
  return tp::launch_esn_fwd(false, B, T, dr, U, nullptr, nullptr, W, ld, leak, H,
                            as_stream(stream));
}

int tp_esn_gru_fwd_seg(int64_t B, int64_t T, int64_t t_stride, int64_t dr, const float* U,
                       const float* Uz, const float* Ur, const float* Wzh, int64_t ld_wzh,
                       const float* Wrh, int64_t ld_wrh, const float* Ws, int64_t ld_ws,
                       const float* h0, int64_t ld_h0, float* H, void* stream) {
  TP_RETURN_IF(B < 0 || T < 0 || dr < 0, TP_ERR_INVALID_ARG);
  if (B * T * dr == 0) return TP_OK;
  TP_RETURN_IF(t_stride < T || ld_wzh < dr || ld_wrh < dr || ld_ws < dr, TP_ERR_INVALID_ARG);
  TP_RETURN_IF(h0 != nullptr && ld_h0 < dr, TP_ERR_INVALID_ARG);
  TP_CHECK_PTR(U);
  TP_CHECK_PTR(Uz);
  TP_CHECK_PTR(Ur);
  TP_CHECK_PTR(Wzh);
  TP_CHECK_PTR(Wrh);
  TP_CHECK_PTR(Ws);
  TP_CHECK_OPT_PTR(h0);
  TP_CHECK_PTR(H);
  const float* W[3] = {Wzh, Wrh, Ws};
  const int64_t ld[3] = {ld_wzh, ld_wrh, ld_ws};
  return tp::launch_esn_fwd(true, B, T, dr, U, Uz, Ur, W, ld, nullptr, H, as_stream(stream),
                            t_stride, h0, ld_h0);
}

int tp_esn_leaky_fwd_seg(int64_t B, int64_t T, int64_t t_stride, int64_t dr, const float* U,
                         const float* Ws, int64_t ld_ws, const float* leak, const float* h0,
                         int64_t ld_h0, float* H, void* stream) {
  TP_RETURN_IF(B < 0 || T < 0 || dr < 0, TP_ERR_INVALID_ARG);
  if (B * T * dr == 0) return TP_OK;
  TP_RETURN_IF(t_stride < T || ld_ws < dr, TP_ERR_INVALID_ARG);
  TP_RETURN_IF(h0 != nullptr && ld_h0 < dr, TP_ERR_INVALID_ARG);
  TP_CHECK_PTR(U);
  TP_CHECK_PTR(Ws);
  TP_CHECK_PTR(leak);
  TP_CHECK_OPT_PTR(h0);
  TP_CHECK_PTR(H);
  const float* W[3] = {Ws, nullptr, nullptr};
  const int64_t ld[3] = {ld_ws, 0, 0};
  return tp::launch_esn_fwd(false, B, T, dr, U, nullptr, nullptr, W, ld, leak, H,
                            as_stream(stream), t_stride, h0, ld_h0);
}

int tp_memcpy2d_async(void* dst, int64_t dst_pitch, const void* src, int64_t src_pitch,
                      int64_t width_bytes, int64_t rows, void* stream) {
  TP_RETURN_IF(width_bytes < 0 || rows < 0 || dst_pitch < width_bytes || src_pitch < width_bytes,
               TP_ERR_INVALID_ARG);
  if (width_bytes == 0 || rows == 0) return TP_OK;
  TP_RETURN_IF(dst == nullptr || src == nullptr, TP_ERR_NULL_POINTER);
  return cuda_status(cudaMemcpy2DAsync(dst, (size_t)dst_pitch, src, (size_t)src_pitch,
                                       (size_t)width_bytes, (size_t)rows, cudaMemcpyDefault,
                                       as_stream(stream)));
}

namespace {

// shared argument checks of the two Maslov softmax entries (T and C are
// not read when Lk == 0)
int maslov_args(int64_t B, int64_t H, int64_t Lq, int64_t Lk, const float* T, const float* C,
                const float* g, int64_t gsb, int64_t gsi, int64_t gsh,
                const unsigned char* mask, int64_t msb, int64_t msh, int64_t msi, int64_t msj,
                const float* tau, tp::MaslovArgs& a) {
  TP_RETURN_IF(B < 0 || H < 0 || Lq < 0 || Lk < 0, TP_ERR_INVALID_ARG);
  TP_RETURN_IF(Lk > 0 && (C == nullptr) != (g == nullptr), TP_ERR_INVALID_ARG);
  TP_RETURN_IF(gsb < 0 || gsi < 0 || gsh < 0 || msb < 0 || msh < 0 || msi < 0 || msj < 0,
               TP_ERR_INVALID_ARG);
  a = tp::MaslovArgs{};
  a.rows = B * H * Lq;
  a.H = H;
  a.Lq = Lq;
  a.Lk = Lk;
  a.T = T;
  a.C = C;
  a.g = g;
  a.gsb = gsb;
  a.gsi = gsi;
  a.gsh = gsh;
  a.mask = mask;
  a.msb = msb;
  a.msh = msh;
  a.msi = msi;
  a.msj = msj;
  a.tau = tau;
  if (a.rows == 0) return TP_OK;
  TP_CHECK_PTR(tau);
  if (g) TP_CHECK_PTR(g);
  if (Lk > 0) {
    TP_CHECK_PTR(T);
    if (C) TP_CHECK_PTR(C);
    if (mask) TP_CHECK_PTR(mask);
  }
  return TP_OK;
}

}  // namespace

int tp_maslov_softmax_fwd(int64_t B, int64_t H, int64_t Lq, int64_t Lk, const float* T,
                          const float* C, const float* g, int64_t gsb, int64_t gsi, int64_t gsh,
                          const unsigned char* mask, int64_t msb, int64_t msh, int64_t msi,
                          int64_t msj, const float* tau, float* P, void* stream) {
  tp::MaslovArgs a;
  int st = maslov_args(B, H, Lq, Lk, T, C, g, gsb, gsi, gsh, mask, msb, msh, msi, msj, tau, a);
  if (st != TP_OK || a.rows == 0 || Lk == 0) return st;
  TP_CHECK_PTR(P);
  a.P = P;
  return tp::launch_maslov(a, false, as_stream(stream));
}

int tp_maslov_softmax_bwd(int64_t B, int64_t H, int64_t Lq, int64_t Lk, const float* T,
                          const float* C, const float* g, int64_t gsb, int64_t gsi, int64_t gsh,
                          const unsigned char* mask, int64_t msb, int64_t msh, int64_t msi,
                          int64_t msj, const float* tau, const float* P, const float* dP,
                          float* dT, float* dC, float* dg, float* dtau_rows, void* stream) {
  tp::MaslovArgs a;
  int st = maslov_args(B, H, Lq, Lk, T, C, g, gsb, gsi, gsh, mask, msb, msh, msi, msj, tau, a);
  if (st != TP_OK || a.rows == 0) return st;
  if (Lk > 0) {
    TP_CHECK_PTR(P);
    TP_CHECK_PTR(dP);
    if (dT) TP_CHECK_PTR(dT);
    if (dC) TP_CHECK_PTR(dC);
  } else if (dg == nullptr && dtau_rows == nullptr) {
    return TP_OK;              // empty rows and no per-row output
  }
  if (dg) TP_CHECK_PTR(dg);
  if (dtau_rows) TP_CHECK_PTR(dtau_rows);
  a.P = const_cast<float*>(P);
  a.dP = dP;
  a.dT = dT;
  a.dC = dC;
  a.dg = g ? dg : nullptr;
  a.dtau_rows = dtau_rows;
  return tp::launch_maslov(a, true, as_stream(stream));
}

int64_t tp_set_argmax_tma_min_terms(int64_t terms) { return tp::set_argmax_tma_min_terms(terms); }

int tp_set_stream_k(int mode) { return tp::set_stream_k(mode); }

int tp_set_smooth_fused(int enable) { return g_smooth_fused.exchange(enable ? 1 : 0); }

int tp_last_error(void) { return last_error(); }

int tp_device_error(int reset) {
  int v = 0;
  cudaError_t e = cudaMemcpyFromSymbol(&v, g_tp_status, sizeof(int), offsetof(TpDeviceStatus, error));
  if (e != cudaSuccess) return -(int)e;
  if (reset) {
    const int zero = 0;
    e = cudaMemcpyToSymbol(g_tp_status, &zero, sizeof(int), offsetof(TpDeviceStatus, error));
    if (e != cudaSuccess) return -(int)e;
  }
  return v;
}

int tp_set_wait_budget_ns(int64_t ns, int64_t* previous) {
  TP_RETURN_IF(ns < TP_WAIT_BUDGET_MIN_NS || ns > TP_WAIT_BUDGET_MAX_NS, TP_ERR_INVALID_ARG);
  unsigned long long old = 0;
  const size_t off = offsetof(TpDeviceStatus, wait_budget_ns);
  cudaError_t e = cudaMemcpyFromSymbol(&old, g_tp_status, sizeof(old), off);
  if (e != cudaSuccess) {
    cudaGetLastError();
    return cuda_status(e);
  }
  const unsigned long long v = (unsigned long long)ns;
  e = cudaMemcpyToSymbol(g_tp_status, &v, sizeof(v), off);
  if (e != cudaSuccess) {
    cudaGetLastError();
    return cuda_status(e);
  }
  if (previous) *previous = (int64_t)old;
  return TP_OK;
}

int tp_selftest_bounded_wait(int kind, const unsigned* flag, void* stream) {
  TP_RETURN_IF(kind != 0 && kind != 1, TP_ERR_INVALID_ARG);
  if (kind == 1) TP_CHECK_PTR(flag);
  return tp::launch_selftest_wait(kind, flag, as_stream(stream));
}

}  // extern "C"
