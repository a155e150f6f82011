// scan.cu -- tropical (max-plus) diagonal SSM scan, forward and argmax-path
// backward (research/tsrn_dml.py:917-980, TropicalSSM; definition of the
// recurrence in the comment block at research/tsrn_dml.py:906-916).
//
//   h[b,t,c] = max(a[c] + h[b,t-1,c], u[b,t,c]),   u = bb + xx,
//   h[b,-1,c] = h0[b,c] or h_init.
//
// The reference evaluates this through a closed form, t*A + cummax(u - t*A)
// (research/tsrn_dml.py:961-972), whose rounding differs from the recurrence
// by up to ~T*ulp.  These kernels evaluate the recurrence itself, one rounded
// add and one exact max per step, so they are bit-exact with the sequential
// oracle.  The input wins ties (u >= a + h_prev), which is the last-index
// rule of torch.cummax that routes the reference's gradient.
//
// Layout: [B,T,C] contiguous, C fastest.  One warp owns 32 consecutive
// channels of one batch row and walks T sequentially; lane c of the warp
// reads element c of each 128-byte row, so every global access of the warp
// is one full, coalesced line.  Tiles of 32 timesteps x 32 channels are
// staged by TMA into a ring of shared-memory stages (mbarrier per stage) so
// that each warp keeps several KB of loads in flight -- the kernel is bound
// by HBM bandwidth, not by the dependency chain (~12 cycles/step/warp).
#include <mutex>

#include "maxplus_internal.cuh"

namespace tp {

namespace {

constexpr int TS = 32;  // timesteps per TMA box (= bits per win-mask word)
constexpr int BOX_BYTES = TS * 32 * 4;

bool make_scan_map(CUtensorMap* map, const float* base, int64_t rows, int64_t C) {
  EncodeTiledFn enc = encode_tiled();
  if (!enc) return false;
  cuuint64_t dims[2] = {(cuuint64_t)C, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)C * 4};
  cuuint32_t box[2] = {32, TS};
  cuuint32_t estr[2] = {1, 1};
  return enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, (void*)base, dims, strides, box, estr,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
             CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// ---------------------------------------------------------------------------
// forward, TMA-staged
// ---------------------------------------------------------------------------
template <bool kHasX, bool kMask, int STAGES>
__global__ void __launch_bounds__(32)
    scan_fwd_tma_kernel(const __grid_constant__ CUtensorMap bmap,
                        const __grid_constant__ CUtensorMap xmap, const ScanArgs p, int cgroups) {
  constexpr int NBOX = kHasX ? 2 : 1;
  __shared__ __align__(128) float buf[STAGES][NBOX][TS][32];
  __shared__ __align__(8) uint64_t full[STAGES];
  const int lane = threadIdx.x;
  const int64_t b = blockIdx.x / cgroups;
  const int64_t c0 = (int64_t)(blockIdx.x % cgroups) * 32;
  const int64_t c = c0 + lane;
  const bool cv = c < p.C;
  const int nchunks = (int)ceil_div(p.T, TS);
  const float a = cv ? p.a[c] : 0.0f;
  float h = (p.h0 && cv) ? p.h0[b * p.C + c] : p.h_init;
  const int64_t row0 = b * p.T;

  if (lane == 0) {
    for (int s = 0; s < STAGES; ++s) tp_mbar_init(&full[s], 1);
    tp_fence_mbar_init();
    for (int s = 0; s < STAGES && s < nchunks; ++s) {
      tp_mbar_arrive_expect_tx(&full[s], NBOX * BOX_BYTES);
      tp_tma_load_2d(&buf[s][0][0][0], &bmap, (int32_t)c0, (int32_t)(row0 + s * TS), &full[s]);
      if (kHasX)
        tp_tma_load_2d(&buf[s][NBOX - 1][0][0], &xmap, (int32_t)c0, (int32_t)(row0 + s * TS),
                       &full[s]);
    }
  }
  __syncwarp();

  for (int ch = 0; ch < nchunks; ++ch) {
    const int s = ch % STAGES;
    if (!tp_mbar_wait(&full[s], (uint32_t)((ch / STAGES) & 1), p.err)) return;
    const int64_t t0 = (int64_t)ch * TS;
    const int rows = (int)((p.T - t0) < TS ? (p.T - t0) : TS);
    // 1) the chunk's inputs into registers (independent loads), 2) hand the
    // stage back to the TMA right away, 3) run the recurrence on registers
    float u[TS];
#pragma unroll
    for (int r = 0; r < TS; ++r) {
      u[r] = buf[s][0][r][lane];
      if (kHasX) u[r] = u[r] + buf[s][NBOX - 1][r][lane];
    }
    __syncwarp();
    if (lane == 0 && ch + STAGES < nchunks) {
      const int64_t nr = row0 + (int64_t)(ch + STAGES) * TS;
      tp_mbar_arrive_expect_tx(&full[s], NBOX * BOX_BYTES);
      tp_tma_load_2d(&buf[s][0][0][0], &bmap, (int32_t)c0, (int32_t)nr, &full[s]);
      if (kHasX) tp_tma_load_2d(&buf[s][NBOX - 1][0][0], &xmap, (int32_t)c0, (int32_t)nr, &full[s]);
    }
    uint32_t bits = 0;
    float* hout = p.h + (row0 + t0) * p.C + c;
    if (rows == TS && cv) {
#pragma unroll
      for (int r = 0; r < TS; ++r) {
        const float d = a + h;
        const bool win = u[r] >= d;
        h = win ? u[r] : d;
        bits |= (uint32_t)win << r;
        hout[(int64_t)r * p.C] = h;
      }
    } else {
#pragma unroll
      for (int r = 0; r < TS; ++r) {
        if (r < rows) {
          const float d = a + h;
          const bool win = u[r] >= d;
          h = win ? u[r] : d;
          bits |= (uint32_t)win << r;
          if (cv) hout[(int64_t)r * p.C] = h;
        }
      }
    }
    if (kMask && cv) p.win[(b * nchunks + ch) * p.C + c] = bits;
  }
}

// ---------------------------------------------------------------------------
// backward, TMA-staged.  kMask: winners from the forward's mask (reads gh and
// the mask only); otherwise recomputed from (bb, xx, h) with h read one step
// behind (the h box of chunk ch starts at row t0 - 1).
// ---------------------------------------------------------------------------
template <bool kMask, bool kHasX, int STAGES>
__global__ void __launch_bounds__(32)
    scan_bwd_tma_kernel(const __grid_constant__ CUtensorMap gmap,
                        const __grid_constant__ CUtensorMap bmap,
                        const __grid_constant__ CUtensorMap xmap,
                        const __grid_constant__ CUtensorMap hmap, const ScanArgs p, int cgroups) {
  constexpr int NBOX = kMask ? 1 : (kHasX ? 4 : 3);  // g [, b, h [, x]]
  __shared__ __align__(128) float buf[STAGES][NBOX][TS][32];
  __shared__ __align__(8) uint64_t full[STAGES];
  const int lane = threadIdx.x;
  const int64_t b = blockIdx.x / cgroups;
  const int64_t c0 = (int64_t)(blockIdx.x % cgroups) * 32;
  const int64_t c = c0 + lane;
  const bool cv = c < p.C;
  const int nchunks = (int)ceil_div(p.T, TS);
  const float a = cv ? p.a[c] : 0.0f;
  const float hm1 = (p.h0 && cv) ? p.h0[b * p.C + c] : p.h_init;
  const int64_t row0 = b * p.T;

  auto issue = [&](int slot, int chunk) {
    const int32_t r = (int32_t)(row0 + (int64_t)chunk * TS);
    tp_mbar_arrive_expect_tx(&full[slot], NBOX * BOX_BYTES);
    tp_tma_load_2d(&buf[slot][0][0][0], &gmap, (int32_t)c0, r, &full[slot]);
    if (!kMask) {
      tp_tma_load_2d(&buf[slot][1][0][0], &bmap, (int32_t)c0, r, &full[slot]);
      tp_tma_load_2d(&buf[slot][2][0][0], &hmap, (int32_t)c0, r - 1, &full[slot]);
      if (kHasX) tp_tma_load_2d(&buf[slot][3][0][0], &xmap, (int32_t)c0, r, &full[slot]);
    }
  };

  if (lane == 0) {
    for (int s = 0; s < STAGES; ++s) tp_mbar_init(&full[s], 1);
    tp_fence_mbar_init();
    for (int s = 0; s < STAGES && s < nchunks; ++s) issue(s, nchunks - 1 - s);
  }
  __syncwarp();

  float carry = 0.0f;  // gradient flowing into h[t] from h[t+1]
  float ga = 0.0f;
  for (int i = 0; i < nchunks; ++i) {
    const int ch = nchunks - 1 - i;
    const int s = i % STAGES;
    if (!tp_mbar_wait(&full[s], (uint32_t)((i / STAGES) & 1), p.err)) return;
    const int64_t t0 = (int64_t)ch * TS;
    const int rows = (int)((p.T - t0) < TS ? (p.T - t0) : TS);
    uint32_t bits = 0;
    if (kMask && cv) bits = p.win_in[(b * nchunks + ch) * p.C + c];
    float* gout = p.gu + (row0 + t0) * p.C + c;
    for (int r = rows - 1; r >= 0; --r) {
      const float G = buf[s][0][r][lane] + carry;
      bool win;
      if (kMask) {
        win = (bits >> r) & 1u;
      } else {
        float u = buf[s][1][r][lane];
        if (kHasX) u = u + buf[s][3][r][lane];
        const float hp = (t0 + r == 0) ? hm1 : buf[s][2][r][lane];
        win = u >= a + hp;
      }
      if (cv) gout[(int64_t)r * p.C] = win ? G : 0.0f;
      const float lost = win ? 0.0f : G;
      ga += lost;
      carry = lost;
    }
    __syncwarp();
    if (lane == 0 && i + STAGES < nchunks) issue(s, nchunks - 1 - (i + STAGES));
  }
  if (cv) {
    if (p.gh0) p.gh0[b * p.C + c] = carry;
    if (p.ws) p.ws[b * p.C + c] = ga;
  }
}

// ---------------------------------------------------------------------------
// plain-load fallbacks (any alignment): one thread per (b, c)
// ---------------------------------------------------------------------------
__global__ void scan_fwd_plain_kernel(const ScanArgs p) {
  const int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (e >= p.B * p.C) return;
  const int64_t b = e / p.C, c = e % p.C;
  const float a = p.a[c];
  float h = p.h0 ? p.h0[b * p.C + c] : p.h_init;
  const int64_t nchunks = ceil_div(p.T, TS);
  uint32_t bits = 0;
  for (int64_t t = 0; t < p.T; ++t) {
    const int64_t off = (b * p.T + t) * p.C + c;
    float u = p.bb[off];
    if (p.xx) u = u + p.xx[off];
    const float d = a + h;
    const bool win = u >= d;
    h = win ? u : d;
    p.h[off] = h;
    bits |= (uint32_t)win << (t % TS);
    if (p.win && ((t % TS) == TS - 1 || t == p.T - 1)) {
      p.win[(b * nchunks + t / TS) * p.C + c] = bits;
      bits = 0;
    }
  }
}

__global__ void scan_bwd_plain_kernel(const ScanArgs p) {
  const int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (e >= p.B * p.C) return;
  const int64_t b = e / p.C, c = e % p.C;
  const float a = p.a[c];
  const float hm1 = p.h0 ? p.h0[b * p.C + c] : p.h_init;
  const int64_t nchunks = ceil_div(p.T, TS);
  float carry = 0.0f, ga = 0.0f;
  for (int64_t t = p.T - 1; t >= 0; --t) {
    const int64_t off = (b * p.T + t) * p.C + c;
    const float G = p.gh[off] + carry;
    bool win;
    if (p.win_in) {
      win = (p.win_in[(b * nchunks + t / TS) * p.C + c] >> (t % TS)) & 1u;
    } else {
      float u = p.bb[off];
      if (p.xx) u = u + p.xx[off];
      const float hp = t == 0 ? hm1 : p.h[off - p.C];
      win = u >= a + hp;
    }
    p.gu[off] = win ? G : 0.0f;
    const float lost = win ? 0.0f : G;
    ga += lost;
    carry = lost;
  }
  if (p.gh0) p.gh0[b * p.C + c] = carry;
  if (p.ws) p.ws[b * p.C + c] = ga;
}

// ga[c] = sum_b ws[b, c] in ascending b (deterministic)
__global__ void scan_ga_reduce_kernel(const float* ws, int64_t B, int64_t C, float* ga) {
  const int64_t c = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= C) return;
  float s = 0.0f;
  for (int64_t b = 0; b < B; ++b) s += ws[b * C + c];
  ga[c] = s;
}

bool scan_tma_ok(const ScanArgs& p, const float* const* ptrs, int n) {
  if (p.C % 4 != 0) return false;
  if (p.B * p.T + TS > (int64_t)INT32_MAX) return false;
  for (int i = 0; i < n; ++i)
    if (ptrs[i] && !aligned16(ptrs[i])) return false;
  return encode_tiled() != nullptr;
}

}  // namespace

int launch_scan_fwd(const ScanArgs& p_in, cudaStream_t stream) {
  if (p_in.B == 0 || p_in.C == 0 || p_in.T == 0) return TP_OK;
  ScanArgs p = p_in;
  p.err = device_error_ptr();
  const float* ptrs[2] = {p.bb, p.xx};
  const int64_t cgroups = ceil_div(p.C, 32);
  const int64_t ctas = p.B * cgroups;
  if (scan_tma_ok(p, ptrs, 2) && ctas < (int64_t)INT32_MAX) {
    CUtensorMap bmap, xmap;
    const int64_t rows = p.B * p.T;
    if (!make_scan_map(&bmap, p.bb, rows, p.C)) return TP_ERR_UNSUPPORTED;
    if (p.xx) {
      if (!make_scan_map(&xmap, p.xx, rows, p.C)) return TP_ERR_UNSUPPORTED;
    } else {
      xmap = bmap;
    }
    const unsigned grid = (unsigned)ctas;
    const int cg = (int)cgroups;
    if (p.xx) {
      if (p.win)
        scan_fwd_tma_kernel<true, true, 4><<<grid, 32, 0, stream>>>(bmap, xmap, p, cg);
      else
        scan_fwd_tma_kernel<true, false, 4><<<grid, 32, 0, stream>>>(bmap, xmap, p, cg);
    } else {
      if (p.win)
        scan_fwd_tma_kernel<false, true, 6><<<grid, 32, 0, stream>>>(bmap, xmap, p, cg);
      else
        scan_fwd_tma_kernel<false, false, 6><<<grid, 32, 0, stream>>>(bmap, xmap, p, cg);
    }
    return launch_status();
  }
  const int64_t lanes = p.B * p.C;
  scan_fwd_plain_kernel<<<(unsigned)ceil_div(lanes, 128), 128, 0, stream>>>(p);
  return launch_status();
}

int launch_scan_bwd(const ScanArgs& p_in, cudaStream_t stream) {
  if (p_in.B == 0 || p_in.C == 0) return TP_OK;
  ScanArgs p = p_in;
  p.err = device_error_ptr();
  if (p.T == 0) {
    int s = TP_OK;
    if (p.gh0) s = cuda_status(cudaMemsetAsync(p.gh0, 0, p.B * p.C * 4, stream));
    if (s == TP_OK && p.ga) s = cuda_status(cudaMemsetAsync(p.ga, 0, p.C * 4, stream));
    return s;
  }
  const float* ptrs[4] = {p.gh, p.bb, p.xx, p.h};
  const int64_t cgroups = ceil_div(p.C, 32);
  const int64_t ctas = p.B * cgroups;
  bool done = false;
  if (scan_tma_ok(p, ptrs, 4) && ctas < (int64_t)INT32_MAX) {
    CUtensorMap gmap, bmap, xmap, hmap;
    const int64_t rows = p.B * p.T;
    if (!make_scan_map(&gmap, p.gh, rows, p.C)) return TP_ERR_UNSUPPORTED;
    bmap = xmap = hmap = gmap;
    if (!p.win_in) {
      if (!make_scan_map(&bmap, p.bb, rows, p.C)) return TP_ERR_UNSUPPORTED;
      if (!make_scan_map(&hmap, p.h, rows, p.C)) return TP_ERR_UNSUPPORTED;
      if (p.xx && !make_scan_map(&xmap, p.xx, rows, p.C)) return TP_ERR_UNSUPPORTED;
    }
    const unsigned grid = (unsigned)ctas;
    const int cg = (int)cgroups;
    if (p.win_in)
      scan_bwd_tma_kernel<true, false, 6><<<grid, 32, 0, stream>>>(gmap, bmap, xmap, hmap, p, cg);
    else if (p.xx)
      scan_bwd_tma_kernel<false, true, 2><<<grid, 32, 0, stream>>>(gmap, bmap, xmap, hmap, p, cg);
    else
      scan_bwd_tma_kernel<false, false, 3><<<grid, 32, 0, stream>>>(gmap, bmap, xmap, hmap, p, cg);
    int s = launch_status();
    if (s != TP_OK) return s;
    done = true;
  }
  if (!done) {
    const int64_t lanes = p.B * p.C;
    scan_bwd_plain_kernel<<<(unsigned)ceil_div(lanes, 128), 128, 0, stream>>>(p);
    int s = launch_status();
    if (s != TP_OK) return s;
  }
  if (p.ga) {
    scan_ga_reduce_kernel<<<(unsigned)ceil_div(p.C, 128), 128, 0, stream>>>(p.ws, p.B, p.C, p.ga);
    return launch_status();
  }
  return TP_OK;
}

}  // namespace tp

// ---------------------------------------------------------------------------
// Allocation-free backward: tp_scan_bwd with its [B, C] partial-sum workspace
// taken from a fixed array in this library's device memory instead of from
// the caller.
// ---------------------------------------------------------------------------
namespace {

constexpr int64_t kScanNoAllocMaxLanes = 262144;  // B*C limit (1 MiB of fp32 partials)

// One array per GPU that loads the library, kept until the process exits.
static __device__ __align__(256) float g_scan_ga_scratch[kScanNoAllocMaxLanes];

// Device address of g_scan_ga_scratch on the current device.  The name of the
// array in host code is only a host-side stand-in, so the address is fetched
// with cudaGetSymbolAddress once per device (with that device current) and
// cached.
int scan_scratch_address(float** out) {
  static std::mutex mu;
  static float* addr[64] = {nullptr};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) {
    cudaGetLastError();
    return tp::cuda_status(e);
  }
  if (dev < 0 || dev >= 64) return TP_ERR_UNSUPPORTED;
  std::lock_guard<std::mutex> lock(mu);
  if (addr[dev] == nullptr) {
    void* ptr = nullptr;
    e = cudaGetSymbolAddress(&ptr, g_scan_ga_scratch);
    if (e != cudaSuccess) {
      cudaGetLastError();  // do not leave the error for an unrelated later call
      return tp::cuda_status(e);
    }
    addr[dev] = static_cast<float*>(ptr);
  }
  *out = addr[dev];
  return TP_OK;
}

}  // namespace

extern "C" int tp_scan_bwd_noalloc(int64_t B, int64_t T, int64_t C, const float* gh,
                                   const float* bb, const float* xx, const float* a,
                                   float h_init, const float* h0, const float* h,
                                   const uint32_t* win_mask, float* gu, float* ga, float* gh0,
                                   void* stream) {
  float* ws = nullptr;
  if (ga != nullptr && B > 0 && C > 0) {
    // tp_scan_bwd's own argument checks come first, so a call that is wrong in
    // several ways reports what tp_scan_bwd would
    if (T < 0) return TP_ERR_INVALID_ARG;
    const int chk = tp::check_scan_bwd_pointers(T, gh, bb, xx, a, h0, h, win_mask, gu, ga, gh0);
    if (chk != TP_OK) return chk;
    // with T == 0 the backward only zeroes ga and gh0: the array is not used
    if (T > 0 && B > kScanNoAllocMaxLanes / C) return TP_ERR_TOO_LARGE;
    const int s = scan_scratch_address(&ws);
    if (s != TP_OK) return s;
  }
  return tp_scan_bwd(B, T, C, gh, bb, xx, a, h_init, h0, h, win_mask, gu, ga, gh0, ws, stream);
}
