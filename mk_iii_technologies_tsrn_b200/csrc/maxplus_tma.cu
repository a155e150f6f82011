// maxplus_tma.cu -- persistent, warp-specialised fp32 max-plus GEMM for sm_100a.
//
//   y[m,n] = max_k (x[m,k] + w[n,k])  (+bias, *scale)   and   argmax[m,n]
//
// This is the large-problem path of tp_maxplus_fwd (the tropical linear of
// tropformer.py:127-145 at GEMM scale, and the M=N=K sweep).  Max-plus is not
// a multiply-add, so tensor cores do not apply; the kernel is bound by the
// CUDA-core issue rate.  Per two k-terms of one output it issues exactly two
// instructions: one packed add.rn.f32x2 (both sums, each one rounded fp32
// add) and one 3-input max.NaN.f32 folding both sums into the accumulator.
//
// CTA (one per SM, persistent over 128x128 output tiles, grouped raster):
//   warps 0-7   compute: 16x16 threads, 8x8 outputs per thread
//   warp  8     producer: one lane issues TMA loads of 128x32 fp32 x/w tiles
//               (128-byte swizzle) into a 4-stage full/empty mbarrier ring
//   warps 9-11  argmax recovery (only when argmax is requested)
//
// Exact argmax without per-term index tracking.  The running max only grows,
// so the lowest k attaining the final max lies in the LAST 64-wide k-chunk in
// which the accumulator changed.  Every 64 k the compute threads compare
// their accumulators with a snapshot kept in shared memory (bitwise, so NaN
// counts once) and record the chunk index (16-bit, in shared memory).  At the end of a tile they store the raw max and
// the chunk index to y/argmax and hand the tile to the recovery warps, which,
// while the compute warps already run the next tile, re-read the 64 terms of
// each output's chunk from global memory (L2), find the first k whose sum
// equals the max (or is NaN when the max is NaN), and write the final argmax
// and the epilogue value.  The result equals torch.max(dim=-1) on the
// reference's broadcast tensor, bit for bit, in values and indices.
//
// Every mbarrier wait is bounded (common.cuh); a timeout records a device
// error and the kernel returns.
#include "maxplus_internal.cuh"

namespace tp {

namespace {

constexpr int BM = 128;
constexpr int BN = 128;
constexpr int BK = 32;           // fp32 per TMA row: 128 bytes (one swizzle atom)
constexpr int STAGES = 4;
constexpr int CHUNK = 64;        // argmax tracking granularity in k
constexpr int KT_PER_CHUNK = CHUNK / BK;
constexpr int N_COMPUTE_WARPS = 8;
constexpr int N_RECOVERY_WARPS = 3;
constexpr int PRODUCER_WARP = N_COMPUTE_WARPS;
constexpr int THREADS = 32 * (N_COMPUTE_WARPS + 1 + N_RECOVERY_WARPS);  // 384
constexpr int TILE_BYTES = BM * BK * 4;                                  // 16 KB
constexpr int STAGE_BYTES = 2 * TILE_BYTES;
constexpr int SNAP_BYTES = 256 * 64 * 4;                                 // 64 KB
constexpr int CIDX_BYTES = 256 * 64 * 2;                                 // 32 KB
constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + SNAP_BYTES + CIDX_BYTES + 256 + 1024;
constexpr int64_t MAX_K = (int64_t)CHUNK * 65535;  // 16-bit chunk index

struct TmaParams {
  int64_t M, N, K;
  const float* x;
  int64_t ldx;
  const float* w;
  int64_t ldw;
  const float* bias;
  float* y;
  int64_t ldy;
  int32_t* am;
  int64_t lda;
  float scale;
  int m_tiles, n_tiles, k_tiles, num_tiles;
  int* err;
};

__device__ __forceinline__ void tile_coords(int tile, int m_tiles, int n_tiles, int& mt, int& nt) {
  constexpr int GROUP = 8;
  const int per_group = GROUP * n_tiles;
  const int g = tile / per_group;
  const int first_m = g * GROUP;
  const int gsize = min(GROUP, m_tiles - first_m);
  const int r = tile - g * per_group;
  mt = first_m + r % gsize;
  nt = r / gsize;
}

// acc = max.NaN(acc, x0 + w0, x1 + w1) with both sums from one add.rn.f32x2.
__device__ __forceinline__ void mp_pair(float& acc, uint64_t xa, uint64_t wb) {
  asm("{\n\t.reg .b64 s;\n\t.reg .f32 lo, hi;\n\t"
      "add.rn.f32x2 s, %1, %2;\n\t"
      "mov.b64 {lo, hi}, s;\n\t"
      "max.NaN.f32 %0, %0, lo, hi;\n\t}"
      : "+f"(acc)
      : "l"(xa), "l"(wb));
}

__device__ __forceinline__ void lds128(uint32_t addr, uint64_t& a, uint64_t& b) {
  asm volatile("ld.shared.v2.u64 {%0, %1}, [%2];" : "=l"(a), "=l"(b) : "r"(addr));
}

__device__ __forceinline__ uint64_t mask_pair(uint64_t v, bool lo_bad, bool hi_bad) {
  const uint64_t NEG = 0xff800000ull;
  if (lo_bad) v = (v & 0xffffffff00000000ull) | NEG;
  if (hi_bad) v = (v & 0x00000000ffffffffull) | (NEG << 32);
  return v;
}

template <bool kArgmax>
__global__ void __launch_bounds__(THREADS, 1)
    maxplus_tma_kernel(const __grid_constant__ CUtensorMap xmap,
                       const __grid_constant__ CUtensorMap wmap, const TmaParams p) {
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  // 1024-byte alignment for the 128-byte swizzle pattern
  unsigned char* smem =
      (unsigned char*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  unsigned char* stage_base = smem;                                  // STAGES x (x tile, w tile)
  float4* snap = (float4*)(smem + STAGES * STAGE_BYTES);             // [16][256]
  uint16_t* cid = (uint16_t*)(smem + STAGES * STAGE_BYTES + SNAP_BYTES);  // [64][256]
  uint64_t* bars = (uint64_t*)(smem + STAGES * STAGE_BYTES + SNAP_BYTES + CIDX_BYTES);
  uint64_t* full = bars;                 // [STAGES]
  uint64_t* empty = bars + STAGES;       // [STAGES]
  uint64_t* done = bars + 2 * STAGES;    // [2] compute -> recovery
  uint64_t* freeb = bars + 2 * STAGES + 2;  // [2] recovery -> compute

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  constexpr bool with_argmax = kArgmax;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      tp_mbar_init(&full[s], 1);
      tp_mbar_init(&empty[s], N_COMPUTE_WARPS);
    }
    for (int b = 0; b < 2; ++b) {
      tp_mbar_init(&done[b], N_COMPUTE_WARPS);
      tp_mbar_init(&freeb[b], N_RECOVERY_WARPS);
    }
    tp_fence_mbar_init();
  }
  __syncthreads();

  if (warp == PRODUCER_WARP) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      tp_prefetch_tensormap(&xmap);
      tp_prefetch_tensormap(&wmap);
      uint32_t it = 0;
      for (int tile = blockIdx.x; tile < p.num_tiles; tile += gridDim.x) {
        int mt, nt;
        tile_coords(tile, p.m_tiles, p.n_tiles, mt, nt);
        for (int kt = 0; kt < p.k_tiles; ++kt, ++it) {
          const uint32_t s = it % STAGES;
          const uint32_t ph = (it / STAGES) & 1u;
          if (!tp_mbar_wait(&empty[s], ph ^ 1u, p.err)) return;
          unsigned char* dst = stage_base + s * STAGE_BYTES;
          tp_mbar_arrive_expect_tx(&full[s], STAGE_BYTES);
          tp_tma_load_2d(dst, &xmap, kt * BK, mt * BM, &full[s]);
          tp_tma_load_2d(dst + TILE_BYTES, &wmap, kt * BK, nt * BN, &full[s]);
        }
      }
    }
    return;
  }

  if (warp > PRODUCER_WARP) {
    // ------------------------------------------------------------ recovery
    if (!with_argmax) return;
    const int rw = warp - PRODUCER_WARP - 1;  // 0..2
    const int half = lane >> 4;               // which of the two outputs of a step
    const int hl = lane & 15;                 // 4 consecutive k per lane
    int lt = 0;
    for (int tile = blockIdx.x; tile < p.num_tiles; tile += gridDim.x, ++lt) {
      int mt, nt;
      tile_coords(tile, p.m_tiles, p.n_tiles, mt, nt);
      const int b = lt & 1;
      if (!tp_mbar_wait(&done[b], (uint32_t)((lt >> 1) & 1), p.err)) return;
      const int64_t m0 = (int64_t)mt * BM, n0 = (int64_t)nt * BN;
      const int64_t mend = min((int64_t)BM, p.M - m0);
      const int64_t nend = min((int64_t)BN, p.N - n0);
      for (int64_t r = rw; r < mend; r += N_RECOVERY_WARPS) {
        const int64_t m = m0 + r;
        // this lane's 4 outputs of the row: n = n0 + 4*lane + c
        int32_t cidx[4];
        float tgt[4];
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          const int64_t nn = 4 * lane + c;
          if (nn < nend) {
            cidx[c] = __ldcg(p.am + m * p.lda + n0 + nn);
            tgt[c] = __ldcg(p.y + m * p.ldy + n0 + nn);
          } else {
            cidx[c] = 0;
            tgt[c] = 0.0f;
          }
        }
        const float* xrow = p.x + m * p.ldx;
        // 64 steps of two outputs each (one per half-warp)
#pragma unroll 4
        for (int st = 0; st < BN / 2; ++st) {
          const int nn = 2 * st + half;           // output column within the tile
          const int src = nn >> 2, comp = nn & 3;  // lane/slot holding its chunk
          int32_t cj = __shfl_sync(0xffffffffu, cidx[0], src);
          float tv = __shfl_sync(0xffffffffu, tgt[0], src);
          const int32_t c1 = __shfl_sync(0xffffffffu, cidx[1], src);
          const float t1 = __shfl_sync(0xffffffffu, tgt[1], src);
          const int32_t c2 = __shfl_sync(0xffffffffu, cidx[2], src);
          const float t2 = __shfl_sync(0xffffffffu, tgt[2], src);
          const int32_t c3 = __shfl_sync(0xffffffffu, cidx[3], src);
          const float t3 = __shfl_sync(0xffffffffu, tgt[3], src);
          if (comp == 1) { cj = c1; tv = t1; }
          if (comp == 2) { cj = c2; tv = t2; }
          if (comp == 3) { cj = c3; tv = t3; }
          const bool valid = nn < nend;
          const int64_t n = n0 + nn;
          const int64_t kb = (int64_t)cj * CHUNK + 4 * hl;
          float xs4[4], ws4[4];
          if (valid && kb + 3 < p.K) {
            const float4 xv = __ldg((const float4*)(xrow + kb));
            const float4 wv = __ldg((const float4*)(p.w + n * p.ldw + kb));
            xs4[0] = xv.x; xs4[1] = xv.y; xs4[2] = xv.z; xs4[3] = xv.w;
            ws4[0] = wv.x; ws4[1] = wv.y; ws4[2] = wv.z; ws4[3] = wv.w;
          } else {
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const bool in = valid && (kb + e < p.K);
              xs4[e] = in ? __ldg(xrow + kb + e) : -__int_as_float(0x7f800000);
              ws4[e] = in ? __ldg(p.w + n * p.ldw + kb + e) : 0.0f;
            }
          }
          const bool tnan = tv != tv;
          int first = 4;
#pragma unroll
          for (int e = 3; e >= 0; --e) {
            const float s = xs4[e] + ws4[e];
            const bool hit = (kb + e < p.K) && (tnan ? (s != s) : (s == tv));
            if (hit) first = e;
          }
          const unsigned ball = __ballot_sync(0xffffffffu, first < 4);
          const unsigned mine = (ball >> (16 * half)) & 0xffffu;
          const int wl = mine ? (__ffs(mine) - 1) : 0;
          const int fe = __shfl_sync(0xffffffffu, first, 16 * half + wl);
          if (valid && hl == 0) {
            const int64_t k = mine ? ((int64_t)cj * CHUNK + 4 * wl + fe) : (int64_t)cj * CHUNK;
            p.am[m * p.lda + n] = (int32_t)k;
            if (p.bias != nullptr || p.scale != 1.0f) {
              float v = tv;
              if (p.bias) v = v + p.bias[n];
              if (p.scale != 1.0f) v = v * p.scale;
              p.y[m * p.ldy + n] = v;
            }
          }
        }
      }
      __syncwarp();
      if (lane == 0) tp_mbar_arrive(&freeb[b]);
    }
    return;
  }

  // -------------------------------------------------------------- compute
  const int t = threadIdx.x;  // 0..255
  const int tx = t & 15;
  const int ty = t >> 4;
  const uint32_t stage_addr = tp_smem_addr(stage_base);
  const uint32_t xsw = (uint32_t)(ty & 7);
  const uint32_t wsw = (uint32_t)(tx & 7);
  const float NEG_INF = -__int_as_float(0x7f800000);
  uint32_t it = 0;
  int lt = 0;
  for (int tile = blockIdx.x; tile < p.num_tiles; tile += gridDim.x, ++lt) {
    int mt, nt;
    tile_coords(tile, p.m_tiles, p.n_tiles, mt, nt);
    float acc[8][8];
#pragma unroll
    for (int i = 0; i < 8; ++i)
#pragma unroll
      for (int j = 0; j < 8; ++j) acc[i][j] = NEG_INF;
    if (with_argmax) {
#pragma unroll
      for (int q = 0; q < 16; ++q) snap[q * 256 + t] = make_float4(NEG_INF, NEG_INF, NEG_INF, NEG_INF);
#pragma unroll
      for (int o = 0; o < 64; ++o) cid[o * 256 + t] = 0;
    }

    for (int kt = 0; kt < p.k_tiles; ++kt, ++it) {
      const uint32_t s = it % STAGES;
      const uint32_t ph = (it / STAGES) & 1u;
      if (!tp_mbar_wait(&full[s], ph, p.err)) return;
      const uint32_t xbase = stage_addr + s * STAGE_BYTES;
      const uint32_t wbase = xbase + TILE_BYTES;
      const int64_t k0 = (int64_t)kt * BK;
      const bool tail = k0 + BK > p.K;
#pragma unroll
      for (int q = 0; q < BK / 4; ++q) {
        uint64_t xa[8][2];
#pragma unroll
        for (int i = 0; i < 8; ++i)
          lds128(xbase + (uint32_t)(ty + 16 * i) * 128u + (((uint32_t)q ^ xsw) << 4), xa[i][0],
                 xa[i][1]);
        if (tail) {
          const int64_t kq = k0 + 4 * q;
          const bool b0 = kq >= p.K, b1 = kq + 1 >= p.K, b2 = kq + 2 >= p.K, b3 = kq + 3 >= p.K;
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            xa[i][0] = mask_pair(xa[i][0], b0, b1);
            xa[i][1] = mask_pair(xa[i][1], b2, b3);
          }
        }
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          uint64_t wb0, wb1;
          lds128(wbase + (uint32_t)(tx + 16 * j) * 128u + (((uint32_t)q ^ wsw) << 4), wb0, wb1);
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            mp_pair(acc[i][j], xa[i][0], wb0);
            mp_pair(acc[i][j], xa[i][1], wb1);
          }
        }
      }
      __syncwarp();
      if (lane == 0) tp_mbar_arrive(&empty[s]);

      if (with_argmax && (((kt + 1) % KT_PER_CHUNK) == 0 || kt == p.k_tiles - 1)) {
        const uint16_t chunk = (uint16_t)(kt / KT_PER_CHUNK);
#pragma unroll
        for (int q = 0; q < 16; ++q) {
          float4 sv = snap[q * 256 + t];
          const float* svp = reinterpret_cast<const float*>(&sv);
          float nv[4];
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            const int o = 4 * q + c;
            const float a = acc[o >> 3][o & 7];
            nv[c] = a;
            if (__float_as_uint(a) != __float_as_uint(svp[c])) cid[o * 256 + t] = chunk;
          }
          snap[q * 256 + t] = make_float4(nv[0], nv[1], nv[2], nv[3]);
        }
      }
    }

    // ---- epilogue
    const int64_t m0 = (int64_t)mt * BM, n0 = (int64_t)nt * BN;
    const int b = lt & 1;
    if (with_argmax) {
      // recovery must have released this done/free slot (tile lt-2)
      if (!tp_mbar_wait(&freeb[b], (uint32_t)(((lt >> 1) & 1) ^ 1), p.err)) return;
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int64_t m = m0 + ty + 16 * i;
      if (m >= p.M) continue;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int64_t n = n0 + tx + 16 * j;
        if (n >= p.N) continue;
        float v = acc[i][j];
        if (with_argmax) {
          const int o = i * 8 + j;
          p.y[m * p.ldy + n] = v;  // raw max; recovery applies bias/scale
          p.am[m * p.lda + n] = (int32_t)cid[o * 256 + t];
        } else {
          if (p.bias) v = v + p.bias[n];
          if (p.scale != 1.0f) v = v * p.scale;
          p.y[m * p.ldy + n] = v;
        }
      }
    }
    if (with_argmax) {
      __threadfence_block();
      __syncwarp();
      if (lane == 0) tp_mbar_arrive(&done[b]);
    }
  }
}

bool make_map(CUtensorMap* map, const float* base, int64_t rows, int64_t K, int64_t ld) {
  EncodeTiledFn enc = encode_tiled();
  if (!enc) return false;
  cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)ld * 4};
  cuuint32_t box[2] = {BK, 128};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, (void*)base, dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

}  // namespace

bool maxplus_tma_eligible(const StridedMaxPlus& p) {
  if (p.dtype != TP_DTYPE_F32) return false;
  if (p.B1 * p.B2 != 1) return false;
  if (p.sx_k != 1 || p.sw_k != 1 || p.sy_n != 1) return false;
  if (p.am && p.sa_n != 1) return false;
  if (p.M < BM || p.N < BN || p.K < 2 * BK || p.K > MAX_K) return false;
  if ((p.sx_m % 4) != 0 || (p.sw_n % 4) != 0) return false;
  if (!aligned16(p.x) || !aligned16(p.w)) return false;
  if (p.M > (int64_t)INT32_MAX || p.N > (int64_t)INT32_MAX) return false;
  const int64_t tiles = ceil_div(p.M, BM) * ceil_div(p.N, BN);
  return tiles >= 16 && tiles < (int64_t)INT32_MAX;
}

int launch_maxplus_fwd_tma(const StridedMaxPlus& p, cudaStream_t stream) {
  if (!maxplus_tma_eligible(p)) return TP_ERR_UNSUPPORTED;
  CUtensorMap xmap, wmap;
  if (!make_map(&xmap, (const float*)p.x, p.M, p.K, p.sx_m)) return TP_ERR_UNSUPPORTED;
  if (!make_map(&wmap, (const float*)p.w, p.N, p.K, p.sw_n)) return TP_ERR_UNSUPPORTED;
  TmaParams tp_;
  tp_.M = p.M;
  tp_.N = p.N;
  tp_.K = p.K;
  tp_.x = (const float*)p.x;
  tp_.ldx = p.sx_m;
  tp_.w = (const float*)p.w;
  tp_.ldw = p.sw_n;
  tp_.bias = p.bias;
  tp_.y = p.y;
  tp_.ldy = p.sy_m;
  tp_.am = p.am;
  tp_.lda = p.am ? p.sa_m : 0;
  tp_.scale = p.scale;
  tp_.m_tiles = (int)ceil_div(p.M, BM);
  tp_.n_tiles = (int)ceil_div(p.N, BN);
  tp_.k_tiles = (int)ceil_div(p.K, BK);
  tp_.num_tiles = tp_.m_tiles * tp_.n_tiles;
  tp_.err = device_error_ptr();
  // The attribute is per function and per device; setting it is cheap.
  cudaError_t e = cudaFuncSetAttribute(maxplus_tma_kernel<true>,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES);
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(maxplus_tma_kernel<false>,
                             cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES);
  if (e != cudaSuccess) return (int)e;
  int grid = num_sms();
  if (grid > tp_.num_tiles) grid = tp_.num_tiles;
  if (p.am)
    maxplus_tma_kernel<true><<<grid, THREADS, SMEM_BYTES, stream>>>(xmap, wmap, tp_);
  else
    maxplus_tma_kernel<false><<<grid, THREADS, SMEM_BYTES, stream>>>(xmap, wmap, tp_);
  return launch_status();
}

}  // namespace tp
