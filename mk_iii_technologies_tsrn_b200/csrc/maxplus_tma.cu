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
//   compute warps   TY x TX threads, TM x TN outputs per thread (template)
//   producer warp   one lane issues TMA loads of 128x32 fp32 x/w tiles
//                   (128-byte swizzle) into a 4-stage full/empty mbarrier ring
//   recovery warps  argmax recovery (only when argmax is requested)
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

#ifndef TP_TMA_TM
#define TP_TMA_TM 4
#endif
#ifndef TP_TMA_TN
#define TP_TMA_TN 8
#endif
#ifndef TP_TMA_CHUNK
#define TP_TMA_CHUNK 64
#endif
#ifndef TP_TMA_QUNROLL
#define TP_TMA_QUNROLL 8
#endif

constexpr int QUNROLL = TP_TMA_QUNROLL;
constexpr int BM = 128;
constexpr int BN = 128;
constexpr int BK = 32;           // fp32 per TMA row: 128 bytes (one swizzle atom)
constexpr int STAGES = 4;
constexpr int TILE_BYTES = BM * BK * 4;                                  // 16 KB
constexpr int STAGE_BYTES = 2 * TILE_BYTES;
constexpr int SNAP_BYTES = BM * BN * 4;                                  // 64 KB
constexpr int CIDX_BYTES = BM * BN * 2;                                  // 32 KB
constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + SNAP_BYTES + CIDX_BYTES + 256 + 1024;

template <int TM_, int TN_, int CHUNK_>
struct Cfg {
  static constexpr int TM = TM_, TN = TN_, CHUNK = CHUNK_;
  static constexpr int TX = BN / TN;       // threads along n
  static constexpr int TY = BM / TM;       // threads along m
  static constexpr int CT = TX * TY;       // compute threads
  static constexpr int CW = CT / 32;       // compute warps
  static constexpr int PRODUCER_WARP = CW;
  static constexpr int RW = 3;             // recovery warps (CW + 1 + RW: multiple of 4)
  static constexpr int THREADS = 32 * (CW + 1 + RW);
  static constexpr int OUTS = TM * TN;     // outputs per compute thread
  static constexpr int KT_PER_CHUNK = CHUNK / BK;
  static constexpr int LANES_PER_OUT = CHUNK / 4;   // recovery: 4 k per lane
  static constexpr int OUT_PER_STEP = 32 / LANES_PER_OUT;
  static constexpr int U = CW >= 16 ? 4 : 8;        // recovery steps in flight
  static constexpr int64_t MAX_K = (int64_t)CHUNK * 65535;  // 16-bit chunk index
  static_assert(CT % 32 == 0, "compute threads must fill warps");
  static_assert(OUTS % 4 == 0, "snapshot uses float4");
  static_assert((TX % 8) == 0 && (TY % 8) == 0, "swizzle phase must be per-thread constant");
  static_assert(CHUNK % BK == 0 && LANES_PER_OUT <= 32, "chunk");
};

using DefaultCfg = Cfg<TP_TMA_TM, TP_TMA_TN, TP_TMA_CHUNK>;

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

// ---------------------------------------------------------------------------
// argmax recovery for one finished tile: for each output, find the first k of
// its recorded chunk whose sum equals the raw max (first NaN when the max is
// NaN); write the index and the epilogue value.  A group of LANES_PER_OUT lanes
// handles one output (4 consecutive k per lane, 16-byte loads); U steps of
// loads are issued before any compare so that the gathers overlap.
// ---------------------------------------------------------------------------
template <class C>
__device__ __forceinline__ void recover_tile(const TmaParams& p, int mt, int nt, int rw, int lane) {
  constexpr int G = C::LANES_PER_OUT;
  constexpr int OPS = C::OUT_PER_STEP;
  constexpr int U = C::U;
  const int grp = lane / G;       // output slot within a warp step
  const int gl = lane % G;        // lane within the group
  const int64_t m0 = (int64_t)mt * BM, n0 = (int64_t)nt * BN;
  const int64_t mend = min((int64_t)BM, p.M - m0);
  const int64_t nend = min((int64_t)BN, p.N - n0);
  const float NEG_INF = -__int_as_float(0x7f800000);
  const int64_t total = mend * BN;
  for (int64_t base = (int64_t)rw * OPS * U; base < total; base += (int64_t)C::RW * OPS * U) {
    int32_t cj[U];
    float tv[U];
    int64_t orow[U], ocol[U];
    bool valid[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int64_t o = base + (int64_t)u * OPS + grp;
      const int64_t r = o / BN, c = o % BN;
      valid[u] = (o < total) && (c < nend);
      orow[u] = m0 + (valid[u] ? r : 0);
      ocol[u] = n0 + (valid[u] ? c : 0);
      cj[u] = valid[u] ? __ldcg(p.am + orow[u] * p.lda + ocol[u]) : 0;
      tv[u] = valid[u] ? __ldcg(p.y + orow[u] * p.ldy + ocol[u]) : 0.0f;
    }
    float4 xv[U], wv[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int64_t kb = (int64_t)cj[u] * C::CHUNK + 4 * gl;
      const bool full = valid[u] && (kb + 3 < p.K);
      const int64_t kq = full ? kb : 0;   // in-bounds dummy address otherwise
      xv[u] = __ldg((const float4*)(p.x + orow[u] * p.ldx + kq));
      wv[u] = __ldg((const float4*)(p.w + ocol[u] * p.ldw + kq));
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int64_t kb = (int64_t)cj[u] * C::CHUNK + 4 * gl;
      float xs[4] = {xv[u].x, xv[u].y, xv[u].z, xv[u].w};
      float ws[4] = {wv[u].x, wv[u].y, wv[u].z, wv[u].w};
      if (valid[u] && kb < p.K && kb + 3 >= p.K) {   // quad straddling K (K % 4 != 0)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const bool in = kb + e < p.K;
          xs[e] = in ? __ldg(p.x + orow[u] * p.ldx + kb + e) : NEG_INF;
          ws[e] = in ? __ldg(p.w + ocol[u] * p.ldw + kb + e) : 0.0f;
        }
      }
      const bool tnan = tv[u] != tv[u];
      int first = 4;
#pragma unroll
      for (int e = 3; e >= 0; --e) {
        const float s = xs[e] + ws[e];
        const bool hit = valid[u] && (kb + e < p.K) && (tnan ? (s != s) : (s == tv[u]));
        if (hit) first = e;
      }
      const unsigned ball = __ballot_sync(0xffffffffu, first < 4);
      const unsigned mine = (ball >> (grp * G)) & ((G == 32) ? 0xffffffffu : ((1u << G) - 1u));
      const int wl = mine ? (__ffs(mine) - 1) : 0;
      const int fe = __shfl_sync(0xffffffffu, first, grp * G + wl);
      if (valid[u] && gl == 0) {
        const int64_t k = (int64_t)cj[u] * C::CHUNK + (mine ? (4 * wl + fe) : 0);
        p.am[orow[u] * p.lda + ocol[u]] = (int32_t)k;
        if (p.bias != nullptr || p.scale != 1.0f) {
          float v = tv[u];
          if (p.bias) v = v + p.bias[ocol[u]];
          if (p.scale != 1.0f) v = v * p.scale;
          p.y[orow[u] * p.ldy + ocol[u]] = v;
        }
      }
    }
  }
}

template <class C, bool kArgmax>
__global__ void __launch_bounds__(C::THREADS, 1)
    maxplus_tma_kernel(const __grid_constant__ CUtensorMap xmap,
                       const __grid_constant__ CUtensorMap wmap, const TmaParams p) {
  constexpr int TM = C::TM, TN = C::TN, TX = C::TX, TY = C::TY, CT = C::CT;
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  // 1024-byte alignment for the 128-byte swizzle pattern
  unsigned char* smem =
      (unsigned char*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  unsigned char* stage_base = smem;                                  // STAGES x (x tile, w tile)
  float4* snap = (float4*)(smem + STAGES * STAGE_BYTES);             // [OUTS/4][CT]
  uint16_t* cid = (uint16_t*)(smem + STAGES * STAGE_BYTES + SNAP_BYTES);  // [OUTS][CT]
  uint64_t* bars = (uint64_t*)(smem + STAGES * STAGE_BYTES + SNAP_BYTES + CIDX_BYTES);
  uint64_t* full = bars;                 // [STAGES]
  uint64_t* empty = bars + STAGES;       // [STAGES]
  uint64_t* done = bars + 2 * STAGES;    // [2] compute -> recovery
  uint64_t* freeb = bars + 2 * STAGES + 2;  // [2] recovery -> compute

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      tp_mbar_init(&full[s], 1);
      tp_mbar_init(&empty[s], C::CW);
    }
    for (int b = 0; b < 2; ++b) {
      tp_mbar_init(&done[b], C::CW);
      tp_mbar_init(&freeb[b], C::RW);
    }
    tp_fence_mbar_init();
  }
  __syncthreads();

  if (warp == C::PRODUCER_WARP) {
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

  if (warp > C::PRODUCER_WARP) {
    // ------------------------------------------------------------ recovery
    if (!kArgmax) return;
    const int rw = warp - C::PRODUCER_WARP - 1;
    int lt = 0;
    for (int tile = blockIdx.x; tile < p.num_tiles; tile += gridDim.x, ++lt) {
      int mt, nt;
      tile_coords(tile, p.m_tiles, p.n_tiles, mt, nt);
      const int b = lt & 1;
      if (!tp_mbar_wait(&done[b], (uint32_t)((lt >> 1) & 1), p.err)) return;
      recover_tile<C>(p, mt, nt, rw, lane);
      __syncwarp();
      if (lane == 0) tp_mbar_arrive(&freeb[b]);
    }
    return;
  }

  // -------------------------------------------------------------- compute
  const int t = threadIdx.x;  // 0..CT-1
  const int tx = t % TX;
  const int ty = t / TX;
  const uint32_t stage_addr = tp_smem_addr(stage_base);
  const uint32_t xsw = (uint32_t)(ty & 7);
  const uint32_t wsw = (uint32_t)(tx & 7);
  const float NEG_INF = -__int_as_float(0x7f800000);
  uint32_t it = 0;
  int lt = 0;
  for (int tile = blockIdx.x; tile < p.num_tiles; tile += gridDim.x, ++lt) {
    int mt, nt;
    tile_coords(tile, p.m_tiles, p.n_tiles, mt, nt);
    float acc[TM][TN];
#pragma unroll
    for (int i = 0; i < TM; ++i)
#pragma unroll
      for (int j = 0; j < TN; ++j) acc[i][j] = NEG_INF;
    if (kArgmax) {
#pragma unroll
      for (int q = 0; q < C::OUTS / 4; ++q)
        snap[q * CT + t] = make_float4(NEG_INF, NEG_INF, NEG_INF, NEG_INF);
#pragma unroll
      for (int o = 0; o < C::OUTS; ++o) cid[o * CT + t] = 0;
    }

    for (int kt = 0; kt < p.k_tiles; ++kt, ++it) {
      const uint32_t s = it % STAGES;
      const uint32_t ph = (it / STAGES) & 1u;
      if (!tp_mbar_wait(&full[s], ph, p.err)) return;
      const uint32_t xbase = stage_addr + s * STAGE_BYTES;
      const uint32_t wbase = xbase + TILE_BYTES;
      const int64_t k0 = (int64_t)kt * BK;
      const bool tail = k0 + BK > p.K;
#pragma unroll QUNROLL
      for (int q = 0; q < BK / 4; ++q) {
        uint64_t xa[TM][2];
#pragma unroll
        for (int i = 0; i < TM; ++i)
          lds128(xbase + (uint32_t)(ty + TY * i) * 128u + (((uint32_t)q ^ xsw) << 4), xa[i][0],
                 xa[i][1]);
        if (tail) {
          const int64_t kq = k0 + 4 * q;
          const bool b0 = kq >= p.K, b1 = kq + 1 >= p.K, b2 = kq + 2 >= p.K, b3 = kq + 3 >= p.K;
#pragma unroll
          for (int i = 0; i < TM; ++i) {
            xa[i][0] = mask_pair(xa[i][0], b0, b1);
            xa[i][1] = mask_pair(xa[i][1], b2, b3);
          }
        }
#pragma unroll
        for (int j = 0; j < TN; ++j) {
          uint64_t wb0, wb1;
          lds128(wbase + (uint32_t)(tx + TX * j) * 128u + (((uint32_t)q ^ wsw) << 4), wb0, wb1);
#pragma unroll
          for (int i = 0; i < TM; ++i) {
            mp_pair(acc[i][j], xa[i][0], wb0);
            mp_pair(acc[i][j], xa[i][1], wb1);
          }
        }
      }
      __syncwarp();
      if (lane == 0) tp_mbar_arrive(&empty[s]);

      if (kArgmax && (((kt + 1) % C::KT_PER_CHUNK) == 0 || kt == p.k_tiles - 1)) {
        const uint16_t chunk = (uint16_t)(kt / C::KT_PER_CHUNK);
#pragma unroll
        for (int q = 0; q < C::OUTS / 4; ++q) {
          float4 sv = snap[q * CT + t];
          const float* svp = reinterpret_cast<const float*>(&sv);
          float nv[4];
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            const int o = 4 * q + c;
            const float a = acc[o / TN][o % TN];
            nv[c] = a;
            if (__float_as_uint(a) != __float_as_uint(svp[c])) cid[o * CT + t] = chunk;
          }
          snap[q * CT + t] = make_float4(nv[0], nv[1], nv[2], nv[3]);
        }
      }
    }

    // ---- epilogue
    const int64_t m0 = (int64_t)mt * BM, n0 = (int64_t)nt * BN;
    const int b = lt & 1;
    if (kArgmax) {
      // recovery must have released this done/free slot (tile lt-2)
      if (!tp_mbar_wait(&freeb[b], (uint32_t)(((lt >> 1) & 1) ^ 1), p.err)) return;
    }
#pragma unroll
    for (int i = 0; i < TM; ++i) {
      const int64_t m = m0 + ty + TY * i;
      if (m >= p.M) continue;
#pragma unroll
      for (int j = 0; j < TN; ++j) {
        const int64_t n = n0 + tx + TX * j;
        if (n >= p.N) continue;
        float v = acc[i][j];
        if (kArgmax) {
          p.y[m * p.ldy + n] = v;  // raw max; recovery applies bias/scale
          p.am[m * p.lda + n] = (int32_t)cid[(i * TN + j) * CT + t];
        } else {
          if (p.bias) v = v + p.bias[n];
          if (p.scale != 1.0f) v = v * p.scale;
          p.y[m * p.ldy + n] = v;
        }
      }
    }
    if (kArgmax) {
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

template <class C, bool kArgmax>
int launch_cfg(const CUtensorMap& xmap, const CUtensorMap& wmap, const TmaParams& tp_,
               cudaStream_t stream) {
  cudaError_t e = cudaFuncSetAttribute(maxplus_tma_kernel<C, kArgmax>,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES);
  if (e != cudaSuccess) return (int)e;
  int grid = num_sms();
  if (grid > tp_.num_tiles) grid = tp_.num_tiles;
  maxplus_tma_kernel<C, kArgmax><<<grid, C::THREADS, SMEM_BYTES, stream>>>(xmap, wmap, tp_);
  return launch_status();
}

}  // namespace

bool maxplus_tma_eligible(const StridedMaxPlus& p) {
  if (p.dtype != TP_DTYPE_F32) return false;
  if (p.B1 * p.B2 != 1) return false;
  if (p.sx_k != 1 || p.sw_k != 1 || p.sy_n != 1) return false;
  if (p.am && p.sa_n != 1) return false;
  if (p.M < BM || p.N < BN || p.K < 2 * BK || p.K > DefaultCfg::MAX_K) return false;
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
  if (p.am) return launch_cfg<DefaultCfg, true>(xmap, wmap, tp_, stream);
  return launch_cfg<DefaultCfg, false>(xmap, wmap, tp_, stream);
}

}  // namespace tp
