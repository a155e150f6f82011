// maxplus_tma.cu -- persistent, warp-specialised fp32 max-plus GEMM for sm_100a.
//
//   y[m,n] = max_k (x[m,k] + w[n,k])  (+bias, *scale)   and   argmax[m,n]
//
// This is the large-problem path of tp_maxplus_fwd (the tropical linear of
// tropformer.py:127-145 at GEMM scale, and the M=N=K sweep).  Max-plus is not
// a multiply-add, so tensor cores do not apply; the kernel is bound by the
// CUDA-core add and max rates.  Per two k-terms of one output it issues two
// instructions: one packed add.rn.f32x2 (both sums, each one rounded fp32
// add) and one 3-input max.NaN.f32 folding both sums into the accumulator.
//
// CTA (one per SM, persistent over 128x128 output tiles, grouped raster):
//   compute warps   TY x TX threads, TM x TN outputs per thread (template)
//   producer warp   one lane issues TMA loads of 128x32 fp32 x/w tiles
//                   (128-byte swizzle, no multicast) into a 4-stage
//                   full/empty mbarrier ring
//
// Exact argmax without per-term index tracking.  The running max only grows,
// so the lowest k attaining the final max lies in the LAST CHUNK-wide k-range
// in which the accumulator changed.  At each chunk boundary the compute
// threads compare their accumulators with a snapshot kept in shared memory
// (bitwise, so NaN counts once) and record the chunk index (16-bit, shared
// memory).  After the main pass over K the producer streams the tile's
// k-tiles through the ring a second time (the data is mostly still in L2).
// The outputs are first bucketed by chunk (a counting sort in shared memory),
// so that each chunk's outputs are searched by all compute warps evenly,
// straight from shared memory: the first k whose sum equals the output's max
// (or is NaN when the max is NaN) is its argmax.  The
// result equals torch.max(dim=-1) on the reference's broadcast tensor, bit
// for bit, in values and indices.
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
constexpr int MAX_ARGMAX_CHUNKS = 512;                                   // argmax path: K <= 512*CHUNK
constexpr int OFFS_BYTES = (MAX_ARGMAX_CHUNKS + 8) * 2;                  // u16 bucket offsets
constexpr int SMEM_BYTES =
    STAGES * STAGE_BYTES + SNAP_BYTES + CIDX_BYTES + OFFS_BYTES + 128 + 1024;

template <int TM_, int TN_, int CHUNK_>
struct Cfg {
  static constexpr int TM = TM_, TN = TN_, CHUNK = CHUNK_;
  static constexpr int TX = BN / TN;       // threads along n
  static constexpr int TY = BM / TM;       // threads along m
  static constexpr int CT = TX * TY;       // compute threads
  static constexpr int CW = CT / 32;       // compute warps
  static constexpr int PRODUCER_WARP = CW;
  static constexpr int THREADS = 32 * (CW + 1);
  static constexpr int OUTS = TM * TN;     // outputs per compute thread
  static constexpr int KT_PER_CHUNK = CHUNK / BK;
  static constexpr int64_t MAX_K = (int64_t)CHUNK * 65535;  // 16-bit chunk index
  static_assert(CT % 32 == 0, "compute threads must fill warps");
  static_assert(OUTS % 4 == 0, "snapshot uses float4");
  static_assert((TX % 8) == 0 && (TY % 8) == 0, "swizzle phase must be per-thread constant");
  static_assert(CHUNK % BK == 0 && KT_PER_CHUNK <= STAGES, "a chunk must fit the ring");
};

using DefaultCfg = Cfg<TP_TMA_TM, TP_TMA_TN, TP_TMA_CHUNK>;

constexpr int MAX_DESTS = 8;   // output copies (the ranks of one NVLink domain)

struct TmaParams {
  int64_t M, N, K;
  const float* bias;
  float* y;
  int64_t ldy;
  int32_t* am;
  int64_t lda;
  float scale;
  // Extra output copies: every (m, n) is also stored at ydst[d][m*ldy + col0 + n]
  // (and adst[d][m*lda + col0 + n]) for d < ndst.  Used by the column-sharded
  // multi-GPU GEMM to write each rank's shard straight into every rank's full
  // output over NVLink (peer pointers), fusing the all-gather into the epilogue.
  float* ydst[MAX_DESTS];
  int32_t* adst[MAX_DESTS];
  int ndst;
  int64_t col0;
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

__device__ __forceinline__ float lds32(uint32_t addr) {
  float v;
  asm volatile("ld.shared.f32 %0, [%1];" : "=f"(v) : "r"(addr));
  return v;
}

__device__ __forceinline__ uint64_t mask_pair(uint64_t v, bool lo_bad, bool hi_bad) {
  const uint64_t NEG = 0xff800000ull;
  if (lo_bad) v = (v & 0xffffffff00000000ull) | NEG;
  if (hi_bad) v = (v & 0x00000000ffffffffull) | (NEG << 32);
  return v;
}

// Barrier among the compute threads only (the producer warp never takes
// part), on an mbarrier so that the wait is bounded like every other wait:
// every compute thread arrives, then waits for the phase to complete.
__device__ __forceinline__ bool compute_sync(uint64_t* bar, uint32_t& phase, int* err) {
  tp_mbar_arrive(bar);
  const bool ok = tp_mbar_wait(bar, phase, err);
  phase ^= 1u;
  return ok;
}

// atomic post-increment of a 16-bit shared counter (through its aligned word)
__device__ __forceinline__ uint32_t atomicAdd_u16(uint16_t* p) {
  uint32_t* w = (uint32_t*)((uintptr_t)p & ~(uintptr_t)3);
  const uint32_t sh = ((uintptr_t)p & 2) ? 16u : 0u;
  const uint32_t old = atomicAdd(w, 1u << sh);
  return (old >> sh) & 0xffffu;
}

// shared-memory address of element (row, k) of a 128 x 32 fp32 tile stored
// with the 128-byte TMA swizzle (16-byte chunk c of row r sits at c ^ (r & 7))
__device__ __forceinline__ uint32_t swz(uint32_t base, int row, int k) {
  return base + (uint32_t)row * 128u + ((((uint32_t)k >> 2) ^ ((uint32_t)row & 7u)) << 4) +
         ((uint32_t)k & 3u) * 4u;
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
  uint16_t* offs = (uint16_t*)(smem + STAGES * STAGE_BYTES + SNAP_BYTES + CIDX_BYTES);
  uint64_t* bars =
      (uint64_t*)(smem + STAGES * STAGE_BYTES + SNAP_BYTES + CIDX_BYTES + OFFS_BYTES);
  uint64_t* full = bars;                 // [STAGES]
  uint64_t* empty = bars + STAGES;       // [STAGES]
  uint64_t* cbar = bars + 2 * STAGES;    // compute-thread barrier

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  // k-tile passes per output tile: the main pass, plus the argmax pass
  constexpr int PASSES = kArgmax ? 2 : 1;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      tp_mbar_init(&full[s], 1);
      tp_mbar_init(&empty[s], C::CW);
    }
    tp_mbar_init(cbar, CT);
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
        for (int pass = 0; pass < PASSES; ++pass) {
          // main pass in k order; the argmax pass chunk by chunk from the last
          // chunk back (its k-tiles were read most recently: likelier L2 hits)
          const int nchunks = (p.k_tiles + C::KT_PER_CHUNK - 1) / C::KT_PER_CHUNK;
          for (int i = 0; i < p.k_tiles; ++i, ++it) {
            int kt = i;
            if (pass == 1) {
              const int c = nchunks - 1 - i / C::KT_PER_CHUNK;   // valid: chunks are full
              kt = c * C::KT_PER_CHUNK + i % C::KT_PER_CHUNK;    // except the last one,
              if (nchunks * C::KT_PER_CHUNK != p.k_tiles) {       // which comes first
                const int last = p.k_tiles - (nchunks - 1) * C::KT_PER_CHUNK;  // its size
                if (i < last) {
                  kt = (nchunks - 1) * C::KT_PER_CHUNK + i;
                } else {
                  const int j = i - last;
                  kt = (nchunks - 2 - j / C::KT_PER_CHUNK) * C::KT_PER_CHUNK + j % C::KT_PER_CHUNK;
                }
              }
            }
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
    }
    return;
  }

  // -------------------------------------------------------------- compute
  const int t = threadIdx.x;  // 0..CT-1
  const int tx = t % TX;
  const int ty = t / TX;
  const uint32_t stage_addr = tp_smem_addr(stage_base);
  const uint32_t snap_addr = tp_smem_addr(snap);
  const uint32_t xsw = (uint32_t)(ty & 7);
  const uint32_t wsw = (uint32_t)(tx & 7);
  const float NEG_INF = -__int_as_float(0x7f800000);
  uint32_t it = 0;
  uint32_t cphase = 0;
  for (int tile = blockIdx.x; tile < p.num_tiles; tile += gridDim.x) {
    int mt, nt;
    tile_coords(tile, p.m_tiles, p.n_tiles, mt, nt);
    const int64_t m0 = (int64_t)mt * BM, n0 = (int64_t)nt * BN;
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

    // ---- main pass: values (+ chunk tracking)
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

    if (!kArgmax) {
      // ---- value-only epilogue
#pragma unroll
      for (int i = 0; i < TM; ++i) {
        const int64_t m = m0 + ty + TY * i;
        if (m >= p.M) continue;
#pragma unroll
        for (int j = 0; j < TN; ++j) {
          const int64_t n = n0 + tx + TX * j;
          if (n >= p.N) continue;
          float v = acc[i][j];
          if (p.bias) v = v + p.bias[n];
          if (p.scale != 1.0f) v = v * p.scale;
          p.y[m * p.ldy + n] = v;
          for (int d = 0; d < p.ndst; ++d) p.ydst[d][m * p.ldy + p.col0 + n] = v;
        }
      }
      continue;
    }

    // ---- argmax pass.  The snapshot holds each output's final max and cid its
    // last-change chunk.  First bucket the tile's outputs by chunk (counting
    // sort in shared memory; the list overwrites cid), then stream the tile's
    // k-tiles through the ring again; each chunk's outputs are shared evenly
    // by the CTA's 4-lane groups, which search 8 k per lane and k-tile with
    // 16-byte shared loads and write the argmax and the final value.
    const int nchunks = (p.k_tiles + C::KT_PER_CHUNK - 1) / C::KT_PER_CHUNK;
    for (int c = t; c <= nchunks; c += CT) offs[c] = 0;
    if (!compute_sync(cbar, cphase, p.err)) return;
#pragma unroll 4
    for (int o = 0; o < C::OUTS; ++o) {                   // count per chunk (in offs[c+1])
      const bool valid = (m0 + ty + TY * (o / TN) < p.M) && (n0 + tx + TX * (o % TN) < p.N);
      if (valid) atomicAdd_u16(&offs[cid[o * CT + t] + 1]);
    }
    if (!compute_sync(cbar, cphase, p.err)) return;
    if (warp == 0) {                              // prefix sum: offs[c] = start of chunk c
      uint32_t carry = 0;
      for (int base = 0; base <= nchunks; base += 32) {
        const int c = base + lane;
        uint32_t v = c <= nchunks ? offs[c] : 0u;
#pragma unroll
        for (int d = 1; d < 32; d <<= 1) {
          const uint32_t up = __shfl_up_sync(0xffffffffu, v, d);
          if (lane >= d) v += up;
        }
        if (c <= nchunks) offs[c] = (uint16_t)(v + carry);
        carry += __shfl_sync(0xffffffffu, v, 31);
      }
    }
    {
      // my outputs' chunk ids, two per register (0xFFFF: not an output); read
      // before the barrier, because the list below overwrites cid
      uint32_t cr[C::OUTS / 2];
#pragma unroll
      for (int q = 0; q < C::OUTS / 2; ++q) {
        uint32_t v[2];
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const int o = 2 * q + h;
          const bool valid = (m0 + ty + TY * (o / TN) < p.M) && (n0 + tx + TX * (o % TN) < p.N);
          v[h] = valid ? (uint32_t)cid[o * CT + t] : 0xFFFFu;
        }
        cr[q] = v[0] | (v[1] << 16);
      }
      if (!compute_sync(cbar, cphase, p.err)) return;
      // scatter: the counter of each chunk walks from its start to its end, so
      // afterwards offs[c] is the end of chunk c (= start of chunk c+1)
#pragma unroll
      for (int q = 0; q < C::OUTS / 2; ++q) {
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const uint32_t c = h ? (cr[q] >> 16) : (cr[q] & 0xffffu);
          if (c != 0xFFFFu) {
            const uint32_t pos = atomicAdd_u16(&offs[c]);
            cid[pos] = (uint16_t)((2 * q + h) * CT + t);   // list entry: output slot
          }
        }
      }
    }
    if (!compute_sync(cbar, cphase, p.err)) return;

    // 4 lanes per output: lane gl covers k = 8*gl .. 8*gl+7 of each k-tile.
    // The stages of a chunk are held only for the shared loads and compares:
    // the items' metadata is fetched before the chunk's wait, and the group
    // reductions and global stores happen after the stages are released.
    const int g = lane >> 2, gl = lane & 3;
    const int group = warp * 8 + g;                  // 0 .. 8*CW-1
    constexpr int NGROUPS = 8 * C::CW;
    constexpr int R = 1;                             // rounds prepared per chunk
    for (int c = nchunks - 1; c >= 0; --c) {
      const int kt0 = c * C::KT_PER_CHUNK;
      const int nkt = min(C::KT_PER_CHUNK, p.k_tiles - kt0);
      const int kbase = kt0 * BK, kmax = (int)p.K;
      const int lo = c > 0 ? offs[c - 1] : 0, hi = offs[c];
      for (int base0 = lo; base0 < hi; base0 += R * NGROUPS) {   // warp-uniform
        bool active[R];
        int mr[R], nr[R];
        float tv[R];
#pragma unroll
        for (int r = 0; r < R; ++r) {
          const int item = base0 + r * NGROUPS + group;
          active[r] = item < hi;
          const int slot = active[r] ? cid[item] : 0;
          const int o = slot / CT, tl = slot % CT;
          mr[r] = tl / TX + TY * (o / TN);
          nr[r] = tl % TX + TX * (o % TN);
          tv[r] = lds32(snap_addr + ((uint32_t)((o >> 2) * CT + tl) * 4u + (o & 3)) * 4u);
        }
        const bool last_batch = base0 + R * NGROUPS >= hi;
        if (base0 == lo) {
          for (int u = 0; u < nkt; ++u) {
            const uint32_t s = (it + u) % STAGES;
            if (!tp_mbar_wait(&full[s], ((it + u) / STAGES) & 1u, p.err)) return;
          }
        }
        int best[R];
#pragma unroll
        for (int r = 0; r < R; ++r) {
          best[r] = 1 << 30;
          const bool tnan = tv[r] != tv[r];
#pragma unroll
          for (int u = 0; u < C::KT_PER_CHUNK; ++u) {
#pragma unroll
            for (int h = 0; h < 2; ++h) {
              if (u < nkt) {
                const uint32_t xb = stage_addr + ((it + u) % STAGES) * STAGE_BYTES;
                const uint32_t q = (uint32_t)(2 * gl + h);       // 16-byte chunk of the row
                uint64_t xv0, xv1, wv0, wv1;
                lds128(xb + (uint32_t)mr[r] * 128u + ((q ^ ((uint32_t)mr[r] & 7u)) << 4), xv0, xv1);
                lds128(xb + TILE_BYTES + (uint32_t)nr[r] * 128u +
                           ((q ^ ((uint32_t)nr[r] & 7u)) << 4),
                       wv0, wv1);
                const float sum[4] = {
                    __uint_as_float((uint32_t)xv0) + __uint_as_float((uint32_t)wv0),
                    __uint_as_float((uint32_t)(xv0 >> 32)) + __uint_as_float((uint32_t)(wv0 >> 32)),
                    __uint_as_float((uint32_t)xv1) + __uint_as_float((uint32_t)wv1),
                    __uint_as_float((uint32_t)(xv1 >> 32)) + __uint_as_float((uint32_t)(wv1 >> 32))};
                const int kl = u * BK + 4 * (int)q;               // chunk-local k of sum[0]
#pragma unroll
                for (int e = 3; e >= 0; --e) {
                  const bool hit = (kbase + kl + e < kmax) &&
                                   (tnan ? (sum[e] != sum[e]) : (sum[e] == tv[r]));
                  if (hit) best[r] = min(best[r], kl + e);
                }
              }
            }
          }
        }
        if (last_batch) {                             // release the chunk's stages
          __syncwarp();
          if (lane == 0)
            for (int u = 0; u < nkt; ++u) tp_mbar_arrive(&empty[(it + u) % STAGES]);
        }
#pragma unroll
        for (int r = 0; r < R; ++r) {
          int b = min(best[r], __shfl_xor_sync(0xffffffffu, best[r], 1));
          b = min(b, __shfl_xor_sync(0xffffffffu, b, 2));
          if (active[r] && gl == 0) {
            const int64_t m = m0 + mr[r], n = n0 + nr[r];
            const int32_t k = b < (1 << 30) ? kbase + b : kbase;
            p.am[m * p.lda + n] = k;
            float v = tv[r];
            if (p.bias) v = v + p.bias[n];
            if (p.scale != 1.0f) v = v * p.scale;
            p.y[m * p.ldy + n] = v;
            for (int d = 0; d < p.ndst; ++d) {
              p.ydst[d][m * p.ldy + p.col0 + n] = v;
              p.adst[d][m * p.lda + p.col0 + n] = k;
            }
          }
        }
      }
      if (lo == hi) {                                 // an empty chunk still holds stages
        for (int u = 0; u < nkt; ++u) {
          const uint32_t s = (it + u) % STAGES;
          if (!tp_mbar_wait(&full[s], ((it + u) / STAGES) & 1u, p.err)) return;
        }
        __syncwarp();
        if (lane == 0)
          for (int u = 0; u < nkt; ++u) tp_mbar_arrive(&empty[(it + u) % STAGES]);
      }
      it += nkt;
    }
    if (!compute_sync(cbar, cphase, p.err)) return;   // the list (in cid) is read until here
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
  if (p.am && ceil_div(p.K, DefaultCfg::CHUNK) > MAX_ARGMAX_CHUNKS) return false;
  if (p.M < BM || p.N < BN || p.K < 2 * BK || p.K > DefaultCfg::MAX_K) return false;
  if ((p.sx_m % 4) != 0 || (p.sw_n % 4) != 0) return false;
  if (!aligned16(p.x) || !aligned16(p.w)) return false;
  if (p.M > (int64_t)INT32_MAX || p.N > (int64_t)INT32_MAX) return false;
  const int64_t tiles = ceil_div(p.M, BM) * ceil_div(p.N, BN);
  return tiles >= 16 && tiles < (int64_t)INT32_MAX;
}

int launch_maxplus_fwd_tma(const StridedMaxPlus& p, cudaStream_t stream) {
  return launch_maxplus_fwd_tma_dests(p, nullptr, nullptr, 0, 0, stream);
}

int launch_maxplus_fwd_tma_dests(const StridedMaxPlus& p, float* const* ydst,
                                 int32_t* const* adst, int ndst, int64_t col0,
                                 cudaStream_t stream) {
  if (!maxplus_tma_eligible(p)) return TP_ERR_UNSUPPORTED;
  if (ndst < 0 || ndst > MAX_DESTS) return TP_ERR_TOO_LARGE;
  CUtensorMap xmap, wmap;
  if (!make_map(&xmap, (const float*)p.x, p.M, p.K, p.sx_m)) return TP_ERR_UNSUPPORTED;
  if (!make_map(&wmap, (const float*)p.w, p.N, p.K, p.sw_n)) return TP_ERR_UNSUPPORTED;
  TmaParams tp_;
  tp_.M = p.M;
  tp_.N = p.N;
  tp_.K = p.K;
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
  tp_.ndst = ndst;
  tp_.col0 = col0;
  for (int d = 0; d < MAX_DESTS; ++d) {
    tp_.ydst[d] = d < ndst ? ydst[d] : nullptr;
    tp_.adst[d] = (d < ndst && adst) ? adst[d] : nullptr;
  }
  if (p.am) return launch_cfg<DefaultCfg, true>(xmap, wmap, tp_, stream);
  return launch_cfg<DefaultCfg, false>(xmap, wmap, tp_, stream);
}

}  // namespace tp
