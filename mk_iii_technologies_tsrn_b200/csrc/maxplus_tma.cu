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
//   TMA loads       128x32 fp32 x/w tiles (128-byte swizzle, no multicast)
//                   into a full/empty mbarrier ring.  The value-only kernel
//                   has a producer warp and 4 stages; the argmax kernel lets
//                   its thread 0 issue the loads, uses 3 stages (more L1 for
//                   the search below) and adds a search warpgroup.
//
// Exact argmax without per-term index tracking.  The running max only grows,
// so the lowest k attaining the final max lies in the LAST CHUNK-wide k-range
// in which the accumulator changed.  At each chunk boundary the compute
// threads compare their accumulators with a snapshot kept in shared memory
// (bitwise, so NaN counts once) and record the chunk index (16-bit, shared
// memory).  At the end of a tile each thread stores its outputs' raw maxima
// in y and their chunk indices in argmax.  While the compute warps run the
// CTA's NEXT tile, a dedicated search warpgroup (one thread per tile column)
// walks the previous tile's outputs 8 k at a time, the next unit's x and w
// quads loaded (through L1/L2) while the current one is tested: the first k
// of the chunk whose sum equals the output's max (or is NaN when the max is
// NaN) is its argmax; then the final y (bias, scale) and the argmax are
// stored.  Two mbarrier pairs hand tiles over (compute -> search: raw maxima
// stored; search -> compute: tile searched, so that a barrier phase is never
// overtaken).  The compute warps search the CTA's last tile themselves after
// their main loop.  The result equals torch.max(dim=-1) on the reference's
// broadcast tensor, bit for bit, in values and indices.
//
// Every mbarrier wait is bounded (common.cuh); a timeout records a device
// error and the kernel returns.
#include <algorithm>
#include <atomic>
#include <mutex>

#include "maxplus_internal.cuh"

namespace tp {

namespace {

#ifndef TP_TMA_TM
#define TP_TMA_TM 4
#endif
#ifndef TP_TMA_TN
#define TP_TMA_TN 8
#endif
#ifndef TP_TMA_SEARCH
#define TP_TMA_SEARCH 128
#endif
// fp32 argmax kernel: TMA ring depth, and whether a dedicated producer warp
// (rather than compute thread 0, inline) issues the loads
#ifndef TP_TMA_ARGMAX_STAGES
#define TP_TMA_ARGMAX_STAGES 3
#endif
#ifndef TP_TMA_ARGMAX_PRODUCER
#define TP_TMA_ARGMAX_PRODUCER 0
#endif
#ifndef TP_TMA_CHUNK
#define TP_TMA_CHUNK 64
#endif
#ifndef TP_TMA_QUNROLL
#define TP_TMA_QUNROLL 8
#endif
// search warpgroup: packed-add units in two alternating buffers (1) or the
// scalar units with a one-deep prefetch (0)
#ifndef TP_TMA_LEAN_SEARCH
#define TP_TMA_LEAN_SEARCH 0
#endif

constexpr int QUNROLL = TP_TMA_QUNROLL;
constexpr int BM = 128;
constexpr int BN = 128;
constexpr int BK = 32;           // fp32 per TMA row: 128 bytes (one swizzle atom)
// Ring depth: the value-only kernel keeps 4 stages; the argmax kernel uses 3,
// which leaves more of the SM's L1 to the argmax search's global loads (the
// search re-reads x and w row chunks that neighbouring outputs share).
template <bool kArgmax>
constexpr int stages() { return kArgmax ? TP_TMA_ARGMAX_STAGES : 4; }
constexpr int TILE_BYTES = BM * BK * 4;                                  // 16 KB
constexpr int STAGE_BYTES = 2 * TILE_BYTES;
constexpr int SNAP_BYTES = BM * BN * 4;                                  // 64 KB
constexpr int CIDX_BYTES = BM * BN * 2;                                  // 32 KB
template <bool kArgmax>
constexpr int smem_bytes() {
  return stages<kArgmax>() * STAGE_BYTES + (kArgmax ? SNAP_BYTES + CIDX_BYTES : 0) + 128 + 1024;
}

template <int TM_, int TN_, int CHUNK_>
struct Cfg {
  static constexpr int TM = TM_, TN = TN_, CHUNK = CHUNK_;
  static constexpr int TX = BN / TN;       // threads along n
  static constexpr int TY = BM / TM;       // threads along m
  static constexpr int CT = TX * TY;       // compute threads
  static constexpr int CW = CT / 32;       // compute warps
  static constexpr int PRODUCER_WARP = CW;           // value-only kernel: a TMA warp
  static constexpr int THREADS = 32 * (CW + 1);
  // The bf16x2 argmax kernel has no producer warp (its thread 0 issues the TMA
  // loads): 16 warps leave 128 registers per thread, room for the search's loads.
  template <bool kArgmax>
  static constexpr int threads() { return kArgmax ? CT : THREADS; }
  // The fp32 argmax kernel adds a search warpgroup (thread 0 still issues the
  // loads): 20 warps at 96 registers each.  (Moving 32 registers per thread
  // from the search warpgroup to the compute warps with setmaxnreg gained
  // 0.7% at K = 8192 but lost 5% at K = 4096, where the slower search falls
  // behind the shorter tiles.)
  static constexpr int SEARCH_THREADS = TP_TMA_SEARCH;   // a divisor of BN, multiple of 32
  template <bool kArgmax>
  static constexpr int threads32() {
    return kArgmax ? CT + SEARCH_THREADS + (TP_TMA_ARGMAX_PRODUCER ? 32 : 0) : THREADS;
  }
  // the argmax kernel's producer warp (when it has one) follows the search warps
  static constexpr int ARGMAX_PRODUCER_WARP = (CT + SEARCH_THREADS) / 32;
  static constexpr int OUTS = TM * TN;     // outputs per compute thread
  static constexpr int KT_PER_CHUNK = CHUNK / BK;
  static constexpr int64_t MAX_K = (int64_t)CHUNK * 65535;  // 16-bit chunk index
  static_assert(CT % 32 == 0, "compute threads must fill warps");
  static_assert(OUTS % 4 == 0, "snapshot uses float4");
  static_assert((TX % 8) == 0 && (TY % 8) == 0, "swizzle phase must be per-thread constant");
  static_assert(CHUNK % BK == 0 && CHUNK % 8 == 0, "chunks are whole k-tiles and search units");
};

using DefaultCfg = Cfg<TP_TMA_TM, TP_TMA_TN, TP_TMA_CHUNK>;
// argmax problems with K <= TP_TMA_SMALLK_MAX use narrower chunks
#ifndef TP_TMA_SMALLK_CHUNK
#define TP_TMA_SMALLK_CHUNK 32
#endif
#ifndef TP_TMA_SMALLK_MAX
#define TP_TMA_SMALLK_MAX 4096
#endif
using SmallKCfg = Cfg<TP_TMA_TM, TP_TMA_TN, TP_TMA_SMALLK_CHUNK>;

constexpr int MAX_DESTS = 8;   // output copies (the ranks of one NVLink domain)

struct TmaParams {
  int64_t M, N, K;
  const float* x;   // the operands again, for the argmax search's global loads
  int64_t ldx;
  const float* w;
  int64_t ldw;
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
  LfAct act;   // value-only epilogue activation (mode -1: none)
  // Stream-K schedule (fp32 kernel; sk = 0: each CTA takes whole tiles
  // blockIdx.x, +gridDim.x, ...).  With sk, the first sk_dp waves stay whole
  // tiles (CTA c: tiles c, c+grid, ...; a wave of neighbouring tiles shares
  // the x/W panels in L2) and the remaining tiles' 64-k chunks form one
  // sequence of sk_units = tiles * sk_cpt units split evenly over the CTAs
  // (at least one tile's chunks each), so a tile may be shared by two CTAs:
  // the later one computes its tail chunks first and leaves partial maxima
  // (and last-change chunks) in slot cta-1; the earlier one computes the head
  // chunks last, merges and finishes the tile.
  // sk = 2 (k-aligned split): the sk_rem remaining tiles are cut into sk_split
  // pieces of k_tiles / sk_split k-tiles (whole 64-k chunks); piece q (of
  // sk_split * sk_rem) is piece q / sk_rem of remaining tile q % sk_rem and
  // goes to CTA q % grid, so that the CTAs walk the same k range at the same
  // time (L2 sharing as in whole-tile waves).  Pieces below the last leave
  // their partials in slot (tile - first) * (sk_split - 1) + piece; the last
  // piece comes in a later round, waits for them and merges in k order.
  int sk;
  int sk_cpt;
  int sk_dp;
  int64_t sk_units;
  int sk_split;
  int sk_rem;
  float* sk_max;       // [slots][OUTS * CT] partial maxima, thread-major
  int32_t* sk_cid;     // [slots][OUTS * CT] their last-change chunks (argmax)
  unsigned* sk_flag;   // [slots] 1 once the slot holds its partials
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
// Two terms: their sums (each one IEEE-rounded fp32 add) folded into acc by a
// 3-input NaN-propagating max.  TP_TMA_SCALAR_ADD selects two scalar adds
// instead of one packed add.f32x2 (same results; a different issue mix).
#ifndef TP_TMA_SCALAR_ADD
#define TP_TMA_SCALAR_ADD 0
#endif
__device__ __forceinline__ void mp_pair(float& acc, uint64_t xa, uint64_t wb) {
#if TP_TMA_SCALAR_ADD
  asm("{\n\t.reg .f32 x0, x1, w0, w1, lo, hi;\n\t"
      "mov.b64 {x0, x1}, %1;\n\tmov.b64 {w0, w1}, %2;\n\t"
      "add.rn.f32 lo, x0, w0;\n\tadd.rn.f32 hi, x1, w1;\n\t"
      "max.NaN.f32 %0, %0, lo, hi;\n\t}"
      : "+f"(acc)
      : "l"(xa), "l"(wb));
#else
  asm("{\n\t.reg .b64 s;\n\t.reg .f32 lo, hi;\n\t"
      "add.rn.f32x2 s, %1, %2;\n\t"
      "mov.b64 {lo, hi}, s;\n\t"
      "max.NaN.f32 %0, %0, lo, hi;\n\t}"
      : "+f"(acc)
      : "l"(xa), "l"(wb));
#endif
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

// Argmax search helpers.  A unit is 8 consecutive k of one output: x and w
// quads (a0 a1, b0 b1).  unit_first_hit returns the first k of the unit whose
// sum equals the output's max tv (tv NaN: whose sum is NaN), or kBestNone.
// The common case -- the unit does not hold the max -- costs eight adds, a
// three-instruction max tree and one compare.
constexpr int kBestNone = 0x7fffffff;

__device__ __forceinline__ int unit_first_hit(float tv, int k, int K, const float4& a0,
                                              const float4& a1, const float4& b0,
                                              const float4& b1) {
  const float s[8] = {a0.x + b0.x, a0.y + b0.y, a0.z + b0.z, a0.w + b0.w,
                      a1.x + b1.x, a1.y + b1.y, a1.z + b1.z, a1.w + b1.w};
  float mx = tp_max3_nan(s[0], s[1], s[2]);
  mx = tp_max3_nan(mx, s[3], s[4]);
  mx = tp_max3_nan(mx, s[5], s[6]);
  mx = tp_max_nan(mx, s[7]);
  const bool tnan = tv != tv;
  int best = kBestNone;
  if (tnan ? (mx != mx) : (mx == tv)) {
#pragma unroll
    for (int e = 7; e >= 0; --e) {
      const bool hit = (k + e < K) && (tnan ? (s[e] != s[e]) : (s[e] == tv));
      if (hit) best = k + e;
    }
  }
  return best;
}

// x and w quads of the unit at xr / wr (its first k is k); k >= K reads as
// x = -inf, w = 0, so that it can never hold the max
__device__ __forceinline__ void load_unit(const float* xr, const float* wr, int k, int K,
                                          float4& a0, float4& a1, float4& b0, float4& b1) {
  if (k + 8 <= K) {
    a0 = __ldg(reinterpret_cast<const float4*>(xr));
    a1 = __ldg(reinterpret_cast<const float4*>(xr + 4));
    b0 = __ldg(reinterpret_cast<const float4*>(wr));
    b1 = __ldg(reinterpret_cast<const float4*>(wr + 4));
  } else {
    const float NEG_INF = -__int_as_float(0x7f800000);
    float xv[8], wv[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const bool in = k + e < K;
      xv[e] = in ? __ldg(xr + e) : NEG_INF;
      wv[e] = in ? __ldg(wr + e) : 0.0f;
    }
    a0 = make_float4(xv[0], xv[1], xv[2], xv[3]);
    a1 = make_float4(xv[4], xv[5], xv[6], xv[7]);
    b0 = make_float4(wv[0], wv[1], wv[2], wv[3]);
    b1 = make_float4(wv[4], wv[5], wv[6], wv[7]);
  }
}

// Packed form of a search unit: x and w of 8 consecutive k as four 64-bit
// pairs each; the eight sums come from four add.rn.f32x2 (each sum one
// rounded fp32 add, as in the main loop) and the max tree from three 3-input
// and one 2-input NaN-propagating max.
struct Unit8 {
  ulonglong2 x0, x1, w0, w1;
};

__device__ __forceinline__ void load_unit8(const float* xr, const float* wr, int k, int K,
                                           Unit8& u) {
  if (k + 8 <= K) {
    u.x0 = __ldg(reinterpret_cast<const ulonglong2*>(xr));
    u.x1 = __ldg(reinterpret_cast<const ulonglong2*>(xr + 4));
    u.w0 = __ldg(reinterpret_cast<const ulonglong2*>(wr));
    u.w1 = __ldg(reinterpret_cast<const ulonglong2*>(wr + 4));
  } else {
    float4 a0, a1, b0, b1;
    load_unit(xr, wr, k, K, a0, a1, b0, b1);
    u.x0 = *reinterpret_cast<const ulonglong2*>(&a0);
    u.x1 = *reinterpret_cast<const ulonglong2*>(&a1);
    u.w0 = *reinterpret_cast<const ulonglong2*>(&b0);
    u.w1 = *reinterpret_cast<const ulonglong2*>(&b1);
  }
}

__device__ __forceinline__ void add2_split(uint64_t a, uint64_t b, float& lo, float& hi) {
  asm("{\n\t.reg .b64 s;\n\tadd.rn.f32x2 s, %2, %3;\n\tmov.b64 {%0, %1}, s;\n\t}"
      : "=f"(lo), "=f"(hi)
      : "l"(a), "l"(b));
}

__device__ __forceinline__ int unit8_first_hit(float tv, bool tnan, int k, int K, const Unit8& u) {
  float s[8];
  add2_split(u.x0.x, u.w0.x, s[0], s[1]);
  add2_split(u.x0.y, u.w0.y, s[2], s[3]);
  add2_split(u.x1.x, u.w1.x, s[4], s[5]);
  add2_split(u.x1.y, u.w1.y, s[6], s[7]);
  float mx = tp_max3_nan(s[0], s[1], s[2]);
  mx = tp_max3_nan(mx, s[3], s[4]);
  mx = tp_max3_nan(mx, s[5], s[6]);
  mx = tp_max_nan(mx, s[7]);
  int best = kBestNone;
  if (tnan ? (mx != mx) : (mx == tv)) {
#pragma unroll
    for (int e = 7; e >= 0; --e) {
      const bool hit = (k + e < K) && (tnan ? (s[e] != s[e]) : (s[e] == tv));
      if (hit) best = k + e;
    }
  }
  return best;
}

// first k of the chunk [kc, kc + 8 * UPO) of output row xr / wr whose sum
// equals tv (NaN: is NaN), or kBestNone; two units in flight, alternating
// between two buffers (no register copies)
template <int UPO>
__device__ __forceinline__ int search_chunk(const float* xr, const float* wr, int kc, int K,
                                            float tv) {
  const bool tnan = tv != tv;
  Unit8 A, B;
  load_unit8(xr, wr, kc, K, A);
#pragma unroll
  for (int u = 0; u < UPO; u += 2) {
    if (u + 1 < UPO) load_unit8(xr + 8 * (u + 1), wr + 8 * (u + 1), kc + 8 * (u + 1), K, B);
    int best = unit8_first_hit(tv, tnan, kc + 8 * u, K, A);
    if (best != kBestNone) return best;
    if (u + 1 < UPO) {
      if (u + 2 < UPO) load_unit8(xr + 8 * (u + 2), wr + 8 * (u + 2), kc + 8 * (u + 2), K, A);
      best = unit8_first_hit(tv, tnan, kc + 8 * (u + 1), K, B);
      if (best != kBestNone) return best;
    }
  }
  return kBestNone;
}

// final value (bias, scale) and argmax of output (m, n), to y/argmax and to
// every extra destination
__device__ __forceinline__ void store_output(const TmaParams& p, int64_t m, int64_t n, float tv,
                                             int32_t k) {
  p.am[m * p.lda + n] = k;
  float v = tv;
  if (p.bias) v = v + p.bias[n];
  if (p.scale != 1.0f) v = v * p.scale;
  p.y[m * p.ldy + n] = v;
  for (int d = 0; d < p.ndst; ++d) {
    p.ydst[d][m * p.ldy + p.col0 + n] = v;
    p.adst[d][m * p.lda + p.col0 + n] = k;
  }
}

template <class C, bool kArgmax>
__global__ void __launch_bounds__(C::template threads32<kArgmax>(), 1)
    maxplus_tma_kernel(const __grid_constant__ CUtensorMap xmap,
                       const __grid_constant__ CUtensorMap wmap, const TmaParams p) {
  constexpr int TM = C::TM, TN = C::TN, TX = C::TX, TY = C::TY, CT = C::CT;
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  // 1024-byte alignment for the 128-byte swizzle pattern
  unsigned char* smem =
      (unsigned char*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  constexpr int STAGES = stages<kArgmax>();
  unsigned char* stage_base = smem;                                  // STAGES x (x tile, w tile)
  float4* snap = (float4*)(smem + STAGES * STAGE_BYTES);             // [OUTS/4][CT]
  uint16_t* cid = (uint16_t*)(smem + STAGES * STAGE_BYTES + SNAP_BYTES);  // [OUTS][CT]
  uint64_t* bars = (uint64_t*)(smem + STAGES * STAGE_BYTES +
                               (kArgmax ? SNAP_BYTES + CIDX_BYTES : 0));
  uint64_t* full = bars;                 // [STAGES]
  uint64_t* empty = bars + STAGES;       // [STAGES]
  uint64_t* tile_ready = bars + 2 * STAGES;        // [2] argmax: raw maxima stored
  uint64_t* search_done = bars + 2 * STAGES + 2;   // [2] argmax: tile searched
  uint64_t* cbar = bars + 2 * STAGES + 4;          // compute threads only (stream-K)
  constexpr int SEARCH_WARPS = C::SEARCH_THREADS / 32;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  __shared__ float lf_sm[64];
  __shared__ int sk_ok;
  // This CTA's schedule: whole tiles blockIdx.x, +gridDim.x, ... (all of
  // them, or the first sch_dp under stream-K) then, under stream-K, the
  // contiguous range [sch_g0, sch_g1) of the global k-tile order (tile
  // major), cut at chunk boundaries.  Kept in shared memory: it is read
  // between segments, not in the main loop.
  __shared__ long long sch_g0, sch_g1;
  __shared__ unsigned sch_nseg, sch_total_kt, sch_dp;
  if (!kArgmax && p.act.mode >= 0) lf_stage(p.act, lf_sm);

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      tp_mbar_init(&full[s], 1);
      tp_mbar_init(&empty[s], C::CW);
    }
    if (kArgmax) {
      for (int b = 0; b < 2; ++b) {
        tp_mbar_init(&tile_ready[b], C::CW);
        tp_mbar_init(&search_done[b], SEARCH_WARPS);
      }
    }
    tp_mbar_init(cbar, CT);
    tp_fence_mbar_init();
    const int cta = (int)blockIdx.x, G = (int)gridDim.x;
    if (kArgmax && p.sk == 2) {
      const int64_t total = (int64_t)p.sk_split * p.sk_rem;
      const unsigned np = cta < total ? (unsigned)((total - cta + G - 1) / G) : 0u;
      sch_g0 = sch_g1 = 0;
      sch_dp = (unsigned)p.sk_dp;
      sch_nseg = (unsigned)p.sk_dp + np;
      sch_total_kt = (unsigned)p.sk_dp * (unsigned)p.k_tiles +
                     np * (unsigned)(p.k_tiles / p.sk_split);
    } else if (p.sk) {
      const int64_t first = (int64_t)p.sk_dp * G;       // first stream-K tile
      auto g_of = [&](int64_t u) -> int64_t {
        return (first + u / p.sk_cpt) * p.k_tiles +
               min((u % p.sk_cpt) * (int64_t)C::KT_PER_CHUNK, (int64_t)p.k_tiles);
      };
      const int64_t g0 = g_of(p.sk_units * cta / G), g1 = g_of(p.sk_units * (cta + 1) / G);
      sch_g0 = g0;
      sch_g1 = g1;
      sch_dp = (unsigned)p.sk_dp;
      sch_nseg = (unsigned)p.sk_dp +
                 (g1 > g0 ? (unsigned)((g1 - 1) / p.k_tiles - g0 / p.k_tiles + 1) : 0u);
      sch_total_kt = (unsigned)p.sk_dp * (unsigned)p.k_tiles + (unsigned)(g1 - g0);
    } else {
      const unsigned my_tiles = (unsigned)((p.num_tiles - cta + G - 1) / G);
      sch_g0 = sch_g1 = 0;
      sch_dp = my_tiles;
      sch_nseg = my_tiles;
      sch_total_kt = my_tiles * (unsigned)p.k_tiles;
    }
  }
  __syncthreads();

  // Segment i of the schedule is tile `tile`, k-tiles [kb, ke); k-tile j of
  // the CTA goes to stage j % STAGES once the stage's previous k-tile is
  // released.
  const int cta = (int)blockIdx.x, G = (int)gridDim.x;
  // (the schedule sizes sch_nseg / sch_total_kt are read from shared memory
  // where used, so that they do not occupy registers across the main loop)
  auto seg = [&](uint32_t i, int& tile, int& kb, int& ke) {
    const uint32_t dp = sch_dp;
    if (kArgmax && i >= dp && p.sk == 2) {
      const int64_t q = (int64_t)cta + (int64_t)(i - dp) * G;
      const int L = p.k_tiles / p.sk_split;
      tile = (int)((int64_t)dp * G + q % p.sk_rem);
      kb = (int)(q / p.sk_rem) * L;
      ke = kb + L;
    } else if (i >= dp) {
      const int64_t g0 = sch_g0, g1 = sch_g1;
      tile = (int)(g0 / p.k_tiles) + (int)(i - dp);
      const int64_t base = (int64_t)tile * p.k_tiles;
      kb = (int)max(g0 - base, (int64_t)0);
      ke = (int)min(g1 - base, (int64_t)p.k_tiles);
    } else {
      tile = cta + (int)i * G;
      kb = 0;
      ke = p.k_tiles;
    }
  };
  // segments the search warpgroup takes: finished here (not a stream-K tail
  // piece, not a split piece below the last) and not the CTA's last segment
  // (the compute warps search that one)
  auto searched = [&](uint32_t i, int kb, int ke) {
    const bool finished = (kArgmax && p.sk == 2) ? ke == p.k_tiles : !(p.sk && kb > 0);
    return finished && i + 1 < sch_nseg;
  };
  auto produce = [&](uint32_t j) -> bool {
    int tile, kt;
    const uint32_t dp_kt = sch_dp * (uint32_t)p.k_tiles;
    if (kArgmax && j >= dp_kt && p.sk == 2) {
      const uint32_t L = (uint32_t)(p.k_tiles / p.sk_split);
      const int64_t q = (int64_t)cta + (int64_t)((j - dp_kt) / L) * G;
      tile = (int)((int64_t)sch_dp * G + q % p.sk_rem);
      kt = (int)((q / p.sk_rem) * L + (j - dp_kt) % L);
    } else if (j >= dp_kt) {
      const int64_t g = sch_g0 + (j - dp_kt);
      tile = (int)(g / p.k_tiles);
      kt = (int)(g % p.k_tiles);
    } else {
      tile = cta + (int)(j / (uint32_t)p.k_tiles) * G;
      kt = (int)(j % (uint32_t)p.k_tiles);
    }
    int mt, nt;
    tile_coords(tile, p.m_tiles, p.n_tiles, mt, nt);
    const uint32_t s = j % STAGES;
    const uint32_t ph = (j / STAGES) & 1u;
    if (!tp_mbar_wait(&empty[s], ph ^ 1u, p.err)) return false;
    unsigned char* dst = stage_base + s * STAGE_BYTES;
    tp_mbar_arrive_expect_tx(&full[s], STAGE_BYTES);
    tp_tma_load_2d(dst, &xmap, kt * BK, mt * BM, &full[s]);
    tp_tma_load_2d(dst + TILE_BYTES, &wmap, kt * BK, nt * BN, &full[s]);
    return true;
  };

  if constexpr (!kArgmax) {
    if (warp == C::PRODUCER_WARP) {
      // ---------------------------------------------------------- producer
      if (lane == 0) {
        tp_prefetch_tensormap(&xmap);
        tp_prefetch_tensormap(&wmap);
        for (uint32_t j = 0; j < sch_total_kt; ++j)
          if (!produce(j)) return;
      }
      return;
    }
  } else if (TP_TMA_ARGMAX_PRODUCER) {
    if (warp == C::ARGMAX_PRODUCER_WARP) {
      if (lane == 0) {
        tp_prefetch_tensormap(&xmap);
        tp_prefetch_tensormap(&wmap);
        for (uint32_t j = 0; j < sch_total_kt; ++j)
          if (!produce(j)) return;
      }
      return;
    }
  } else {
    // thread 0 fills all but one stage now, then one stage per k-tile: at
    // k-tile j it refills the stage of k-tile j-1 with k-tile j+STAGES-1
    if (threadIdx.x == 0) {
      tp_prefetch_tensormap(&xmap);
      tp_prefetch_tensormap(&wmap);
      for (uint32_t j = 0; j < STAGES - 1 && j < sch_total_kt; ++j)
        if (!produce(j)) return;
    }
  }

  constexpr int UPO = C::CHUNK / 8;            // 8-k search units per output
  const int Kc = (int)p.K;
  const int Mc = (int)p.M, Nc = (int)p.N;

  if constexpr (kArgmax) {
    if (threadIdx.x >= CT && threadIdx.x < CT + C::SEARCH_THREADS) {
      // ---------------------------------------------------- search warpgroup
      // This CTA's finished tiles but the last, each once its raw maxima and
      // chunks are stored; thread sid walks column sid of the tile row by
      // row (a warp covers 32 adjacent columns: coalesced y / argmax loads).
      const int sid = (int)threadIdx.x - CT;
      uint32_t h = 0;               // tiles taken so far
      for (uint32_t i = 0; i < sch_nseg; ++i) {
        int tile, kb, ke;
        seg(i, tile, kb, ke);
        if (!searched(i, kb, ke)) continue;
        const bool ok = tp_mbar_wait(&tile_ready[h & 1], (h >> 1) & 1u, p.err);
        if (!__all_sync(0xffffffffu, ok)) return;
        int mt, nt;
        tile_coords(tile, p.m_tiles, p.n_tiles, mt, nt);
        const int m0 = mt * BM;
        // SEARCH_THREADS may be below BN: thread sid walks columns sid,
        // sid + SEARCH_THREADS, ... of the tile
        for (int col = sid; col < BN; col += C::SEARCH_THREADS) {
        const int n = nt * BN + col;
        const int rows = n < Nc ? min(BM, Mc - m0) : 0;
        const float* wrow = p.w + (int64_t)n * p.ldw;
        float tv = 0.0f;
        int kc = 0;
        if (rows > 0) {
          tv = p.y[(int64_t)m0 * p.ldy + n];
          kc = p.am[(int64_t)m0 * p.lda + n] * C::CHUNK;
        }
        for (int r = 0; r < rows; ++r) {
          const int m = m0 + r;
          float ntv = 0.0f;
          int nkc = 0;
          if (r + 1 < rows) {
            ntv = p.y[(int64_t)(m + 1) * p.ldy + n];
            nkc = p.am[(int64_t)(m + 1) * p.lda + n] * C::CHUNK;
          }
          const float* xr = p.x + (int64_t)m * p.ldx + kc;
          const float* wr = wrow + kc;
#if TP_TMA_LEAN_SEARCH
          const int best = search_chunk<UPO>(xr, wr, kc, Kc, tv);
#else
          float4 a0, a1, b0, b1;
          load_unit(xr, wr, kc, Kc, a0, a1, b0, b1);
          int best = kBestNone;
          for (int u = 0; u < UPO; ++u) {
            float4 c0 = a0, c1 = a1, d0 = b0, d1 = b1;
            if (u + 1 < UPO)
              load_unit(xr + 8 * (u + 1), wr + 8 * (u + 1), kc + 8 * (u + 1), Kc, c0, c1, d0, d1);
            best = unit_first_hit(tv, kc + 8 * u, Kc, a0, a1, b0, b1);
            if (best != kBestNone) break;
            a0 = c0;
            a1 = c1;
            b0 = d0;
            b1 = d1;
          }
#endif
          store_output(p, m, n, tv, best != kBestNone ? best : kc);
          tv = ntv;
          kc = nkc;
        }
        }
        __syncwarp();
        if (lane == 0) tp_mbar_arrive(&search_done[h & 1]);
        ++h;
      }
      return;
    }
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
  uint32_t h = 0;               // tiles handed to the search warpgroup so far
  // barrier of the compute threads (producer / search warps take no part),
  // waits bounded like every other
  uint32_t cphase = 0;
  auto compute_sync = [&]() -> bool {
    tp_mbar_arrive(cbar);
    const bool ok = tp_mbar_wait(cbar, cphase, p.err);
    cphase ^= 1u;
    return ok;
  };
  for (uint32_t si = 0; si < sch_nseg; ++si) {
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
    int kb0, ke0;
    {
      int tile0;
      seg(si, tile0, kb0, ke0);
    }
    for (int kt = kb0; kt < ke0; ++kt, ++it) {
      const uint32_t s = it % STAGES;
      const uint32_t ph = (it / STAGES) & 1u;
      if (kArgmax && !TP_TMA_ARGMAX_PRODUCER && threadIdx.x == 0 &&
          it + STAGES - 1 < sch_total_kt)
        if (!produce(it + STAGES - 1)) return;
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

    // this segment again (tile origin, k range), after the main loop
    int tile, kb, ke, mt, nt;
    seg(si, tile, kb, ke);
    tile_coords(tile, p.m_tiles, p.n_tiles, mt, nt);
    const int64_t m0 = (int64_t)mt * BM, n0 = (int64_t)nt * BN;
    if (kArgmax && p.sk == 2 && ke < p.k_tiles) {
      // ---- k-aligned split, a piece below the last: partial maxima (+ chunks)
      // to its slot, then release the slot's flag
      const int64_t slot = (int64_t)(tile - (int)sch_dp * G) * (p.sk_split - 1) +
                           kb / (p.k_tiles / p.sk_split);
      float* wm = p.sk_max + slot * C::OUTS * CT;
#pragma unroll
      for (int o = 0; o < C::OUTS; ++o) wm[o * CT + t] = acc[o / TN][o % TN];
      if (kArgmax) {
        int32_t* wc = p.sk_cid + slot * C::OUTS * CT;
#pragma unroll
        for (int o = 0; o < C::OUTS; ++o) wc[o * CT + t] = (int32_t)cid[o * CT + t];
      }
      if (!compute_sync()) return;
      if (t == 0) {
        __threadfence();
        asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(p.sk_flag + slot), "r"(1u)
                     : "memory");
      }
      continue;
    }
    if (kArgmax && p.sk == 2 && kb > 0) {
      // ---- k-aligned split, the last piece (pieces below ran in earlier
      // rounds): wait for their flags, then fold the partials in k order and
      // this piece last -- a higher piece wins only with a strictly larger max
      // (or a NaN where the lower has none), so ties keep the lowest k.
      const int64_t slot0 = (int64_t)(tile - (int)sch_dp * G) * (p.sk_split - 1);
      if (t == 0) {
        int ok = 1;
        for (int sp = 0; ok && sp < p.sk_split - 1; ++sp)
          ok = tp_flag_wait(p.sk_flag + slot0 + sp, p.err) ? 1 : 0;
        sk_ok = ok;
      }
      if (!compute_sync() || !sk_ok) return;
      const float* wm = p.sk_max + slot0 * C::OUTS * CT;
      const int32_t* wc = kArgmax ? p.sk_cid + slot0 * C::OUTS * CT : nullptr;
#pragma unroll
      for (int o = 0; o < C::OUTS; ++o) {
        float v = __ldcg(wm + o * CT + t);
        int32_t c = kArgmax ? __ldcg(wc + o * CT + t) : 0;
        for (int sp = 1; sp < p.sk_split - 1; ++sp) {
          const int64_t off = (int64_t)sp * C::OUTS * CT + o * CT + t;
          const float h = __ldcg(wm + off);
          if constexpr (!kArgmax) {
            v = tp_max_nan(v, h);
          } else if (v == v && (h != h || h > v)) {
            v = h;
            c = __ldcg(wc + off);
          }
        }
        float& a = acc[o / TN][o % TN];
        if constexpr (!kArgmax) {
          a = tp_max_nan(v, a);
        } else if (v == v && (a != a || a > v)) {
          // this piece's own maximum stands
        } else {
          a = v;
          cid[o * CT + t] = (uint16_t)c;
        }
      }
    }
    if (p.sk == 1 && kb > 0) {
      // ---- stream-K tail piece: partial maxima (+ chunks) to slot cta-1,
      // then release the flag for the CTA that finishes this tile
      float* wm = p.sk_max + (int64_t)(cta - 1) * C::OUTS * CT;
#pragma unroll
      for (int o = 0; o < C::OUTS; ++o) wm[o * CT + t] = acc[o / TN][o % TN];
      if (kArgmax) {
        int32_t* wc = p.sk_cid + (int64_t)(cta - 1) * C::OUTS * CT;
#pragma unroll
        for (int o = 0; o < C::OUTS; ++o) wc[o * CT + t] = (int32_t)cid[o * CT + t];
      }
      if (!compute_sync()) return;
      if (t == 0) {
        __threadfence();
        asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(p.sk_flag + cta - 1), "r"(1u)
                     : "memory");
      }
      continue;
    }
    if (p.sk == 1 && ke < p.k_tiles) {
      // ---- stream-K head piece (the CTA's last segment): wait for the tail's
      // partials, then merge.  The tail wins only with a strictly larger max
      // (or a NaN where the head has none): ties keep the head's lower k.
      if (t == 0) sk_ok = tp_flag_wait(p.sk_flag + cta, p.err) ? 1 : 0;
      if (!compute_sync() || !sk_ok) return;
      const float* wm = p.sk_max + (int64_t)cta * C::OUTS * CT;
      const int32_t* wc = p.sk_cid + (int64_t)cta * C::OUTS * CT;
#pragma unroll
      for (int o = 0; o < C::OUTS; ++o) {
        float& a = acc[o / TN][o % TN];
        const float tv = __ldcg(wm + o * CT + t);
        if constexpr (!kArgmax) {
          a = tp_max_nan(a, tv);
        } else if (a == a && (tv != tv || tv > a)) {
          a = tv;
          cid[o * CT + t] = (uint16_t)__ldcg(wc + o * CT + t);
        }
      }
    }

    if constexpr (!kArgmax) {
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
          if (p.act.mode >= 0) v = lf_apply(p.act, lf_sm, n, v);
          p.y[m * p.ldy + n] = v;
          for (int d = 0; d < p.ndst; ++d) p.ydst[d][m * p.ldy + p.col0 + n] = v;
        }
      }
    } else {
      // ---- argmax: store this tile's raw maxima and chunks, then hand the
      // tile to the search warpgroup (all but the CTA's last segment)
#pragma unroll
      for (int i = 0; i < TM; ++i) {
        const int64_t m = m0 + ty + TY * i;
        if (m >= p.M) continue;
#pragma unroll
        for (int j = 0; j < TN; ++j) {
          const int64_t n = n0 + tx + TX * j;
          if (n >= p.N) continue;
          p.y[m * p.ldy + n] = acc[i][j];
          p.am[m * p.lda + n] = (int32_t)cid[(i * TN + j) * CT + t];
        }
      }
      if (searched(si, kb, ke)) {
        __syncwarp();
        bool ok = true;
        // the search of the tile handed two before has ended before this
        // barrier's next phase
        if (lane == 0 && h >= 2)
          ok = tp_mbar_wait(&search_done[h & 1], ((h - 2) >> 1) & 1u, p.err);
        if (!__shfl_sync(0xffffffffu, ok, 0)) return;
        if (lane == 0) tp_mbar_arrive(&tile_ready[h & 1]);
        ++h;
      }
    }
  }

  // (a stream-K range spans at least one tile's chunks, so its last segment
  // is never a tail piece: it is finished here)
  if (kArgmax && sch_nseg > 0) {
    // ---- the CTA's last tile, searched by the compute warps after their
    // main loop; each output's units are tested four at a time
    int tile, kb, ke, mt, nt;
    seg(sch_nseg - 1, tile, kb, ke);
    tile_coords(tile, p.m_tiles, p.n_tiles, mt, nt);
    const int64_t last_m0 = (int64_t)mt * BM, last_n0 = (int64_t)nt * BN;
    for (int o = 0; o < C::OUTS; ++o) {
      const int m = (int)last_m0 + ty + TY * (o / TN), n = (int)last_n0 + tx + TX * (o % TN);
      if (m >= Mc || n >= Nc) continue;
      const float tv = p.y[(int64_t)m * p.ldy + n];
      const int kc = p.am[(int64_t)m * p.lda + n] * C::CHUNK;
      const float* xr = p.x + (int64_t)m * p.ldx + kc;
      const float* wr = p.w + (int64_t)n * p.ldw + kc;
      int best = kBestNone;
      for (int j0 = 0; j0 < UPO && best == kBestNone; j0 += 4) {
        float4 dx[4][2], dw[4][2];
#pragma unroll
        for (int u = 0; u < 4; ++u)
          if (j0 + u < UPO)
            load_unit(xr + 8 * (j0 + u), wr + 8 * (j0 + u), kc + 8 * (j0 + u), Kc, dx[u][0],
                      dx[u][1], dw[u][0], dw[u][1]);
#pragma unroll
        for (int u = 0; u < 4; ++u)
          if (j0 + u < UPO && best == kBestNone)
            best = unit_first_hit(tv, kc + 8 * (j0 + u), Kc, dx[u][0], dx[u][1], dw[u][0],
                                  dw[u][1]);
      }
      store_output(p, m, n, tv, best != kBestNone ? best : kc);
    }
  }
}

// ===========================================================================
// Packed bf16x2 kernel (TP_DTYPE_BF16_ARITH): the reference expression on bf16
// tensors, where every sum x + w is rounded to bf16.  Same CTA structure as the
// fp32 kernel; a k-tile is 128 x 64 bf16 (128-byte rows).  Each accumulator
// register holds two bf16 lanes: the running max over the even and over the
// odd k of one output.  Per two terms: one add.rn.bf16x2 (both sums rounded to
// bf16, ties to even -- the rounding torch applies) and one max.NaN.bf16x2.
// Chunk tracking compares the max of the two lanes (16-bit snapshot); the
// deferred argmax search tests 32-k units (packed adds and a max tree) and
// compares in fp32 (bf16 values widen exactly).
// ===========================================================================
constexpr int BK16 = 64;                         // bf16 per TMA row (128 bytes)
constexpr int CHUNK16 = 128;                     // argmax chunk: two k-tiles
constexpr int KT_PER_CHUNK16 = CHUNK16 / BK16;
constexpr int SNAP16_BYTES = BM * BN * 2;        // 16-bit combined maxima
constexpr uint32_t BF2_NEG_INF = 0xff80ff80u;
constexpr int64_t MAX_K16 = (int64_t)CHUNK16 * 65535;

template <bool kArgmax>
constexpr int smem_bytes16() {
  return stages<kArgmax>() * STAGE_BYTES + (kArgmax ? SNAP16_BYTES + CIDX_BYTES : 0) + 128 + 1024;
}

__device__ __forceinline__ uint32_t bf2_add(uint32_t a, uint32_t b) {
  uint32_t r;
  asm("add.rn.bf16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  return r;
}
__device__ __forceinline__ uint32_t bf2_max(uint32_t a, uint32_t b) {
  uint32_t r;
  asm("max.NaN.bf16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  return r;
}
// max.NaN of the two lanes, as a bf16 bit pattern
__device__ __forceinline__ uint32_t bf2_lanes_max(uint32_t a) {
  uint16_t r;
  asm("{\n\t.reg .b16 lo, hi;\n\tmov.b32 {lo, hi}, %1;\n\tmax.NaN.bf16 %0, lo, hi;\n\t}"
      : "=h"(r)
      : "r"(a));
  return (uint32_t)r;
}
__device__ __forceinline__ float bf_bits_to_f32(uint32_t b16) { return __uint_as_float(b16 << 16); }

__device__ __forceinline__ uint4 lds128u4(uint32_t addr) {
  uint4 v;
  asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "r"(addr));
  return v;
}

// lanes of a bf16x2 word at k (lo) and k+1 (hi): those at or past K become -inf
__device__ __forceinline__ uint32_t bf2_mask(uint32_t v, int64_t k, int64_t K) {
  if (k >= K) v = (v & 0xffff0000u) | 0xff80u;
  if (k + 1 >= K) v = (v & 0x0000ffffu) | 0xff800000u;
  return v;
}

// 32 bf16 terms of one output: x and w row chunks (8 words each) at k
struct Unit16 {
  uint4 a[4], b[4];
};

__device__ __forceinline__ void load_unit16(const uint16_t* xr, const uint16_t* wr, int k, int K,
                                            Unit16& u) {
  if (k + 32 <= K) {
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      u.a[c] = __ldg(reinterpret_cast<const uint4*>(xr) + c);
      u.b[c] = __ldg(reinterpret_cast<const uint4*>(wr) + c);
    }
  } else {
    uint32_t aw[16], bw[16];
#pragma unroll
    for (int e = 0; e < 16; ++e) {
      const int k0 = k + 2 * e;
      const uint32_t xl = k0 < K ? __ldg(xr + 2 * e) : 0xff80u;
      const uint32_t xh = k0 + 1 < K ? __ldg(xr + 2 * e + 1) : 0xff80u;
      const uint32_t wl = k0 < K ? __ldg(wr + 2 * e) : 0u;
      const uint32_t wh = k0 + 1 < K ? __ldg(wr + 2 * e + 1) : 0u;
      aw[e] = xl | (xh << 16);
      bw[e] = wl | (wh << 16);
    }
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      u.a[c] = make_uint4(aw[4 * c], aw[4 * c + 1], aw[4 * c + 2], aw[4 * c + 3]);
      u.b[c] = make_uint4(bw[4 * c], bw[4 * c + 1], bw[4 * c + 2], bw[4 * c + 3]);
    }
  }
}

// first k of the unit whose bf16 sum equals tv (NaN: is NaN), or kBestNone
__device__ __forceinline__ int unit_first_hit16(float tv, int k, int K, const Unit16& u) {
  uint32_t s[16];
#pragma unroll
  for (int c = 0; c < 4; ++c) {
    s[4 * c + 0] = bf2_add(u.a[c].x, u.b[c].x);
    s[4 * c + 1] = bf2_add(u.a[c].y, u.b[c].y);
    s[4 * c + 2] = bf2_add(u.a[c].z, u.b[c].z);
    s[4 * c + 3] = bf2_add(u.a[c].w, u.b[c].w);
  }
  uint32_t m = s[0];
#pragma unroll
  for (int e = 1; e < 16; ++e) m = bf2_max(m, s[e]);
  const float mx = bf_bits_to_f32(bf2_lanes_max(m));
  const bool tnan = tv != tv;
  int best = kBestNone;
  if (tnan ? (mx != mx) : (mx == tv)) {
#pragma unroll
    for (int e = 31; e >= 0; --e) {
      const uint32_t w = s[e >> 1];
      const float se = bf_bits_to_f32((e & 1) ? (w >> 16) : (w & 0xffffu));
      const bool hit = (k + e < K) && (tnan ? (se != se) : (se == tv));
      if (hit) best = k + e;
    }
  }
  return best;
}

template <class C, bool kArgmax>
__global__ void __launch_bounds__(C::template threads<kArgmax>(), 1)
    maxplus_tma_bf16_kernel(const __grid_constant__ CUtensorMap xmap,
                            const __grid_constant__ CUtensorMap wmap, const TmaParams p) {
  constexpr int TM = C::TM, TN = C::TN, TX = C::TX, TY = C::TY, CT = C::CT;
  constexpr int OUTS = TM * TN;
  static_assert(OUTS % 8 == 0, "16-bit snapshots are moved eight at a time");
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* smem =
      (unsigned char*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  constexpr int STAGES = stages<kArgmax>();
  unsigned char* stage_base = smem;
  uint4* snap = (uint4*)(smem + STAGES * STAGE_BYTES);                      // [OUTS/8][CT]
  uint16_t* cid = (uint16_t*)(smem + STAGES * STAGE_BYTES + SNAP16_BYTES);  // [OUTS][CT]
  uint64_t* bars = (uint64_t*)(smem + STAGES * STAGE_BYTES +
                               (kArgmax ? SNAP16_BYTES + CIDX_BYTES : 0));
  uint64_t* full = bars;
  uint64_t* empty = bars + STAGES;
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      tp_mbar_init(&full[s], 1);
      tp_mbar_init(&empty[s], C::CW);
    }
    tp_fence_mbar_init();
  }
  __syncthreads();

  const uint32_t my_tiles = (uint32_t)((p.num_tiles - (int)blockIdx.x + (int)gridDim.x - 1) /
                                       (int)gridDim.x);
  const uint32_t total_kt = my_tiles * (uint32_t)p.k_tiles;
  auto produce = [&](uint32_t j) -> bool {
    const int tile = (int)blockIdx.x + (int)(j / (uint32_t)p.k_tiles) * (int)gridDim.x;
    const int kt = (int)(j % (uint32_t)p.k_tiles);
    int mt, nt;
    tile_coords(tile, p.m_tiles, p.n_tiles, mt, nt);
    const uint32_t s = j % STAGES;
    const uint32_t ph = (j / STAGES) & 1u;
    if (!tp_mbar_wait(&empty[s], ph ^ 1u, p.err)) return false;
    unsigned char* dst = stage_base + s * STAGE_BYTES;
    tp_mbar_arrive_expect_tx(&full[s], STAGE_BYTES);
    tp_tma_load_2d(dst, &xmap, kt * BK16, mt * BM, &full[s]);
    tp_tma_load_2d(dst + TILE_BYTES, &wmap, kt * BK16, nt * BN, &full[s]);
    return true;
  };

  if constexpr (!kArgmax) {
    if (warp == C::PRODUCER_WARP) {
      if (lane == 0) {
        tp_prefetch_tensormap(&xmap);
        tp_prefetch_tensormap(&wmap);
        for (uint32_t j = 0; j < total_kt; ++j)
          if (!produce(j)) return;
      }
      return;
    }
  } else {
    if (threadIdx.x == 0) {
      tp_prefetch_tensormap(&xmap);
      tp_prefetch_tensormap(&wmap);
      for (uint32_t j = 0; j < STAGES - 1 && j < total_kt; ++j)
        if (!produce(j)) return;
    }
  }

  // -------------------------------------------------------------- compute
  const int t = threadIdx.x;
  const int tx = t % TX;
  const int ty = t / TX;
  const uint32_t stage_addr = tp_smem_addr(stage_base);
  const uint32_t xsw = (uint32_t)(ty & 7);
  const uint32_t wsw = (uint32_t)(tx & 7);
  const uint16_t* xg = reinterpret_cast<const uint16_t*>(p.x);
  const uint16_t* wg = reinterpret_cast<const uint16_t*>(p.w);

  // deferred argmax search (as in the fp32 kernel), 32-k units
  constexpr int UPO = CHUNK16 / 32;
  constexpr int UNITS = OUTS * UPO;
  const int Kc = (int)p.K;
  const int Mc = (int)p.M, Nc = (int)p.N;
  int s_u = UNITS + 1;
  int s_m0 = 0, s_n0 = 0;
  float s_tv = 0.0f, s_ntv = 0.0f;
  int s_kc = 0, s_nkc = 0;
  int s_best = kBestNone;
  const uint16_t* s_xp = nullptr;
  const uint16_t* s_wp = nullptr;
  Unit16 su;
  const int steps = kArgmax ? (UNITS + p.k_tiles - 1) / p.k_tiles : 0;

  auto prefetch = [&](int o) {
    const int m = s_m0 + ty + TY * (o / TN), n = s_n0 + tx + TX * (o % TN);
    if (o < OUTS && m < Mc && n < Nc) {
      s_ntv = p.y[(int64_t)m * p.ldy + n];
      s_nkc = p.am[(int64_t)m * p.lda + n] * CHUNK16;
    }
  };
  auto step = [&]() {
    if (s_u >= 1 && s_u <= UNITS) {
      const int pu = s_u - 1;
      if (s_xp != nullptr) {
        if (s_best == kBestNone) s_best = unit_first_hit16(s_tv, s_kc + 32 * (pu % UPO), Kc, su);
        if (pu % UPO == UPO - 1) {
          const int o = pu / UPO;
          store_output(p, s_m0 + ty + TY * (o / TN), s_n0 + tx + TX * (o % TN), s_tv,
                       s_best != kBestNone ? s_best : s_kc);
        }
      }
    }
    if (s_u < UNITS) {
      if (s_u % UPO == 0) {
        const int o = s_u / UPO;
        const int m = s_m0 + ty + TY * (o / TN), n = s_n0 + tx + TX * (o % TN);
        s_tv = s_ntv;
        s_kc = s_nkc;
        s_best = kBestNone;
        if (m < Mc && n < Nc) {
          s_xp = xg + (int64_t)m * p.ldx + s_kc;
          s_wp = wg + (int64_t)n * p.ldw + s_kc;
        } else {
          s_xp = s_wp = nullptr;
        }
        prefetch(o + 1);
      }
      // once a unit held the output's max, its remaining units are not loaded
      if (s_xp != nullptr && s_best == kBestNone) {
        load_unit16(s_xp, s_wp, s_kc + 32 * (s_u % UPO), Kc, su);
        s_xp += 32;
        s_wp += 32;
      }
    }
    if (s_u <= UNITS) ++s_u;
  };

  uint32_t it = 0;
  for (int tile = blockIdx.x; tile < p.num_tiles; tile += gridDim.x) {
    int mt, nt;
    tile_coords(tile, p.m_tiles, p.n_tiles, mt, nt);
    const int64_t m0 = (int64_t)mt * BM, n0 = (int64_t)nt * BN;
    uint32_t acc[TM][TN];
#pragma unroll
    for (int i = 0; i < TM; ++i)
#pragma unroll
      for (int j = 0; j < TN; ++j) acc[i][j] = BF2_NEG_INF;
    if (kArgmax) {
#pragma unroll
      for (int q = 0; q < OUTS / 8; ++q)
        snap[q * CT + t] = make_uint4(0xff80ff80u, 0xff80ff80u, 0xff80ff80u, 0xff80ff80u);
#pragma unroll
      for (int o = 0; o < OUTS; ++o) cid[o * CT + t] = 0;
    }

    for (int kt = 0; kt < p.k_tiles; ++kt, ++it) {
      const uint32_t s = it % STAGES;
      const uint32_t ph = (it / STAGES) & 1u;
      if (kArgmax && threadIdx.x == 0 && it + STAGES - 1 < total_kt)
        if (!produce(it + STAGES - 1)) return;
      if (!tp_mbar_wait(&full[s], ph, p.err)) return;
      if (kArgmax)
        for (int r = 0; r < steps; ++r) step();
      const uint32_t xbase = stage_addr + s * STAGE_BYTES;
      const uint32_t wbase = xbase + TILE_BYTES;
      const int64_t k0 = (int64_t)kt * BK16;
      const bool tail = k0 + BK16 > p.K;
#pragma unroll 4
      for (int q = 0; q < 8; ++q) {
        uint32_t xw[TM][4];
#pragma unroll
        for (int i = 0; i < TM; ++i) {
          const uint4 v =
              lds128u4(xbase + (uint32_t)(ty + TY * i) * 128u + (((uint32_t)q ^ xsw) << 4));
          xw[i][0] = v.x;
          xw[i][1] = v.y;
          xw[i][2] = v.z;
          xw[i][3] = v.w;
        }
        if (tail) {
          const int64_t kq = k0 + 8 * q;
#pragma unroll
          for (int i = 0; i < TM; ++i)
#pragma unroll
            for (int c = 0; c < 4; ++c) xw[i][c] = bf2_mask(xw[i][c], kq + 2 * c, p.K);
        }
#pragma unroll
        for (int j = 0; j < TN; ++j) {
          const uint4 wv =
              lds128u4(wbase + (uint32_t)(tx + TX * j) * 128u + (((uint32_t)q ^ wsw) << 4));
#pragma unroll
          for (int i = 0; i < TM; ++i) {
            acc[i][j] = bf2_max(acc[i][j], bf2_add(xw[i][0], wv.x));
            acc[i][j] = bf2_max(acc[i][j], bf2_add(xw[i][1], wv.y));
            acc[i][j] = bf2_max(acc[i][j], bf2_add(xw[i][2], wv.z));
            acc[i][j] = bf2_max(acc[i][j], bf2_add(xw[i][3], wv.w));
          }
        }
      }
      __syncwarp();
      if (lane == 0) tp_mbar_arrive(&empty[s]);

      if (kArgmax && (((kt + 1) % KT_PER_CHUNK16) == 0 || kt == p.k_tiles - 1)) {
        const uint16_t chunk = (uint16_t)(kt / KT_PER_CHUNK16);
#pragma unroll
        for (int q = 0; q < OUTS / 8; ++q) {
          const uint4 sv = snap[q * CT + t];
          const uint32_t sw[4] = {sv.x, sv.y, sv.z, sv.w};
          uint32_t nw[4];
#pragma unroll
          for (int h = 0; h < 4; ++h) {
            const int o0 = 8 * q + 2 * h, o1 = o0 + 1;
            const uint32_t m0v = bf2_lanes_max(acc[o0 / TN][o0 % TN]);
            const uint32_t m1v = bf2_lanes_max(acc[o1 / TN][o1 % TN]);
            if (m0v != (sw[h] & 0xffffu)) cid[o0 * CT + t] = chunk;
            if (m1v != (sw[h] >> 16)) cid[o1 * CT + t] = chunk;
            nw[h] = m0v | (m1v << 16);
          }
          snap[q * CT + t] = make_uint4(nw[0], nw[1], nw[2], nw[3]);
        }
      }
    }

    if constexpr (!kArgmax) {
#pragma unroll
      for (int i = 0; i < TM; ++i) {
        const int64_t m = m0 + ty + TY * i;
        if (m >= p.M) continue;
#pragma unroll
        for (int j = 0; j < TN; ++j) {
          const int64_t n = n0 + tx + TX * j;
          if (n >= p.N) continue;
          float v = bf_bits_to_f32(bf2_lanes_max(acc[i][j]));
          if (p.bias) v = v + p.bias[n];
          if (p.scale != 1.0f) v = v * p.scale;
          p.y[m * p.ldy + n] = v;
          for (int d = 0; d < p.ndst; ++d) p.ydst[d][m * p.ldy + p.col0 + n] = v;
        }
      }
    } else {
      while (s_u <= UNITS) step();
#pragma unroll
      for (int i = 0; i < TM; ++i) {
        const int64_t m = m0 + ty + TY * i;
        if (m >= p.M) continue;
#pragma unroll
        for (int j = 0; j < TN; ++j) {
          const int64_t n = n0 + tx + TX * j;
          if (n >= p.N) continue;
          p.y[m * p.ldy + n] = bf_bits_to_f32(bf2_lanes_max(acc[i][j]));
          p.am[m * p.lda + n] = (int32_t)cid[(i * TN + j) * CT + t];
        }
      }
      s_m0 = (int)m0;
      s_n0 = (int)n0;
      s_u = 0;
      prefetch(0);
    }
  }

  if (s_u == 0) {
    // drain: the CTA's last tile, two units in flight at a time
    for (int o = 0; o < OUTS; ++o) {
      const int m = s_m0 + ty + TY * (o / TN), n = s_n0 + tx + TX * (o % TN);
      if (m >= Mc || n >= Nc) continue;
      const float tv = p.y[(int64_t)m * p.ldy + n];
      const int kc = p.am[(int64_t)m * p.lda + n] * CHUNK16;
      const uint16_t* xr = xg + (int64_t)m * p.ldx + kc;
      const uint16_t* wr = wg + (int64_t)n * p.ldw + kc;
      int best = kBestNone;
      for (int j0 = 0; j0 < UPO && best == kBestNone; j0 += 2) {
        Unit16 d0, d1;
        load_unit16(xr + 32 * j0, wr + 32 * j0, kc + 32 * j0, Kc, d0);
        if (j0 + 1 < UPO) load_unit16(xr + 32 * (j0 + 1), wr + 32 * (j0 + 1), kc + 32 * (j0 + 1), Kc, d1);
        best = unit_first_hit16(tv, kc + 32 * j0, Kc, d0);
        if (best == kBestNone && j0 + 1 < UPO)
          best = unit_first_hit16(tv, kc + 32 * (j0 + 1), Kc, d1);
      }
      store_output(p, m, n, tv, best != kBestNone ? best : kc);
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

bool make_map16(CUtensorMap* map, const void* base, int64_t rows, int64_t K, int64_t ld) {
  EncodeTiledFn enc = encode_tiled();
  if (!enc) return false;
  cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)ld * 2};
  cuuint32_t box[2] = {BK16, 128};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims,
                   strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

template <class C, bool kArgmax>
int launch_cfg16(const CUtensorMap& xmap, const CUtensorMap& wmap, const TmaParams& tp_,
                 cudaStream_t stream) {
  cudaError_t e = cudaFuncSetAttribute(maxplus_tma_bf16_kernel<C, kArgmax>,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       smem_bytes16<kArgmax>());
  if (e != cudaSuccess) return (int)e;
  int grid = num_sms();
  if (grid > tp_.num_tiles) grid = tp_.num_tiles;
  maxplus_tma_bf16_kernel<C, kArgmax>
      <<<grid, C::template threads<kArgmax>(), smem_bytes16<kArgmax>(), stream>>>(xmap, wmap, tp_);
  return launch_status();
}

template <class C, bool kArgmax>
int launch_cfg(const CUtensorMap& xmap, const CUtensorMap& wmap, const TmaParams& tp_,
               cudaStream_t stream) {
  cudaError_t e = cudaFuncSetAttribute(maxplus_tma_kernel<C, kArgmax>,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       smem_bytes<kArgmax>());
  if (e != cudaSuccess) return (int)e;
  int grid = num_sms();
  if (grid > tp_.num_tiles) grid = tp_.num_tiles;
  maxplus_tma_kernel<C, kArgmax>
      <<<grid, C::template threads32<kArgmax>(), smem_bytes<kArgmax>(), stream>>>(xmap, wmap, tp_);
  return launch_status();
}

}  // namespace

namespace {
std::atomic<int64_t> g_argmax_tma_min_terms{(int64_t)1 << 30};
// 0 off, 1 when it removes a partial last wave, 2 always (even split of
// chunks), 3 always (k-aligned split of tiles when K allows it)
std::atomic<int> g_stream_k{1};

// Stream-ordered workspace for the stream-K partials: a library-owned pool per
// device that keeps its memory (allocation after the first is cheap), so that
// every caller of the forward gets the schedule without passing a buffer.
std::mutex g_sk_pool_mu;
cudaMemPool_t g_sk_pool[64] = {};

cudaMemPool_t sk_pool(int dev) {
  if (dev < 0 || dev >= 64) return nullptr;
  std::lock_guard<std::mutex> lk(g_sk_pool_mu);
  if (g_sk_pool[dev] == nullptr) {
    cudaMemPoolProps props = {};
    props.allocType = cudaMemAllocationTypePinned;
    props.location.type = cudaMemLocationTypeDevice;
    props.location.id = dev;
    cudaMemPool_t pool = nullptr;
    if (cudaMemPoolCreate(&pool, &props) != cudaSuccess) {
      (void)cudaGetLastError();
      return nullptr;
    }
    uint64_t keep = UINT64_MAX;
    (void)cudaMemPoolSetAttribute(pool, cudaMemPoolAttrReleaseThreshold, &keep);
    g_sk_pool[dev] = pool;
  }
  return g_sk_pool[dev];
}
}  // namespace

int set_stream_k(int mode) { return g_stream_k.exchange(mode < 0 ? 0 : (mode > 3 ? 3 : mode)); }

int64_t argmax_tma_min_terms() { return g_argmax_tma_min_terms.load(std::memory_order_relaxed); }

int64_t set_argmax_tma_min_terms(int64_t terms) {
  return g_argmax_tma_min_terms.exchange(terms < 0 ? 0 : terms);
}

bool maxplus_tma_eligible(const StridedMaxPlus& p) {
  if (p.act.mode >= 0 && (p.am || p.dtype != TP_DTYPE_F32)) return false;
  if (p.dtype == TP_DTYPE_BF16_ARITH) {
    // packed bf16x2 kernel: 16-byte aligned bf16 rows
    if (p.B1 * p.B2 != 1) return false;
    if (p.sx_k != 1 || p.sw_k != 1 || p.sy_n != 1) return false;
    if (p.am && p.sa_n != 1) return false;
    if (p.M < BM || p.N < BN || p.K < 2 * BK16 || p.K > MAX_K16) return false;
    if (p.am && p.M * p.N * p.K < argmax_tma_min_terms()) return false;
    if ((p.sx_m % 8) != 0 || (p.sw_n % 8) != 0) return false;
    if (!aligned16(p.x) || !aligned16(p.w)) return false;
    if (p.M > (int64_t)INT32_MAX || p.N > (int64_t)INT32_MAX) return false;
    const int64_t tiles = ceil_div(p.M, BM) * ceil_div(p.N, BN);
    return tiles >= 16 && tiles < (int64_t)INT32_MAX;
  }
  if (p.dtype != TP_DTYPE_F32) return false;
  if (p.B1 * p.B2 != 1) return false;
  if (p.sx_k != 1 || p.sw_k != 1 || p.sy_n != 1) return false;
  if (p.am && p.sa_n != 1) return false;
  if (p.M < BM || p.N < BN || p.K < 2 * BK || p.K > DefaultCfg::MAX_K) return false;
  // With argmax, each CTA searches its last tile after its main loop; below
  // about 2^30 terms that fixed cost (~0.17 ms) outweighs the faster main loop
  // and the per-term generic kernel is quicker (measured: 1024x256x256 0.05 vs
  // 0.22 ms, 8192x256x256 0.19 vs 0.22 ms; 1024^3 0.38 vs 0.36 ms).
  if (p.am && p.M * p.N * p.K < argmax_tma_min_terms()) return false;
  if ((p.sx_m % 4) != 0 || (p.sw_n % 4) != 0) return false;
  if (!aligned16(p.x) || !aligned16(p.w)) return false;
  if (p.M > (int64_t)INT32_MAX || p.N > (int64_t)INT32_MAX) return false;
  const int64_t tiles = ceil_div(p.M, BM) * ceil_div(p.N, BN);
  return tiles >= 16 && tiles < (int64_t)INT32_MAX;
}

// The fp32 schedule (whole tiles / stream-K / k-aligned pieces) and launch
// for one chunk width C.
template <class C>
int launch_fp32_sched(const StridedMaxPlus& p, const CUtensorMap& xmap, const CUtensorMap& wmap,
                      TmaParams tp_, cudaStream_t stream) {
  // Stream-K when the tiles leave the last wave partly idle (every CTA must
  // cover at least one tile's chunks) and K is long (K >= 4096: shorter tiles
  // do not repay the split -- 2048^3 with argmax measured 1.07 ms whole-tile
  // vs 1.17 ms split), unless the stream is being captured (the workspace is
  // allocated on the stream).  With argmax only when the idle share is at
  // least 5% of the run: below it the split tiles cost about what they save
  // (measured: 8192 x 1024 x 8192, 3.46 waves, 5.62 -> 5.27 ms; 8192 x 2048 x
  // 8192, 6.92 waves, 9.72 -> 9.97 ms; value-only gains in both).
  const int grid = std::min(num_sms(), tp_.num_tiles);
  const int mode = g_stream_k.load(std::memory_order_relaxed);
  const int waves = (int)ceil_div(tp_.num_tiles, grid);
  const double idle = (double)(waves * grid - tp_.num_tiles) / ((double)waves * grid);
  bool sk = mode != 0 && tp_.num_tiles >= grid && grid > 1 &&
            (mode >= 2 || (tp_.num_tiles % grid != 0 && p.K >= 4096 &&
                           (!p.am || idle >= 0.05)));
  // The remainder after the whole-tile waves (rem tiles, grid <= rem < 2 grid)
  // as whole tiles (2 rounds), an even split of its chunks (rem / grid
  // tile-times), or tiles cut into S k-aligned pieces of whole 64-k chunks
  // (ceil(S rem / grid) / S).  Forced mode 3 takes the S in {2, 4} with the
  // fewest rounds.  Auto mode, argmax kernel: the cheapest of the three with
  // S = 2, each split charged its measured overhead in tile-times at
  // K = 8192 (even split 0.34: 8192 x 1024 x 8192 took 5.28 ms for an ideal
  // 4.81; halves 0.10: 5.11 ms for 4.97; quarters were dearer still,
  // 2048^2 x 8192 2.95 ms against 2.89 ms whole); value-only: the even split
  // (no measurable overhead).
  const int sk_dp = std::max(0, tp_.num_tiles / grid - 1);
  const int rem = tp_.num_tiles - sk_dp * grid;
  int split = 0;
  if (sk && p.am && mode == 3) {
    double best = 1e30;
    for (int S = 2; S <= 4; S *= 2) {
      if (tp_.k_tiles % (S * C::KT_PER_CHUNK) != 0) continue;
      const double cost = (double)ceil_div((int64_t)S * rem, (int64_t)grid) / S;
      if (cost < best - 1e-9) {
        best = cost;
        split = S;
      }
    }
  } else if (sk && p.am && mode == 1) {
    const double whole = (double)ceil_div(rem, grid);
    const double even = (double)rem / grid + 0.34;
    const double halves = tp_.k_tiles % (2 * C::KT_PER_CHUNK) == 0
                              ? (double)ceil_div((int64_t)2 * rem, (int64_t)grid) / 2 + 0.10
                              : 1e30;
    if (whole <= even && whole <= halves) sk = false;
    else if (halves < even) split = 2;
  }
  void* ws = nullptr;
  if (sk) {
    cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
    int dev = 0;
    cudaMemPool_t pool = nullptr;
    if (cudaStreamIsCapturing(stream, &cap) != cudaSuccess || cap != cudaStreamCaptureStatusNone ||
        cudaGetDevice(&dev) != cudaSuccess || (pool = sk_pool(dev)) == nullptr) {
      (void)cudaGetLastError();
      sk = false;
    } else {
      const size_t slot = (size_t)C::OUTS * C::CT;
      const size_t nslots = split ? (size_t)(split - 1) * rem : (size_t)grid;
      const size_t bytes = nslots * slot * (p.am ? 8 : 4) + nslots * 4 + 256;
      if (cudaMallocFromPoolAsync(&ws, bytes, pool, stream) != cudaSuccess) {
        (void)cudaGetLastError();
        sk = false;
      } else {
        // whole-tile waves for all but the last full wave; stream-K over that
        // wave and the remainder (at least one tile's chunks per CTA)
        tp_.sk = split ? 2 : 1;
        tp_.sk_cpt = (int)ceil_div(tp_.k_tiles, C::KT_PER_CHUNK);
        tp_.sk_dp = sk_dp;
        tp_.sk_units = (int64_t)rem * tp_.sk_cpt;
        tp_.sk_split = split;
        tp_.sk_rem = rem;
        tp_.sk_max = (float*)ws;
        tp_.sk_cid = p.am ? (int32_t*)(tp_.sk_max + nslots * slot) : nullptr;
        tp_.sk_flag = (unsigned*)((char*)ws + nslots * slot * (p.am ? 8 : 4));
        const cudaError_t e = cudaMemsetAsync(tp_.sk_flag, 0, nslots * 4, stream);
        if (e != cudaSuccess) {
          (void)cudaFreeAsync(ws, stream);
          return (int)e;
        }
      }
    }
  }
  const int st = p.am ? launch_cfg<C, true>(xmap, wmap, tp_, stream)
                      : launch_cfg<C, false>(xmap, wmap, tp_, stream);
  if (ws != nullptr) {
    const cudaError_t e = cudaFreeAsync(ws, stream);
    if (st == TP_OK && e != cudaSuccess) return (int)e;
  }
  return st;
}
int launch_maxplus_fwd_tma(const StridedMaxPlus& p, cudaStream_t stream) {
  return launch_maxplus_fwd_tma_dests(p, nullptr, nullptr, 0, 0, stream);
}

int launch_maxplus_fwd_tma_dests(const StridedMaxPlus& p, float* const* ydst,
                                 int32_t* const* adst, int ndst, int64_t col0,
                                 cudaStream_t stream) {
  if (!maxplus_tma_eligible(p)) return TP_ERR_UNSUPPORTED;
  if (ndst < 0 || ndst > MAX_DESTS) return TP_ERR_TOO_LARGE;
  const bool bf16 = p.dtype == TP_DTYPE_BF16_ARITH;
  CUtensorMap xmap, wmap;
  if (bf16) {
    if (!make_map16(&xmap, p.x, p.M, p.K, p.sx_m)) return TP_ERR_UNSUPPORTED;
    if (!make_map16(&wmap, p.w, p.N, p.K, p.sw_n)) return TP_ERR_UNSUPPORTED;
  } else {
    if (!make_map(&xmap, (const float*)p.x, p.M, p.K, p.sx_m)) return TP_ERR_UNSUPPORTED;
    if (!make_map(&wmap, (const float*)p.w, p.N, p.K, p.sw_n)) return TP_ERR_UNSUPPORTED;
  }
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
  tp_.k_tiles = (int)ceil_div(p.K, bf16 ? BK16 : BK);
  tp_.num_tiles = tp_.m_tiles * tp_.n_tiles;
  tp_.err = device_error_ptr();
  tp_.ndst = ndst;
  tp_.col0 = col0;
  tp_.act = p.act;
  for (int d = 0; d < MAX_DESTS; ++d) {
    tp_.ydst[d] = d < ndst ? ydst[d] : nullptr;
    tp_.adst[d] = (d < ndst && adst) ? adst[d] : nullptr;
  }
  tp_.sk = 0;
  tp_.sk_cpt = 0;
  tp_.sk_dp = 0;
  tp_.sk_units = 0;
  tp_.sk_split = 0;
  tp_.sk_rem = 0;
  tp_.sk_max = nullptr;
  tp_.sk_cid = nullptr;
  tp_.sk_flag = nullptr;
  if (bf16) {
    if (p.am) return launch_cfg16<DefaultCfg, true>(xmap, wmap, tp_, stream);
    return launch_cfg16<DefaultCfg, false>(xmap, wmap, tp_, stream);
  }
  // Argmax chunk width: 64-k chunks at K > 4096, 32 below (measured with
  // argmax: 4096^3 5.57 -> 5.05 ms, 2048^3 1.07 -> 0.87 ms with 32; 8192^3
  // 37.5 ms with 64 against 38.1 with 32): the deferred search re-reads one
  // chunk of x and W per output from L2, which matters more when a CTA has
  // few tiles, while narrower chunks cost snapshot compares in the main loop.
  if (p.am && p.K <= TP_TMA_SMALLK_MAX) return launch_fp32_sched<SmallKCfg>(p, xmap, wmap, tp_, stream);
  return launch_fp32_sched<DefaultCfg>(p, xmap, wmap, tp_, stream);
}


}  // namespace tp
