// scan_chunked.cu -- chunk-parallel evaluation of the tropical SSM scan
// (research/tsrn_dml.py:917-980, TropicalSSM) for shapes whose (batch x
// channel) lanes cannot fill the GPU: the sequential kernels of scan.cu run
// one warp per 32 channels of a batch row, so B=2, C=1024 (config 3's batch
// split over 8 GPUs) gives 64 warps for 148 SMs.  Here time is cut into
// chunks of L steps (a multiple of 32) and each (batch, chunk, 4 channels)
// is one thread, so the lanes multiply by T / L.
//
// Forward, bit-exact with the sequential recurrence h_t = (u_t >= a + h_{t-1})
// ? u_t : fl(a + h_{t-1}):
//   1. beta: every chunk runs the recurrence from h = -inf (its own inputs
//      only) and keeps its last state beta_j.
//   2. carry: the state after chunk j from any start h is max(chain_L(h),
//      beta_j), where chain_L is L rounded additions of a (rounding is
//      monotone, so fl(a + max(p, q)) = max(fl(a+p), fl(a+q)) and the carry
//      and the chunk's own winners separate).  Which side wins decides the
//      bits: a carry that never loses gives chain_L(h) exactly, a carry that
//      loses once gives beta_j exactly (from the step it loses, the run
//      equals the chunk's own run).  Runs of chunks compose the same way,
//      (n1, G1) then (n2, G2) -> (n1 + n2, max(chain_n2(G1), G2)), so one
//      block per (b, c) scans its chunks in parallel (warp shuffles, log
//      depth); chain_n is evaluated exactly in a few steps per binade
//      (chain_exact.cuh) after a rounding-error bound has settled most
//      comparisons.  An exact tie at zero (where +0 and -0 differ) sends the
//      lane to a chunk-by-chunk walk that replays the chunk.  The pass writes
//      each chunk's exact starting state.
//   3. output: every chunk reruns the recurrence from its exact starting
//      state and writes h and the win-mask words -- the same bits as the
//      sequential kernel.
// Backward (G_t = g_t + carry_{t+1}; gu_t = win ? G : 0; carry_t = win ? 0 : G):
//   A. summary: every chunk runs its reverse walk from carry 0 and keeps the
//      carry leaving its first step, and whether any input won in it.  A
//      chunk with a winner sends the same carry whatever enters it.
//   B. carry: one thread per (b, c) walks the chunks backwards; a chunk with
//      no winner passes the entering carry through its L rounded adds of g
//      (in order, exact).  gh0 is the carry leaving chunk 0.
//   C. output: every chunk reruns its reverse walk from its exact entering
//      carry (from b, x, h: on the winners pass A recomputed and stored as
//      mask words, one bit per element read instead of b, x and h again)
//      and writes gu -- bit-exact -- and its partial sum of the lost
//      gradients; ga sums the partials (ascending batch, descending chunk),
//      an order that differs from one sequential sum over T: ga agrees with
//      the sequential kernel to rounding, gu and gh0 bit for bit.
//
// Memory: pass 1 reads b, x once and pass 3 reads them again; pass 1 marks
// the lines evict-last in L2 and pass 3 evict-first, so that at the sizes this
// mode exists for (2 x 32 MiB at B=2) the second read comes from L2; the
// backward's passes A and C do the same.  Loads are 128-bit across 4 channels
// (C % 4 == 0 and 16-byte aligned tensors and enough threads; otherwise one
// channel per thread).
#include <math.h>

#include "chain_exact.cuh"
#include "maxplus_internal.cuh"

namespace tp {

namespace {

// rows whose loads are issued together: 8 with four channels per thread
// (128-bit loads), 16 with one channel per thread (keeps ~100 KB of loads in
// flight per SM at 40% occupancy)
template <int V>
constexpr int row_block() { return V == 4 ? 8 : 16; }
constexpr int kPassThreads = 128;   // threads per block of the chunk-parallel passes

struct ChunkArgs {
  int64_t B, T, C;
  int L, nch, nw;                 // chunk length, chunks, mask words per row
  const float* bb;
  const float* xx;                // may be null (u = bb)
  const float* a;
  float h_init;
  const float* h0;                // [B, C] or null
  // forward
  float* h;
  uint32_t* win;                  // [B, nw, C] or null
  // backward
  const float* gh;
  const float* hin;               // forward states (recompute path)
  const uint32_t* win_in;         // or the forward's mask
  float* gu;
  float* ga;
  float* gh0;
  // workspace planes, [B][nch][C] each
  float* beta;
  float* hs;
  float* cout;
  float* cin;
  float* gap;
  int* tflag;                      // 1: no input won in the chunk
  int* err;                        // device status block (bounded waits)
  uint32_t* wmask;                 // backward from b, x, h: pass A's winners [B, nw, C]
};

template <int V>
__device__ __forceinline__ void ldv(float (&d)[V], const float* p) {
  if constexpr (V == 4) {
    const float4 t = __ldg(reinterpret_cast<const float4*>(p));
    d[0] = t.x; d[1] = t.y; d[2] = t.z; d[3] = t.w;
  } else {
    d[0] = __ldg(p);
  }
}

// L2 eviction policies: the first pass over an input keeps its lines in L2
// (evict_last) for the second pass, which reads them for the last time
// (evict_first); at the sizes this mode serves the inputs fit in L2
__device__ __forceinline__ uint64_t l2_policy(bool keep) {
  uint64_t pol;
  if (keep) asm("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(pol));
  else asm("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
  return pol;
}

template <int V>
__device__ __forceinline__ void ldv_pol(float (&d)[V], const float* p, uint64_t pol) {
  if constexpr (V == 4) {
    asm("ld.global.nc.L2::cache_hint.v4.f32 {%0, %1, %2, %3}, [%4], %5;"
        : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
        : "l"(p), "l"(pol));
  } else {
    asm("ld.global.nc.L2::cache_hint.f32 %0, [%1], %2;" : "=f"(d[0]) : "l"(p), "l"(pol));
  }
}

template <int V>
__device__ __forceinline__ void ldw_pol(uint32_t (&d)[V], const uint32_t* p, uint64_t pol) {
  if constexpr (V == 4) {
    asm("ld.global.nc.L2::cache_hint.v4.u32 {%0, %1, %2, %3}, [%4], %5;"
        : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
        : "l"(p), "l"(pol));
  } else {
    asm("ld.global.nc.L2::cache_hint.u32 %0, [%1], %2;" : "=r"(d[0]) : "l"(p), "l"(pol));
  }
}

template <int V>
__device__ __forceinline__ void stv(float* p, const float (&s)[V]) {
  if constexpr (V == 4) {
    *reinterpret_cast<float4*>(p) = make_float4(s[0], s[1], s[2], s[3]);
  } else {
    p[0] = s[0];
  }
}

template <int V>
__device__ __forceinline__ void stv_stream(float* p, const float (&s)[V]) {
  if constexpr (V == 4) {
    __stcs(reinterpret_cast<float4*>(p), make_float4(s[0], s[1], s[2], s[3]));
  } else {
    __stcs(p, s[0]);
  }
}

template <int V>
__device__ __forceinline__ void stw(uint32_t* p, const uint32_t (&s)[V]) {
  if constexpr (V == 4) {
    *reinterpret_cast<uint4*>(p) = make_uint4(s[0], s[1], s[2], s[3]);
  } else {
    p[0] = s[0];
  }
}

// one step of the recurrence, exactly as scan.cu evaluates it
__device__ __forceinline__ bool fwd_step(float& h, float a, float u) {
  const float d = a + h;
  const bool win = u >= d;
  h = win ? u : d;
  return win;
}

// thread -> (b, chunk j, first channel c) of the chunk-parallel passes
struct Slot {
  int64_t b, c;
  int j, rows;
  int64_t t0;
};

template <int V>
__device__ __forceinline__ bool slot_of(const ChunkArgs& p, Slot& s) {
  const int64_t nq = p.C / V;
  const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= p.B * p.nch * nq) return false;
  const int64_t q = idx % nq;
  const int64_t r = idx / nq;
  s.j = (int)(r % p.nch);
  s.b = r / p.nch;
  s.c = q * V;
  s.t0 = (int64_t)s.j * p.L;
  s.rows = (int)((p.T - s.t0) < p.L ? (p.T - s.t0) : p.L);
  return true;
}

// ---------------------------------------------------------------------------
// forward pass 1 (kOut = false: chunk state from -inf into beta) and pass 3
// (kOut = true: from the exact starting state, writing h and the mask)
// ---------------------------------------------------------------------------
template <int V, bool kHasX, bool kOut, bool kMask>
__global__ void __launch_bounds__(kPassThreads) chunk_fwd_kernel(const ChunkArgs p) {
  Slot s;
  if (!slot_of<V>(p, s)) return;
  const int64_t o = (s.b * p.nch + s.j) * p.C + s.c;
  float a[V], h[V];
  ldv<V>(a, p.a + s.c);
  if (kOut) {
    ldv<V>(h, p.hs + o);
  } else {
#pragma unroll
    for (int v = 0; v < V; ++v) h[v] = -INFINITY;
  }
  const int64_t base = (s.b * p.T + s.t0) * p.C + s.c;
  const float* pb = p.bb + base;
  const float* px = kHasX ? p.xx + base : nullptr;
  const uint64_t pol = l2_policy(!kOut);
  float* ph = kOut ? p.h + base : nullptr;
  constexpr int kRowBlock = row_block<V>();
  uint32_t bits[V];
#pragma unroll
  for (int v = 0; v < V; ++v) bits[v] = 0u;
  int t = 0;
  for (; t + kRowBlock <= s.rows; t += kRowBlock) {
    float u[kRowBlock][V];
#pragma unroll
    for (int k = 0; k < kRowBlock; ++k) {
      const int64_t off = (int64_t)(t + k) * p.C;
      ldv_pol<V>(u[k], pb + off, pol);
      if (kHasX) {
        float xv[V];
        ldv_pol<V>(xv, px + off, pol);
#pragma unroll
        for (int v = 0; v < V; ++v) u[k][v] = u[k][v] + xv[v];
      }
    }
#pragma unroll
    for (int k = 0; k < kRowBlock; ++k) {
#pragma unroll
      for (int v = 0; v < V; ++v) {
        const bool w = fwd_step(h[v], a[v], u[k][v]);
        if (kMask) bits[v] |= (uint32_t)w << ((t + k) & 31);
      }
      if (kOut) stv_stream<V>(ph + (int64_t)(t + k) * p.C, h);
    }
    if (kMask && ((t + kRowBlock) & 31) == 0) {
      stw<V>(p.win + (s.b * p.nw + (s.t0 + t) / 32) * p.C + s.c, bits);
#pragma unroll
      for (int v = 0; v < V; ++v) bits[v] = 0u;
    }
  }
  for (; t < s.rows; ++t) {
    const int64_t off = (int64_t)t * p.C;
    float u[V];
    ldv_pol<V>(u, pb + off, pol);
    if (kHasX) {
      float xv[V];
      ldv_pol<V>(xv, px + off, pol);
#pragma unroll
      for (int v = 0; v < V; ++v) u[v] = u[v] + xv[v];
    }
#pragma unroll
    for (int v = 0; v < V; ++v) {
      const bool w = fwd_step(h[v], a[v], u[v]);
      if (kMask) bits[v] |= (uint32_t)w << (t & 31);
    }
    if (kOut) stv_stream<V>(ph + off, h);
  }
  if (kMask && (s.rows & 31) != 0)   // the last, partial word of the sequence
    stw<V>(p.win + (s.b * p.nw + (s.t0 + s.rows - 1) / 32) * p.C + s.c, bits);
  if (!kOut) stv<V>(p.beta + o, h);
}

// The carry after n steps in which it keeps winning is chain_exact(h, a, n).
// A cheap upper bound settles the usual case first: chain_n(h) <= h + n a +
// n 2^-24 max_k |f_k| (+ 2^-150 per add below the normal range), and every
// |f_k| <= |h| + n |a| up to the same errors.  The margin n 2^-20 (|h| + n |a|)
// + n 2^-126 exceeds that bound together with the rounding of these few fp32
// operations (each at most 2^-24 of |h| + n |a| + margin), so a bound below g
// proves the chain ends below g; an overflow makes the bound infinite and
// merely skips the shortcut.
__device__ __forceinline__ bool chain_below(float h, float a, float nf, float g) {
  if (!isfinite(a) || !isfinite(h)) return false;
  const float mag = fabsf(h) + nf * fabsf(a);
  const float ub = fmaf(nf, a, h) + nf * 0x1p-20f * mag + nf * 0x1p-126f;
  return ub < g;
}

// state after a chunk of `rows` steps entered with h, given the chunk's own
// state from -inf (beta); exact (see the file comment).
__device__ float chunk_compose(float h, float beta, float a, int rows, const ChunkArgs& p,
                               int64_t b, int64_t c, int64_t t0) {
  // a = +inf: -inf + a is NaN, so the chunk's own state is NaN, yet any other
  // entering state becomes +inf and stays there
  if (a == INFINITY) return (h == -INFINITY || h != h) ? beta : a;
  if (beta != beta) return beta;          // NaN inside the chunk whatever enters
  if (h != h) return h;                   // a NaN state stays NaN
  if (h == -INFINITY) return beta;
  if (chain_below(h, a, (float)rows, beta)) return beta;
  const float ch = chain_exact(h, a, rows);
  if (ch != ch) return ch;
  if (ch > beta) return ch;
  if (ch < beta) return beta;
  if (ch != 0.0f) return beta;            // equal nonzero values have equal bits
  // a tie at zero: replay the chunk from h
  float hh = h;
  const int64_t base = (b * p.T + t0) * p.C + c;
  for (int t = 0; t < rows; ++t) {
    float u = p.bb[base + (int64_t)t * p.C];
    if (p.xx) u = u + p.xx[base + (int64_t)t * p.C];
    fwd_step(hh, a, u);
  }
  return hh;
}

// max(chain_n(g0), g1): a stretch of n steps with own state g1 (from -inf),
// entered with g0; NaN wins; equal zeros (signs may differ) set tie0.
// Needs a != +inf (see chunk_compose).
__device__ __forceinline__ float join_chain(float g0, float g1, float a, int64_t n, bool& tie0) {
  if (g1 != g1) return g1;
  if (g0 != g0) return g0;
  if (g0 == -INFINITY || chain_below(g0, a, (float)n, g1)) return g1;
  const float ch = chain_exact(g0, a, n);
  if (ch != ch) return ch;
  if (ch > g1) return ch;
  if (ch < g1) return g1;
  if (ch == 0.0f) tie0 = true;            // equal nonzero values have equal bits
  return g1;
}

// forward pass 2: the exact starting state of every chunk, by a parallel
// scan over the chunks of one (b, c) lane per block.  The run through chunks
// i..j from any entering state h is max(chain_n(h), G) with n their steps and
// G their state from -inf, so runs compose as (n1, G1) then (n2, G2) ->
// (n1 + n2, max(chain_n2(G1), G2)) -- associative, exact with chain_exact.
// Each warp scans 32 chunks with shuffles (5 levels); warp totals chain in
// order; a tile of blockDim.x chunks at a time.  Equal zeros anywhere (their
// sign bits are not decided by the values) send the lane to the chunk-by-
// chunk walk, which replays such chunks.
constexpr int kScanWarps = 4;

__global__ void __launch_bounds__(kScanWarps * 32) chunk_fwd_scan_kernel(const ChunkArgs p) {
  __shared__ int64_t s_n[kScanWarps];
  __shared__ float s_g[kScanWarps];
  __shared__ float s_carry;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int64_t b = blockIdx.x / p.C, c = blockIdx.x % p.C;
  const float a = p.a[c];
  const float e0 = p.h0 ? p.h0[b * p.C + c] : p.h_init;
  const float* beta = p.beta + b * p.nch * p.C + c;
  float* hs = p.hs + b * p.nch * p.C + c;
  if (a == INFINITY) {                    // see chunk_compose
    const float later = (e0 == -INFINITY || e0 != e0) ? __int_as_float(0x7fc00000) : a;
    for (int j = threadIdx.x; j < p.nch; j += blockDim.x) hs[(int64_t)j * p.C] = j == 0 ? e0 : later;
    return;
  }
  if (threadIdx.x == 0) s_carry = e0;
  bool tie0 = false;
  for (int j0 = 0; j0 < p.nch; j0 += blockDim.x) {
    const int j = j0 + threadIdx.x;
    const bool in = j < p.nch;
    const int64_t t0 = (int64_t)j * p.L;
    int64_t n = in ? ((p.T - t0) < p.L ? (p.T - t0) : p.L) : 0;
    float g = in ? __ldcg(beta + (int64_t)j * p.C) : -INFINITY;
#pragma unroll
    for (int d = 1; d < 32; d *= 2) {     // inclusive scan of the warp's chunks
      const int64_t np = __shfl_up_sync(0xffffffffu, n, d);
      const float gp = __shfl_up_sync(0xffffffffu, g, d);
      if (lane >= d) {
        g = join_chain(gp, g, a, n, tie0);
        n += np;
      }
    }
    if (lane == 31) {
      s_n[warp] = n;
      s_g[warp] = g;
    }
    __syncthreads();
    if (threadIdx.x == 0) {               // state entering each warp's first chunk
      float st = s_carry;
      for (int w = 0; w < (int)(blockDim.x >> 5); ++w) {
        const float enter = st;
        if (s_n[w] > 0) st = join_chain(st, s_g[w], a, s_n[w], tie0);
        s_g[w] = enter;
      }
      s_carry = st;
    }
    __syncthreads();
    const int64_t ne = __shfl_up_sync(0xffffffffu, n, 1);
    const float ge = __shfl_up_sync(0xffffffffu, g, 1);
    const float enter = s_g[warp];
    const float start = lane == 0 ? enter : join_chain(enter, ge, a, ne, tie0);
    if (in) hs[(int64_t)j * p.C] = start;
    __syncthreads();                      // s_g is rewritten by the next tile
  }
  if (__syncthreads_or(tie0) && threadIdx.x == 0) {
    float h = e0;
    for (int j = 0; j < p.nch; ++j) {
      hs[(int64_t)j * p.C] = h;
      const int64_t t0 = (int64_t)j * p.L;
      const int rows = (int)((p.T - t0) < p.L ? (p.T - t0) : p.L);
      h = chunk_compose(h, __ldcg(beta + (int64_t)j * p.C), a, rows, p, b, c, t0);
    }
  }
}

constexpr int kWalkGroup = 64;   // values read together by the ga reduction

// ---------------------------------------------------------------------------
// backward: pass A (kOut = false: carry leaving the chunk from carry 0, and
// whether an input won in it) and pass C (kOut = true: from the exact
// entering carry, writing gu and the chunk's partial ga)
// ---------------------------------------------------------------------------
// kSave (pass A from b, x, h): the winners it recomputes are also stored as
// mask words (p.wmask, the forward's layout), so that pass C reads gh and the
// mask instead of gh, b, x and h again.
template <int V, bool kMask, bool kHasX, bool kOut, bool kSave = false>
__global__ void __launch_bounds__(kPassThreads) chunk_bwd_kernel(const ChunkArgs p) {
  static_assert(!kSave || (!kMask && !kOut), "pass A from b, x, h saves the winners");
  Slot s;
  if (!slot_of<V>(p, s)) return;
  const int64_t o = (s.b * p.nch + s.j) * p.C + s.c;
  float a[V], hm1[V], carry[V], part[V];
  bool any[V];
  ldv<V>(a, p.a + s.c);
  if (p.h0) {
    ldv<V>(hm1, p.h0 + s.b * p.C + s.c);
  } else {
#pragma unroll
    for (int v = 0; v < V; ++v) hm1[v] = p.h_init;
  }
  if (kOut) {
    ldv<V>(carry, p.cin + o);
  } else {
#pragma unroll
    for (int v = 0; v < V; ++v) carry[v] = 0.0f;
  }
#pragma unroll
  for (int v = 0; v < V; ++v) {
    part[v] = 0.0f;
    any[v] = false;
  }
  const int64_t base = (s.b * p.T + s.t0) * p.C + s.c;
  const uint64_t pol = l2_policy(!kOut);
  uint32_t word[V], wbits[V];
#pragma unroll
  for (int v = 0; v < V; ++v) wbits[v] = 0u;
  int cur_w = -1;
  auto step_row = [&](int t, const float (&g)[V], const float (&u)[V], const float (&hp)[V]) {
    if (kMask) {
      const int w = (int)((s.t0 + t) / 32);
      if (w != cur_w) {
        ldw_pol<V>(word, p.win_in + (s.b * p.nw + w) * p.C + s.c, pol);
        cur_w = w;
      }
    }
    float out[V];
#pragma unroll
    for (int v = 0; v < V; ++v) {
      bool win;
      if (kMask) win = (word[v] >> ((s.t0 + t) & 31)) & 1u;
      else win = u[v] >= a[v] + hp[v];
      const float G = g[v] + carry[v];
      out[v] = win ? G : 0.0f;
      const float lost = win ? 0.0f : G;
      part[v] += lost;
      carry[v] = lost;
      any[v] |= win;
      if (kSave) wbits[v] |= (uint32_t)win << ((s.t0 + t) & 31);
    }
    if (kOut) stv_stream<V>(p.gu + base + (int64_t)t * p.C, out);
    if (kSave && ((s.t0 + t) & 31) == 0) {   // the word's lowest row: it is complete
      stw<V>(p.wmask + (s.b * p.nw + (s.t0 + t) / 32) * p.C + s.c, wbits);
#pragma unroll
      for (int v = 0; v < V; ++v) wbits[v] = 0u;
    }
  };
  constexpr int kRowBlock = row_block<V>();
  int t = s.rows - 1;
  for (; t + 1 >= kRowBlock; t -= kRowBlock) {
    float g[kRowBlock][V], u[kRowBlock][V], hp[kRowBlock][V];
#pragma unroll
    for (int k = 0; k < kRowBlock; ++k) {
      const int tt = t - k;
      const int64_t off = base + (int64_t)tt * p.C;
      ldv_pol<V>(g[k], p.gh + off, pol);
      if (!kMask) {
        ldv_pol<V>(u[k], p.bb + off, pol);
        if (kHasX) {
          float xv[V];
          ldv_pol<V>(xv, p.xx + off, pol);
#pragma unroll
          for (int v = 0; v < V; ++v) u[k][v] = u[k][v] + xv[v];
        }
        if (s.t0 + tt == 0) {
#pragma unroll
          for (int v = 0; v < V; ++v) hp[k][v] = hm1[v];
        } else {
          ldv_pol<V>(hp[k], p.hin + off - p.C, pol);
        }
      }
    }
#pragma unroll
    for (int k = 0; k < kRowBlock; ++k) step_row(t - k, g[k], u[k], hp[k]);
  }
  for (; t >= 0; --t) {
    float g[V], u[V], hp[V];
    const int64_t off = base + (int64_t)t * p.C;
    ldv_pol<V>(g, p.gh + off, pol);
    if (!kMask) {
      ldv_pol<V>(u, p.bb + off, pol);
      if (kHasX) {
        float xv[V];
        ldv_pol<V>(xv, p.xx + off, pol);
#pragma unroll
        for (int v = 0; v < V; ++v) u[v] = u[v] + xv[v];
      }
      if (s.t0 + t == 0) {
#pragma unroll
        for (int v = 0; v < V; ++v) hp[v] = hm1[v];
      } else {
        ldv_pol<V>(hp, p.hin + off - p.C, pol);
      }
    }
    step_row(t, g, u, hp);
  }
  if (kOut) {
    stv<V>(p.gap + o, part);
  } else {
    stv<V>(p.cout + o, carry);
#pragma unroll
    for (int v = 0; v < V; ++v) p.tflag[o + v] = any[v] ? 0 : 1;
  }
}

// backward pass B: the exact carry entering every chunk (from the end).  One
// warp per block, one (b, c) lane per thread.  The per-chunk words (no-winner
// flag, carry out) do not depend on the walk: a window of up to kBwdWin chunks is
// copied into shared memory with cp.async before it is walked.  A chunk with
// no winner passes the carry through all of its gradients in order (one add
// per step); its rows stream through a two-slot ring of kRing rows in shared
// memory, up to kSlots - 1 slots' copies in flight while one slot is added.
constexpr int kRing = 32;
constexpr int kSlots = 8;
constexpr int kBwdWin = 64;      // chunk words per window (48 KB of shared memory in all)

__global__ void __launch_bounds__(32) chunk_bwd_carry_kernel(const ChunkArgs p) {
  __shared__ int s_tf[kBwdWin][32];
  __shared__ float s_co[kBwdWin][32];
  __shared__ float s_g[kSlots][kRing][32];
  const int lane = threadIdx.x;
  const int64_t e = (int64_t)blockIdx.x * 32 + lane;
  const bool live = e < p.B * p.C;
  const int64_t b = live ? e / p.C : 0, c = live ? e % p.C : 0;
  const int64_t base = b * p.nch * p.C + c;
  const float* g = p.gh + b * p.T * p.C + c;
  float carry = 0.0f;
  for (int w1 = p.nch; w1 > 0; w1 -= kBwdWin) {          // window of chunks [w0, w1)
    const int w0 = max(0, w1 - kBwdWin);
    if (live) {
      for (int j = w0; j < w1; ++j) {
        tp_cp_async4(&s_tf[j - w0][lane], p.tflag + base + (int64_t)j * p.C, 4);
        tp_cp_async4(&s_co[j - w0][lane], p.cout + base + (int64_t)j * p.C, 4);
      }
    }
    tp_cp_async_commit();
    tp_cp_async_wait<0>();
    if (!live) continue;
    for (int j = w1 - 1; j >= w0; --j) {
      p.cin[base + (int64_t)j * p.C] = carry;
      if (!s_tf[j - w0][lane]) {
        carry = s_co[j - w0][lane];
        continue;
      }
      // no winner in chunk j: carry <- g_t + carry for t from its last row down
      const int64_t t0 = (int64_t)j * p.L;
      const int rows = (int)((p.T - t0) < p.L ? (p.T - t0) : p.L);
      const int nb = (rows + kRing - 1) / kRing;
      // ring slot bi % kSlots <- rows of batch bi (one commit group per batch;
      // batches past the end commit empty groups so that the wait count holds)
      auto issue = [&](int bi) {
        if (bi < nb) {
          const int top = rows - 1 - bi * kRing;
          const float* src = g + (t0 + top) * p.C;     // row top, then upwards
          float* dst = &s_g[bi % kSlots][0][lane];
          const int cnt = min(kRing, top + 1);
          for (int q = 0; q < cnt; ++q, src -= p.C, dst += 32) tp_cp_async4(dst, src, 4);
        }
        tp_cp_async_commit();
      };
      for (int bi = 0; bi < kSlots - 1; ++bi) issue(bi);
      for (int bi = 0; bi < nb; ++bi) {
        issue(bi + kSlots - 1);
        tp_cp_async_wait<kSlots - 1>();       // batch bi has landed
        const int top = rows - 1 - bi * kRing;
        const int cnt = min(kRing, top + 1);
        const float* sg = &s_g[bi % kSlots][0][lane];
        if (cnt == kRing) {
#pragma unroll
          for (int q = 0; q < kRing; ++q) carry = sg[q * 32] + carry;
        } else {
          for (int q = 0; q < cnt; ++q) carry = sg[q * 32] + carry;
        }
      }
      tp_cp_async_wait<0>();
    }
  }
  if (live && p.gh0) p.gh0[b * p.C + c] = carry;
}

// backward pass B with the gradient rows staged by TMA (C % 4 == 0, aligned
// gh): one warp per (b, 32 channels).  The rows of every chunk in which some
// lane has no winner arrive as boxes of kWalkBox rows x 32 channels, one copy
// instruction per box, kWalkSlots boxes in flight across chunk boundaries;
// the lanes then only add (the row copies of the plain walk above cost one
// instruction per row and a memory round trip per chunk).  With few boxes in
// flight the warp waits on each copy's latency: 24 slots (96 KB of dynamic
// shared memory) keep it adding.
constexpr int kWalkBox = 32;
constexpr int kWalkSlots = 24;
constexpr int kTmaWin = 64;      // chunk words per window

struct WalkSmem {
  float g[kWalkSlots][kWalkBox][32];
  int tf[kTmaWin][32];
  float co[kTmaWin][32];
  int need[kTmaWin];
  uint64_t full[kWalkSlots];
};

bool make_walk_map(CUtensorMap* map, const float* base, int64_t rows, int64_t C) {
  EncodeTiledFn enc = encode_tiled();
  if (!enc) return false;
  cuuint64_t dims[2] = {(cuuint64_t)C, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)C * 4};
  cuuint32_t box[2] = {32, kWalkBox};
  cuuint32_t estr[2] = {1, 1};
  return enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, (void*)base, dims, strides, box, estr,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
             CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

__global__ void __launch_bounds__(32)
    chunk_bwd_carry_tma_kernel(const __grid_constant__ CUtensorMap gmap, const ChunkArgs p,
                               int cgroups) {
  extern __shared__ __align__(128) unsigned char walk_smem[];
  WalkSmem& sm = *reinterpret_cast<WalkSmem*>(walk_smem);
  auto& s_g = sm.g;
  auto& s_tf = sm.tf;
  auto& s_co = sm.co;
  auto& s_need = sm.need;
  auto& full = sm.full;
  const unsigned all = 0xffffffffu;
  const int lane = threadIdx.x;
  const int64_t b = blockIdx.x / cgroups;
  const int64_t c0 = (int64_t)(blockIdx.x % cgroups) * 32;
  const int64_t c = c0 + lane;
  const bool live = c < p.C;
  const int64_t base = b * p.nch * p.C + c;
  const int64_t row0 = b * p.T;
  auto boxes_of = [&](int j) {
    const int64_t t0 = (int64_t)j * p.L;
    const int rows = (int)((p.T - t0) < p.L ? (p.T - t0) : p.L);
    return (rows + kWalkBox - 1) / kWalkBox;
  };
  if (lane == 0) {
    for (int s = 0; s < kWalkSlots; ++s) tp_mbar_init(&full[s], 1);
    tp_fence_mbar_init();
  }
  __syncwarp();
  uint32_t issued = 0, used = 0;      // boxes copied / added so far (lane 0 counts the first)
  float carry = 0.0f;
  for (int w1 = p.nch; w1 > 0; w1 -= kTmaWin) {            // window of chunks [w0, w1)
    const int w0 = max(0, w1 - kTmaWin);
    if (live) {
      for (int j = w0; j < w1; ++j) {
        tp_cp_async4(&s_tf[j - w0][lane], p.tflag + base + (int64_t)j * p.C, 4);
        tp_cp_async4(&s_co[j - w0][lane], p.cout + base + (int64_t)j * p.C, 4);
      }
    }
    tp_cp_async_commit();
    tp_cp_async_wait<0>();
    __syncwarp();
    // chunks in which some lane has no winner, last first
    int nneed = 0;
    for (int j = w1 - 1; j >= w0; --j) {
      if (__any_sync(all, live && s_tf[j - w0][lane] != 0)) {
        if (lane == 0) s_need[nneed] = j;
        ++nneed;
      }
    }
    __syncwarp();
    // lane 0's copy cursor: needed chunk pn, box pq of it (top box first)
    int pn = 0, pq = nneed > 0 ? boxes_of(s_need[0]) - 1 : 0;
    auto issue_next = [&]() {
      if (pn >= nneed) return;
      const int j = s_need[pn];
      const uint32_t s = issued % kWalkSlots;
      tp_mbar_arrive_expect_tx(&full[s], kWalkBox * 32 * (uint32_t)sizeof(float));
      tp_tma_load_2d(&s_g[s][0][0], &gmap, (int32_t)c0,
                     (int32_t)(row0 + (int64_t)j * p.L + (int64_t)pq * kWalkBox), &full[s]);
      ++issued;
      if (--pq < 0 && ++pn < nneed) pq = boxes_of(s_need[pn]) - 1;
    };
    if (lane == 0)
      for (int k = 0; k < kWalkSlots; ++k) issue_next();
    int ni = 0;
    for (int j = w1 - 1; j >= w0; --j) {
      if (live) p.cin[base + (int64_t)j * p.C] = carry;
      const bool needed = ni < nneed && s_need[ni] == j;
      const bool adds = live && s_tf[j - w0][lane] != 0;
      if (live && !adds) carry = s_co[j - w0][lane];
      if (!needed) continue;                 // every lane has a winner in chunk j
      ++ni;
      const int64_t t0 = (int64_t)j * p.L;
      const int rows = (int)((p.T - t0) < p.L ? (p.T - t0) : p.L);
      for (int q = boxes_of(j) - 1; q >= 0; --q) {
        const uint32_t s = used % kWalkSlots;
        if (!tp_mbar_wait(&full[s], (used / kWalkSlots) & 1u, p.err)) return;
        const int cnt = min(kWalkBox, rows - q * kWalkBox);   // the box's rows inside the chunk
        if (adds) {                          // carry <- g_t + carry, t from the box's top down
          const float* sg = &s_g[s][0][lane];
          if (cnt == kWalkBox) {
#pragma unroll
            for (int r = kWalkBox - 1; r >= 0; --r) carry = sg[r * 32] + carry;
          } else {
            for (int r = cnt - 1; r >= 0; --r) carry = sg[r * 32] + carry;
          }
        }
        ++used;
        __syncwarp();                        // every lane is done with slot s
        if (lane == 0) issue_next();
      }
    }
  }
  if (live && p.gh0) p.gh0[b * p.C + c] = carry;
}

// ga[c] = sum over b (ascending) of the chunk partials summed in descending
// chunk order
__global__ void chunk_ga_reduce_kernel(const ChunkArgs p) {
  const int64_t c = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= p.C) return;
  float total = 0.0f;
  for (int64_t b = 0; b < p.B; ++b) {
    const float* gp = p.gap + b * p.nch * p.C + c;
    float sb = 0.0f;
    for (int j0 = p.nch - 1; j0 >= 0; j0 -= kWalkGroup) {
      float v[kWalkGroup];
#pragma unroll
      for (int k = 0; k < kWalkGroup; ++k) v[k] = __ldcg(gp + (int64_t)max(j0 - k, 0) * p.C);
#pragma unroll
      for (int k = 0; k < kWalkGroup; ++k)
        if (j0 - k >= 0) sb += v[k];
    }
    total += sb;
  }
  p.ga[c] = total;
}

int64_t align256(int64_t n) { return (n + 255) & ~(int64_t)255; }

unsigned blocks_for(int64_t threads, int per_block) {
  return (unsigned)ceil_div(threads, per_block);
}

}  // namespace

int scan_chunk_pick(int64_t B, int64_t T, int64_t C) {
  // 64-step chunks: measured best at T = 4096, C = 1024 for B = 2 and 4
  // (B = 2: forward 0.044 ms at 64 against 0.052 at 32 and 0.055 at 128;
  // backward 0.186 / 0.218 / 0.244 ms) -- shorter chunks lengthen the
  // backward's per-lane walks, longer ones leave the parallel passes too few
  // threads
  (void)B;
  (void)C;
  return T >= 128 ? 64 : 32;
}

int64_t scan_chunked_workspace_bytes(int64_t B, int64_t T, int64_t C, int chunk) {
  if (B <= 0 || T <= 0 || C <= 0) return 0;
  const int L = chunk > 0 ? chunk : scan_chunk_pick(B, T, C);
  const int64_t plane = B * ceil_div(T, L) * C;
  const int64_t mask = B * ceil_div(T, (int64_t)32) * C;      // uint32 words
  return 4 * align256(plane * 4) + align256(mask * 4);
}

static int prepare(ChunkArgs& p, int chunk, void* ws, int64_t ws_bytes) {
  p.L = chunk > 0 ? chunk : scan_chunk_pick(p.B, p.T, p.C);
  if (p.L % 32 != 0 || p.L <= 0) return TP_ERR_INVALID_ARG;
  p.nch = (int)ceil_div(p.T, p.L);
  p.nw = (int)ceil_div(p.T, 32);
  const int64_t plane = p.B * (int64_t)p.nch * p.C;
  if (ws == nullptr || ws_bytes < scan_chunked_workspace_bytes(p.B, p.T, p.C, p.L))
    return TP_ERR_WORKSPACE;
  if (((uintptr_t)ws & 255u) != 0) return TP_ERR_MISALIGNED;
  char* w = static_cast<char*>(ws);
  float* f0 = reinterpret_cast<float*>(w);
  float* f1 = reinterpret_cast<float*>(w + align256(plane * 4));
  float* f2 = reinterpret_cast<float*>(w + 2 * align256(plane * 4));
  int* i0 = reinterpret_cast<int*>(w + 3 * align256(plane * 4));
  // forward: beta, hs; backward: cout, cin, gap, tflag (+ the winners' mask
  // when they are recomputed from b, x, h)
  p.beta = f0;
  p.hs = f1;
  p.wmask = reinterpret_cast<uint32_t*>(w + 4 * align256(plane * 4));
  p.err = device_error_ptr();
  p.cout = f0;
  p.cin = f1;
  p.gap = f2;
  p.tflag = i0;
  return TP_OK;
}

// Four channels per thread (128-bit loads) when that still leaves 32 warps of
// threads per SM; else one channel per thread, for 4x the threads (at B = 2,
// C = 1024, 64-step chunks the 4-channel passes filled 11% of the warp slots).
static bool vec4_ok(const ChunkArgs& p, const void* const* ptrs, int n) {
  if (p.C % 4 != 0) return false;
  if (p.B * (int64_t)p.nch * (p.C / 4) < (int64_t)num_sms() * 1024) return false;
  for (int i = 0; i < n; ++i)
    if (ptrs[i] && !aligned16(ptrs[i])) return false;
  return true;
}

int launch_scan_fwd_chunked(const ScanArgs& q, int chunk, void* ws, int64_t ws_bytes,
                            cudaStream_t stream) {
  if (q.B == 0 || q.C == 0 || q.T == 0) return TP_OK;
  ChunkArgs p{};
  p.B = q.B; p.T = q.T; p.C = q.C;
  p.bb = q.bb; p.xx = q.xx; p.a = q.a; p.h_init = q.h_init; p.h0 = q.h0;
  p.h = q.h; p.win = q.win;
  int s = prepare(p, chunk, ws, ws_bytes);
  if (s != TP_OK) return s;
  const void* ptrs[6] = {p.bb, p.xx, p.a, p.h0, p.h, p.win};
  const bool v4 = vec4_ok(p, ptrs, 6);
  const int V = v4 ? 4 : 1;
  const int64_t slots = p.B * p.nch * (p.C / V);
  const unsigned g1 = blocks_for(slots, kPassThreads);
#define TP_FWD1(VV, HX) chunk_fwd_kernel<VV, HX, false, false><<<g1, kPassThreads, 0, stream>>>(p)
#define TP_FWD3(VV, HX, MK) chunk_fwd_kernel<VV, HX, true, MK><<<g1, kPassThreads, 0, stream>>>(p)
  if (v4) {
    if (p.xx) TP_FWD1(4, true); else TP_FWD1(4, false);
  } else {
    if (p.xx) TP_FWD1(1, true); else TP_FWD1(1, false);
  }
  if ((s = launch_status()) != TP_OK) return s;
  {
    const int64_t want = ceil_div((int64_t)p.nch, 32) * 32;
    const int threads = want < kScanWarps * 32 ? (int)want : kScanWarps * 32;
    chunk_fwd_scan_kernel<<<(unsigned)(p.B * p.C), threads, 0, stream>>>(p);
  }
  if ((s = launch_status()) != TP_OK) return s;
  const bool mk = p.win != nullptr;
  if (v4) {
    if (p.xx) { if (mk) TP_FWD3(4, true, true); else TP_FWD3(4, true, false); }
    else      { if (mk) TP_FWD3(4, false, true); else TP_FWD3(4, false, false); }
  } else {
    if (p.xx) { if (mk) TP_FWD3(1, true, true); else TP_FWD3(1, true, false); }
    else      { if (mk) TP_FWD3(1, false, true); else TP_FWD3(1, false, false); }
  }
#undef TP_FWD1
#undef TP_FWD3
  (void)V;
  return launch_status();
}

int launch_scan_bwd_chunked(const ScanArgs& q, int chunk, void* ws, int64_t ws_bytes,
                            cudaStream_t stream) {
  if (q.B == 0 || q.C == 0) return TP_OK;
  if (q.T == 0) {
    int s = TP_OK;
    if (q.gh0) s = cuda_status(cudaMemsetAsync(q.gh0, 0, q.B * q.C * 4, stream));
    if (s == TP_OK && q.ga) s = cuda_status(cudaMemsetAsync(q.ga, 0, q.C * 4, stream));
    return s;
  }
  ChunkArgs p{};
  p.B = q.B; p.T = q.T; p.C = q.C;
  p.bb = q.bb; p.xx = q.xx; p.a = q.a; p.h_init = q.h_init; p.h0 = q.h0;
  p.gh = q.gh; p.hin = q.h; p.win_in = q.win_in; p.gu = q.gu; p.ga = q.ga; p.gh0 = q.gh0;
  int s = prepare(p, chunk, ws, ws_bytes);
  if (s != TP_OK) return s;
  const bool mk = p.win_in != nullptr;
  const void* ptrs[8] = {p.gh, p.a, p.h0, p.gu, mk ? nullptr : p.bb, mk ? nullptr : p.xx,
                         mk ? nullptr : p.hin, p.win_in};
  const bool v4 = vec4_ok(p, ptrs, 8);
  const int64_t slots = p.B * p.nch * (p.C / (v4 ? 4 : 1));
  const unsigned g1 = blocks_for(slots, kPassThreads);
  const bool hx = !mk && p.xx != nullptr;
  // pass A; from b, x, h it also saves the winners, which pass C then reads
  // as a mask (one bit per element instead of three fp32 values)
#define TP_BWD_A(VV)                                                                          \
  do {                                                                                        \
    if (mk) chunk_bwd_kernel<VV, true, false, false><<<g1, kPassThreads, 0, stream>>>(p);     \
    else if (hx)                                                                              \
      chunk_bwd_kernel<VV, false, true, false, true><<<g1, kPassThreads, 0, stream>>>(p);     \
    else chunk_bwd_kernel<VV, false, false, false, true><<<g1, kPassThreads, 0, stream>>>(p); \
  } while (0)
  if (v4) TP_BWD_A(4); else TP_BWD_A(1);
#undef TP_BWD_A
  if ((s = launch_status()) != TP_OK) return s;
  {
    const int64_t cgroups = ceil_div(p.C, 32);
    CUtensorMap gmap;
    const int smem = (int)sizeof(WalkSmem);
    const bool attr_set = cudaFuncSetAttribute(chunk_bwd_carry_tma_kernel,
                                               cudaFuncAttributeMaxDynamicSharedMemorySize,
                                               smem) == cudaSuccess;
    if (!attr_set) cudaGetLastError();
    if (attr_set && p.C % 4 == 0 && aligned16(p.gh) &&
        p.B * p.T + kWalkBox < (int64_t)INT32_MAX && p.B * cgroups < (int64_t)INT32_MAX &&
        make_walk_map(&gmap, p.gh, p.B * p.T, p.C))
      chunk_bwd_carry_tma_kernel<<<(unsigned)(p.B * cgroups), 32, smem, stream>>>(gmap, p,
                                                                                 (int)cgroups);
    else
      chunk_bwd_carry_kernel<<<blocks_for(p.B * p.C, 32), 32, 0, stream>>>(p);
  }
  if ((s = launch_status()) != TP_OK) return s;
  {
    ChunkArgs pc = p;
    if (!mk) pc.win_in = p.wmask;
    if (v4) chunk_bwd_kernel<4, true, false, true><<<g1, kPassThreads, 0, stream>>>(pc);
    else chunk_bwd_kernel<1, true, false, true><<<g1, kPassThreads, 0, stream>>>(pc);
  }
  if ((s = launch_status()) != TP_OK) return s;
  if (p.ga) {
    chunk_ga_reduce_kernel<<<blocks_for(p.C, 128), 128, 0, stream>>>(p);
    return launch_status();
  }
  return TP_OK;
}

}  // namespace tp
