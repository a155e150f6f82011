// esn.cu -- echo-state reservoir recurrences, whole sequence in one launch.
//
// Two recurrences (h_{-1} = 0, t = 0 .. T-1, H[:, t] = h_t):
//   GRU-gated (EchoStateReservoir, research/tsrn_dml.py:808-843, loop :834-840)
//     z = sigmoid(h Wzh^T + Uz_t)   r = sigmoid(h Wrh^T + Ur_t)
//     h~ = tanh((r * h) Ws^T + U_t) h = (1 - z) * h + z * h~
//   leaky (EchoStateReservoir, tsrn_gpu.py:466-487)
//     h = (1 - lk) * h + lk * tanh(h Ws^T + U_t)
// U, Uz, Ur are the input projections, computed for all t before the loop.
//
// Batch rows never interact, so the work splits into independent groups of
// Bg rows, one thread-block cluster per group and no grid-wide barrier.  CTA
// j of a cluster owns output columns [j*ncl, (j+1)*ncl) and keeps those rows
// of the weights in shared memory (read from L2 when they do not fit).  Each
// CTA holds the group's full state h (and r*h) in shared memory; the owner of
// a column broadcasts its new values to every CTA of the cluster with
// distributed-shared-memory stores.  The next step's U/Uz/Ur slices are fetched with cp.async while
// the current step computes.  New values travel as st.async stores that
// complete on the receiving CTA's mbarrier (armed with the exchange's byte
// count), so a CTA waits only for its own incoming data -- no cluster-wide
// barrier per step.  Eight adjacent lanes own one column: each takes
// every eighth 16-byte granule of k for all batch rows of the group (one
// weight load serves every row), and a shuffle reduction leaves row r's sum
// on lane r.
#include <mutex>
#include <utility>
#include <vector>

#include "maxplus_internal.cuh"

namespace tp {

namespace {

// lanes per column (k split) and the most columns a CTA owns (their product is
// the largest block); build parameters
#ifndef TP_ESN_KS
#define TP_ESN_KS 8
#endif
#ifndef TP_ESN_MAX_NCL
#define TP_ESN_MAX_NCL 64
#endif
constexpr int ESN_KS = TP_ESN_KS;
constexpr int ESN_MAX_NCL = TP_ESN_MAX_NCL;
static_assert(ESN_KS * ESN_MAX_NCL <= 1024, "one CTA holds at most 1024 threads");
constexpr int ESN_MAX_NT = ESN_MAX_NCL * ESN_KS;
constexpr int ESN_MAX_RB = 8;      // batch rows per cluster

struct EsnParams {
  int B, T, dr, dr4;
  int64_t ts;         // steps between consecutive batch rows of U, Uz, Ur, H (>= T)
  const float* h0;    // initial state [B][ld_h0] (NULL: zeros)
  int64_t ld_h0;
  const float* U;
  const float* Uz;
  const float* Ur;
  const float* W[3];  // GRU: Wzh, Wrh, Ws; leaky: Ws
  int64_t ld[3];
  const float* leak;  // leaky: device scalar lk
  float* H;
  int* err;           // device error word (bounded waits)
  int ncl;            // columns per CTA
  int off_h, off_pre; // shared-memory offsets in floats
};

__device__ __forceinline__ uint32_t esn_cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ uint32_t esn_cluster_size() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_nctarank;" : "=r"(r));
  return r;
}
// cluster barrier of all threads of all CTAs, in two halves: the arrive
// releases this thread's shared and distributed-shared writes, the wait
// acquires the other CTAs'.  Work between the two overlaps the barrier.
__device__ __forceinline__ void esn_cluster_arrive() {
  asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
}
__device__ __forceinline__ void esn_cluster_wait() {
  asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ void esn_cluster_sync() {
  esn_cluster_arrive();
  esn_cluster_wait();
}
// v to CTA `rank`'s copy of *local, completing 4 bytes on that CTA's copy of
// *mbar (its receive barrier for this exchange)
__device__ __forceinline__ void esn_st_async(const float* local, const uint64_t* mbar,
                                             uint32_t rank, float v) {
  uint32_t ra, rm;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(ra) : "r"(tp_smem_addr(local)),
               "r"(rank));
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(rm) : "r"(tp_smem_addr(mbar)),
               "r"(rank));
  asm volatile("st.async.shared::cluster.mbarrier::complete_tx::bytes.f32 [%0], %1, [%2];" ::"r"(ra),
               "f"(v), "r"(rm)
               : "memory");
}
__device__ __forceinline__ float esn_sigmoid(float v) { return 1.0f / (1.0f + expf(-v)); }

template <bool kSmemW>
__device__ __forceinline__ float4 esn_wload(const float4* w, int g) {
  if (kSmemW) return w[g];
  return __ldg(w + g);
}
// acc (even, odd lanes of k) += a . b over one 16-byte granule, packed f32x2
__device__ __forceinline__ float2 esn_dot4(float4 a, float4 b, float2 acc) {
  acc = tp_fma2(make_float2(a.x, a.y), make_float2(b.x, b.y), acc);
  return tp_fma2(make_float2(a.z, a.w), make_float2(b.z, b.w), acc);
}

// Sums v[r] (one partial per row r < RB) over the 8 lanes of a column group
// and returns the total of row (ks % RB) on lane ks: plain butterflies for the
// offsets >= RB, then recursive halving (each step a lane keeps half of the
// rows, N live values, and hands the other half to its partner).
template <int RB, int O, int N>
struct EsnReduce {
  static __device__ __forceinline__ void run(float (&v)[RB], int ks) {
    if constexpr (O >= RB) {
#pragma unroll
      for (int i = 0; i < RB; ++i) v[i] += __shfl_xor_sync(0xffffffffu, v[i], O);
      EsnReduce<RB, O / 2, N>::run(v, ks);
    } else {
      const bool hi = (ks & O) != 0;
#pragma unroll
      for (int i = 0; i < N / 2; ++i) {
        const float send = hi ? v[i] : v[i + N / 2];
        const float keep = hi ? v[i + N / 2] : v[i];
        v[i] = keep + __shfl_xor_sync(0xffffffffu, send, O);
      }
      EsnReduce<RB, O / 2, N / 2>::run(v, ks);
    }
  }
};
template <int RB, int N>
struct EsnReduce<RB, 0, N> {
  static __device__ __forceinline__ void run(float (&)[RB], int) {}
};
template <int RB>
__device__ __forceinline__ float esn_reduce_rows(float (&v)[RB], int ks) {
  EsnReduce<RB, ESN_KS / 2, RB>::run(v, ks);
  return v[0];
}

// Block of ESN_KS * round4(ncl) threads: lane group cl (8 lanes, ks = k slice)
// computes column c0 + cl for all RB rows of the cluster's batch group.
template <bool kGru, bool kSmemW, int RB>
__global__ void __launch_bounds__(ESN_MAX_NT, 1) esn_kernel(EsnParams p) {
  extern __shared__ __align__(16) float esn_sm[];
  constexpr int G = kGru ? 3 : 1;  // weight matrices
  constexpr int P = kGru ? 3 : 1;  // streamed inputs per step
  constexpr int PARTS = ESN_KS / RB;
  const uint32_t crank = esn_cluster_rank();
  const uint32_t csize = esn_cluster_size();
  const int b0 = (int)(blockIdx.x / csize) * RB;
  const int ncl = p.ncl, dr = p.dr, dr4 = p.dr4, NG = dr4 >> 2;
  const int c0 = (int)crank * ncl;
  const int items = RB * ncl;
  const int tid = threadIdx.x, nt = blockDim.x;
  const int cl = tid / ESN_KS, ks = tid % ESN_KS;
  const int row = ks % RB, part = ks / RB;
  const bool col_ok = cl < ncl && c0 + cl < dr;
  const bool row_ok = b0 + row < p.B;
  float* wsm = esn_sm;
  float* hs = esn_sm + p.off_h;   // GRU: h [RB][dr4], r*h [RB][dr4]; leaky: h [2][RB][dr4]
  float* rhs = hs + RB * dr4;
  float* pre = esn_sm + p.off_pre;  // [3][P][RB][ncl], ring of step inputs

  if (kSmemW) {
#pragma unroll
    for (int g = 0; g < G; ++g)
      for (int e = tid; e < ncl * dr4; e += nt) {
        const int c = e / dr4, k = e - c * dr4;
        float v = 0.0f;
        if (c0 + c < dr && k < dr) v = p.W[g][(int64_t)(c0 + c) * p.ld[g] + k];
        wsm[(g * ncl + c) * dr4 + k] = v;
      }
  }
  // state buffers: h_{-1} = h0 (or 0) in the buffer step 0 reads (GRU: h;
  // leaky: buffer 0), zeros elsewhere
  for (int e = tid; e < 2 * RB * dr4; e += nt) {
    float v = 0.0f;
    if (p.h0 && e < RB * dr4) {
      const int r = e / dr4, k = e - r * dr4;
      if (k < dr && b0 + r < p.B) v = p.h0[(int64_t)(b0 + r) * p.ld_h0 + k];
    }
    hs[e] = v;
  }

  // stage step t's inputs into ring slot t % 3 (one commit group per call,
  // empty past the end so that the group count stays uniform)
  auto prefetch = [&](int t) {
    float* dst = pre + (t % 3) * P * items;
    for (int e = tid; t < p.T && e < P * items; e += nt) {
      const int pi = e / items, it = e - pi * items;
      const int bl = it / ncl, c = it - bl * ncl;
      const int b = b0 + bl, cg = c0 + c;
      const float* src = pi == 0 ? p.U : (pi == 1 ? p.Uz : p.Ur);
      const bool ok = b < p.B && cg < dr;
      tp_cp_async4(dst + e, ok ? src + ((int64_t)b * p.ts + t) * dr + cg : src, ok ? 4 : 0);
    }
    tp_cp_async_commit();
  };
  auto wrow = [&](int g) -> const float4* {
    const int c = min(cl, ncl - 1);
    if (kSmemW) return reinterpret_cast<const float4*>(wsm + (g * ncl + c) * dr4);
    const int cg = min(c0 + c, dr - 1);
    return reinterpret_cast<const float4*>(p.W[g] + (int64_t)cg * p.ld[g]);
  };
  const float4* w_s = wrow(G - 1);
  const float4* w_z = kGru ? wrow(0) : w_s;
  const float4* w_r = kGru ? wrow(1) : w_s;
  const int pidx = row * ncl + min(cl, ncl - 1);
  float hprev = 0.0f, zv = 0.0f;
  if (p.h0 && col_ok && row_ok) hprev = p.h0[(int64_t)(b0 + row) * p.ld_h0 + c0 + cl];
  const float lk = kGru ? 0.0f : *p.leak;

  // Receive barriers, one phase per exchange: each expects the bytes of every
  // valid (row, column) of the group (all CTAs send to all, this one
  // included).  Leaky: mb[b] for the h buffer b (step t writes buffer
  // (t+1)&1).  GRU: mb[0] for r*h, mb[1] for h (single buffers: a sender's
  // next write needs values this CTA sends only after its reads).  A barrier
  // is re-armed (arrive + expect) by thread 0 right after its phase is
  // waited for.
  __shared__ __align__(8) uint64_t mb[2];
  const uint32_t xbytes = (uint32_t)(min(RB, p.B - b0) * dr * (int)sizeof(float));
  if (tid == 0) {
    tp_mbar_init(&mb[0], 1);
    tp_mbar_init(&mb[1], 1);
    tp_fence_mbar_init();
    tp_mbar_arrive_expect_tx(&mb[0], xbytes);
    tp_mbar_arrive_expect_tx(&mb[1], xbytes);
  }
  // waits are bounded; after a timeout (recorded) the kernel runs on without
  // waiting, so that no CTA leaves while others may still write into it
  bool failed = false;
  auto recv = [&](int b, uint32_t parity) {
    if (!failed && !tp_mbar_wait(&mb[b], parity, p.err)) failed = true;
    if (tid == 0) tp_mbar_arrive_expect_tx(&mb[b], xbytes);
  };

  prefetch(0);
  prefetch(1);
  tp_cp_async_wait<1>();
  esn_cluster_sync();  // every CTA of the cluster is running; barriers, weights, state, step 0

  for (int t = 0; t < p.T; ++t) {
    prefetch(t + 2);
    const float* pin = pre + (t % 3) * P * items;
    if (kGru && t >= 1) recv(1, (uint32_t)(t - 1) & 1u);           // h_{t-1}
    if (!kGru && t >= 1) recv(t & 1, (uint32_t)((t - 1) >> 1) & 1u);  // h_{t-1}
    if (kGru) {
      // half-step A: z, r and r * h_{t-1} for column c0 + cl
      float2 az[RB], ar[RB];
#pragma unroll
      for (int r = 0; r < RB; ++r) az[r] = ar[r] = make_float2(0.0f, 0.0f);
      for (int g = ks; g < NG; g += ESN_KS) {
        const float4 a = esn_wload<kSmemW>(w_z, g);
        const float4 b = esn_wload<kSmemW>(w_r, g);
#pragma unroll
        for (int r = 0; r < RB; ++r) {
          const float4 h = reinterpret_cast<const float4*>(hs + r * dr4)[g];
          az[r] = esn_dot4(h, a, az[r]);
          ar[r] = esn_dot4(h, b, ar[r]);
        }
      }
      float vz[RB], vr[RB];
#pragma unroll
      for (int r = 0; r < RB; ++r) {
        vz[r] = az[r].x + az[r].y;
        vr[r] = ar[r].x + ar[r].y;
      }
      const float sz = esn_reduce_rows<RB>(vz, ks);
      const float sr = esn_reduce_rows<RB>(vr, ks);
      const float z = esn_sigmoid(sz + pin[items + pidx]);
      const float r = esn_sigmoid(sr + pin[2 * items + pidx]);
      zv = z;
      const float rh = r * hprev;
      __syncthreads();  // every thread has seen the last phase before any send
      if (col_ok && row_ok)
        for (uint32_t rk = part; rk < csize; rk += PARTS)
          esn_st_async(rhs + row * dr4 + c0 + cl, &mb[0], rk, rh);
      recv(0, (uint32_t)t & 1u);                                      // r*h_{t-1}
    }
    // GRU half-step B / leaky step: h~ and h_t for column c0 + cl
    const float* src = kGru ? rhs : hs + (t & 1) * RB * dr4;
    float* dst = kGru ? hs : hs + ((t + 1) & 1) * RB * dr4;
    float2 acc[RB];
#pragma unroll
    for (int r = 0; r < RB; ++r) acc[r] = make_float2(0.0f, 0.0f);
    for (int g = ks; g < NG; g += ESN_KS) {
      const float4 w = esn_wload<kSmemW>(w_s, g);
#pragma unroll
      for (int r = 0; r < RB; ++r)
        acc[r] = esn_dot4(reinterpret_cast<const float4*>(src + r * dr4)[g], w, acc[r]);
    }
    float va[RB];
#pragma unroll
    for (int r = 0; r < RB; ++r) va[r] = acc[r].x + acc[r].y;
    const float a = esn_reduce_rows<RB>(va, ks);
    const float ht = tanhf(a + pin[pidx]);
    const float z = kGru ? zv : lk;
    const float h = __fadd_rn(__fmul_rn(1.0f - z, hprev), __fmul_rn(z, ht));
    hprev = h;
    // the next step's inputs landed (the newest group may still be in
    // flight); the barrier publishes them to every thread, frees this step's
    // input slot, and orders every thread's view of the last phase before the
    // sends below
    tp_cp_async_wait<1>();
    __syncthreads();
    if (col_ok && row_ok) {
      for (uint32_t rk = part; rk < csize; rk += PARTS)
        esn_st_async(dst + row * dr4 + c0 + cl, &mb[kGru ? 1 : (t + 1) & 1], rk, h);
      if (part == 0) p.H[((int64_t)(b0 + row) * p.ts + t) * dr + c0 + cl] = h;
    }
  }
  // the last exchange has fully arrived here, and (cluster barrier) everywhere
  // else, before any CTA leaves
  if (p.T >= 1) {
    if (kGru)
      recv(1, (uint32_t)(p.T - 1) & 1u);
    else
      recv(p.T & 1, (uint32_t)((p.T - 1) >> 1) & 1u);
  }
  esn_cluster_sync();
}


// ---------------------------------------------------------------------------
// Backward through time of both recurrences, one launch (same cluster layout,
// exchanges and input ring as the forward; time runs from T-1 down to 0).
// With g the state gradient carried from step t+1 (0 after the last step):
//   GRU:   dh = dH_t + g,  dah = dh fa_t                    (exchanged)
//          dm = dah Ws,   dar = dm fr_t,  daz = dh fz_t    (both exchanged)
//          g  = dh keep_t + dm r_t + daz Wzh + dar Wrh
//   leaky: dh = dH_t + g,  da = dh fa_t                     (exchanged)
//          g  = dh (1 - lk) + da Ws
// fa = z (1 - h~^2), fz = (h~ - h_{t-1}) z (1 - z), fr = h_{t-1} r (1 - r),
// keep = 1 - z (GRU); fa = lk (1 - s^2) (leaky): per-step factors formed
// for all steps beforehand.  Column k of a product v W is the dot of v with
// row k of W^T, so the kernel takes the transposed weights and reads them
// like the forward reads its own.  Outputs per step: GRU dah, daz, dar (the
// gradients of the three pre-activations); leaky da and dh.
// ---------------------------------------------------------------------------
struct EsnBwdParams {
  int B, T, dr, dr4;
  const float* dH;    // [B][T][dr]
  const float* F[5];  // GRU: fa, fz, fr, keep, r; leaky: fa
  const float* W[3];  // transposed weights: GRU WzhT, WrhT, WsT; leaky WsT
  int64_t ld[3];
  const float* leak;  // leaky: device scalar lk
  float* out[3];      // GRU: dAh, dAz, dAr; leaky: dA, dHs
  int* err;
  int ncl;
  int off_x, off_pre; // shared-memory offsets in floats
};

template <bool kGru, bool kSmemW, int RB>
__global__ void __launch_bounds__(ESN_MAX_NT, 1) esn_bwd_kernel(EsnBwdParams p) {
  extern __shared__ __align__(16) float esn_sm[];
  constexpr int G = kGru ? 3 : 1;  // weight matrices
  constexpr int P = kGru ? 6 : 2;  // streamed inputs per step: dH and the factors
  constexpr int PARTS = ESN_KS / RB;
  const uint32_t crank = esn_cluster_rank();
  const uint32_t csize = esn_cluster_size();
  const int b0 = (int)(blockIdx.x / csize) * RB;
  const int ncl = p.ncl, dr = p.dr, dr4 = p.dr4, NG = dr4 >> 2;
  const int c0 = (int)crank * ncl;
  const int items = RB * ncl;
  const int tid = threadIdx.x, nt = blockDim.x;
  const int cl = tid / ESN_KS, ks = tid % ESN_KS;
  const int row = ks % RB, part = ks / RB;
  const bool col_ok = cl < ncl && c0 + cl < dr;
  const bool row_ok = b0 + row < p.B;
  float* wsm = esn_sm;
  // exchange buffers: GRU dah, daz, dar [RB][dr4] each; leaky da [2][RB][dr4]
  float* xs = esn_sm + p.off_x;
  float* pre = esn_sm + p.off_pre;  // [3][P][RB][ncl], ring of step inputs

  if (kSmemW) {
#pragma unroll
    for (int g = 0; g < G; ++g)
      for (int e = tid; e < ncl * dr4; e += nt) {
        const int c = e / dr4, k = e - c * dr4;
        float v = 0.0f;
        if (c0 + c < dr && k < dr) v = p.W[g][(int64_t)(c0 + c) * p.ld[g] + k];
        wsm[(g * ncl + c) * dr4 + k] = v;
      }
  }
  for (int e = tid; e < 3 * RB * dr4; e += nt) xs[e] = 0.0f;

  // stage step s's inputs (time T-1-s) into ring slot s % 3
  auto prefetch = [&](int s) {
    float* dst = pre + (s % 3) * P * items;
    const int t = p.T - 1 - s;
    for (int e = tid; s < p.T && e < P * items; e += nt) {
      const int pi = e / items, it = e - pi * items;
      const int bl = it / ncl, c = it - bl * ncl;
      const int b = b0 + bl, cg = c0 + c;
      const float* src = pi == 0 ? p.dH : p.F[pi - 1];
      const bool ok = b < p.B && cg < dr;
      tp_cp_async4(dst + e, ok ? src + ((int64_t)b * p.T + t) * dr + cg : src, ok ? 4 : 0);
    }
    tp_cp_async_commit();
  };
  auto wrow = [&](int g) -> const float4* {
    const int c = min(cl, ncl - 1);
    if (kSmemW) return reinterpret_cast<const float4*>(wsm + (g * ncl + c) * dr4);
    const int cg = min(c0 + c, dr - 1);
    return reinterpret_cast<const float4*>(p.W[g] + (int64_t)cg * p.ld[g]);
  };
  const float4* w_s = wrow(G - 1);
  const float4* w_z = kGru ? wrow(0) : w_s;
  const float4* w_r = kGru ? wrow(1) : w_s;
  const int pidx = row * ncl + min(cl, ncl - 1);
  const float lk = kGru ? 0.0f : *p.leak;
  float g = 0.0f;   // state gradient from the step after

  // receive barriers: GRU mb[0] dah, mb[1] daz + dar; leaky mb[b] for the da
  // buffer b (step s writes buffer s & 1).  Re-armed by thread 0 after each
  // wait, as in the forward.
  __shared__ __align__(8) uint64_t mb[2];
  const uint32_t xbytes = (uint32_t)(min(RB, p.B - b0) * dr * (int)sizeof(float));
  const uint32_t xb1 = kGru ? 2 * xbytes : xbytes;
  if (tid == 0) {
    tp_mbar_init(&mb[0], 1);
    tp_mbar_init(&mb[1], 1);
    tp_fence_mbar_init();
    tp_mbar_arrive_expect_tx(&mb[0], xbytes);
    tp_mbar_arrive_expect_tx(&mb[1], xb1);
  }
  bool failed = false;
  auto recv = [&](int b, uint32_t parity) {
    if (!failed && !tp_mbar_wait(&mb[b], parity, p.err)) failed = true;
    if (tid == 0) tp_mbar_arrive_expect_tx(&mb[b], b == 1 ? xb1 : xbytes);
  };
  auto dot = [&](const float4* w, const float* v) -> float {
    float2 acc[RB];
#pragma unroll
    for (int r = 0; r < RB; ++r) acc[r] = make_float2(0.0f, 0.0f);
    for (int q = ks; q < NG; q += ESN_KS) {
      const float4 wv = esn_wload<kSmemW>(w, q);
#pragma unroll
      for (int r = 0; r < RB; ++r)
        acc[r] = esn_dot4(reinterpret_cast<const float4*>(v + r * dr4)[q], wv, acc[r]);
    }
    float va[RB];
#pragma unroll
    for (int r = 0; r < RB; ++r) va[r] = acc[r].x + acc[r].y;
    return esn_reduce_rows<RB>(va, ks);
  };

  prefetch(0);
  prefetch(1);
  tp_cp_async_wait<1>();
  esn_cluster_sync();  // every CTA of the cluster is running; barriers, weights, step 0

  for (int s = 0; s < p.T; ++s) {
    const int t = p.T - 1 - s;
    prefetch(s + 2);
    const float* pin = pre + (s % 3) * P * items;
    // every input of this step into registers now: the slot is refilled at
    // the start of step s + 3, which a thread may reach while this one is
    // still in the step's second half
    float f[P];
#pragma unroll
    for (int q = 0; q < P; ++q) f[q] = pin[q * items + pidx];
    const float dh = f[0] + g;
    const int64_t o = ((int64_t)(b0 + row) * p.T + t) * dr + c0 + cl;
    if (kGru) {
      float* dahs = xs;
      float* dazs = xs + RB * dr4;
      float* dars = xs + 2 * RB * dr4;
      const float dah = dh * f[1];
      __syncthreads();  // every thread has seen the last phase before any send
      if (col_ok && row_ok)
        for (uint32_t rk = part; rk < csize; rk += PARTS)
          esn_st_async(dahs + row * dr4 + c0 + cl, &mb[0], rk, dah);
      recv(0, (uint32_t)s & 1u);
      const float dm = dot(w_s, dahs);
      const float dar = dm * f[3];
      const float daz = dh * f[2];
      // the next step's inputs landed; the barrier publishes them and orders
      // every thread's view of the last phase before the sends below
      tp_cp_async_wait<1>();
      __syncthreads();
      if (col_ok && row_ok) {
        for (uint32_t rk = part; rk < csize; rk += PARTS) {
          esn_st_async(dazs + row * dr4 + c0 + cl, &mb[1], rk, daz);
          esn_st_async(dars + row * dr4 + c0 + cl, &mb[1], rk, dar);
        }
        if (part == 0) {
          p.out[0][o] = dah;
          p.out[1][o] = daz;
          p.out[2][o] = dar;
        }
      }
      recv(1, (uint32_t)s & 1u);
      const float gz = dot(w_z, dazs);
      const float gr = dot(w_r, dars);
      g = dh * f[4] + dm * f[5] + gz + gr;
    } else {
      float* das = xs + (s & 1) * RB * dr4;
      const float da = dh * f[1];
      tp_cp_async_wait<1>();
      __syncthreads();
      if (col_ok && row_ok) {
        for (uint32_t rk = part; rk < csize; rk += PARTS)
          esn_st_async(das + row * dr4 + c0 + cl, &mb[s & 1], rk, da);
        if (part == 0) {
          p.out[0][o] = da;
          p.out[1][o] = dh;
        }
      }
      recv(s & 1, (uint32_t)(s >> 1) & 1u);
      g = dh * (1.0f - lk) + dot(w_s, das);
    }
  }
  // every exchange was received inside its step; the cluster barrier keeps
  // each CTA alive until all have left the loop
  esn_cluster_sync();
}

struct EsnPlan {
  int CS, ncl, RB, nt;
  bool smemW;
  size_t smem;
  int clusters;
};

size_t esn_smem_bytes(bool gru, bool smemW, int dr4, int ncl, int RB, bool bwd = false) {
  const int G = gru ? 3 : 1;
  const int P = bwd ? (gru ? 6 : 2) : (gru ? 3 : 1);
  const size_t w = smemW ? (size_t)G * ncl * dr4 : 0;
  const size_t state = (size_t)(bwd ? 3 : 2) * RB * dr4;
  const size_t pre = (size_t)3 * P * RB * ncl;
  return (w + state + pre) * sizeof(float);
}

// the kernel of a (direction, recurrence, weight placement, rows) choice, and
// its parameter block
template <bool kBwd, bool kGru, bool kSmemW, int RB>
struct EsnKernel {
  using Params = EsnParams;
  static constexpr auto fn = esn_kernel<kGru, kSmemW, RB>;
};
template <bool kGru, bool kSmemW, int RB>
struct EsnKernel<true, kGru, kSmemW, RB> {
  using Params = EsnBwdParams;
  static constexpr auto fn = esn_bwd_kernel<kGru, kSmemW, RB>;
};

template <class Kn>
int esn_configure(const EsnPlan& pl, cudaLaunchConfig_t* cfg, cudaLaunchAttribute* attr) {
  auto kern = Kn::fn;
  cudaError_t e =
      cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)pl.smem);
  if (e != cudaSuccess) return (int)e;
  if (pl.CS > 8) {
    e = cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
    if (e != cudaSuccess) return (int)e;
  }
  *cfg = cudaLaunchConfig_t{};
  cfg->gridDim = dim3((unsigned)(pl.clusters * pl.CS));
  cfg->blockDim = dim3((unsigned)pl.nt);
  cfg->dynamicSmemBytes = pl.smem;
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = pl.CS;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg->attrs = attr;
  cfg->numAttrs = 1;
  return TP_OK;
}

// kind 0: occupancy query (max active clusters into *out); kind 1: launch
// (params: the kernel's parameter block; unused for kind 0)
template <class Kn>
int esn_run(int kind, const EsnPlan& pl, const void* params, cudaStream_t stream, int* out) {
  cudaLaunchConfig_t cfg;
  cudaLaunchAttribute attr[1];
  int st = esn_configure<Kn>(pl, &cfg, attr);
  if (st != TP_OK) return st;
  if (kind == 0) {
    cfg.gridDim = dim3((unsigned)pl.CS);
    return (int)cudaOccupancyMaxActiveClusters(out, (const void*)Kn::fn, &cfg);
  }
  cfg.stream = stream;
  const typename Kn::Params& p = *static_cast<const typename Kn::Params*>(params);
  cudaError_t e = cudaLaunchKernelEx(&cfg, Kn::fn, p);
  if (e != cudaSuccess) return (int)e;
  return launch_status();
}

template <bool kBwd, bool kGru, bool kSmemW>
int esn_run_rb(int kind, const EsnPlan& pl, const void* p, cudaStream_t s, int* out) {
  switch (pl.RB) {
    case 1: return esn_run<EsnKernel<kBwd, kGru, kSmemW, 1>>(kind, pl, p, s, out);
    case 2: return esn_run<EsnKernel<kBwd, kGru, kSmemW, 2>>(kind, pl, p, s, out);
    case 4: return esn_run<EsnKernel<kBwd, kGru, kSmemW, 4>>(kind, pl, p, s, out);
    default: return esn_run<EsnKernel<kBwd, kGru, kSmemW, 8>>(kind, pl, p, s, out);
  }
}

template <bool kBwd>
int esn_dispatch_dir(bool gru, int kind, const EsnPlan& pl, const void* p, cudaStream_t s,
                     int* out) {
  if (gru) return pl.smemW ? esn_run_rb<kBwd, true, true>(kind, pl, p, s, out)
                           : esn_run_rb<kBwd, true, false>(kind, pl, p, s, out);
  return pl.smemW ? esn_run_rb<kBwd, false, true>(kind, pl, p, s, out)
                  : esn_run_rb<kBwd, false, false>(kind, pl, p, s, out);
}

int esn_dispatch(bool bwd, bool gru, int kind, const EsnPlan& pl, const void* p, cudaStream_t s,
                 int* out) {
  return bwd ? esn_dispatch_dir<true>(gru, kind, pl, p, s, out)
             : esn_dispatch_dir<false>(gru, kind, pl, p, s, out);
}

// Plan: over cluster sizes CS (at most cs_cap CTAs, <= 64 columns each) and
// rows per cluster RB (power of two <= 8), the candidate with the lowest
// waves x (2 + RB) score (below); weights stay in shared memory when they
// fit, else they are read from L2 (global_ok).
int esn_plan(bool bwd, bool gru, int B, int dr, bool global_ok, int cs_cap, EsnPlan* pl) {
  const int dr4 = (dr + 3) & ~3;
  int dev = 0, smem_max = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return (int)e;
  e = cudaDeviceGetAttribute(&smem_max, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
  if (e != cudaSuccess) return (int)e;
  smem_max -= 1024;   // the kernel's static shared memory (receive barriers)
  // candidate (CS, RB) -> filled plan, or false when it cannot run
  auto make = [&](int CS, int RB, EsnPlan* out, int* maxc) -> int {
    const int ncl = (dr + CS - 1) / CS;
    if (ncl > ESN_MAX_NCL) return -1;
    bool smemW = esn_smem_bytes(gru, true, dr4, ncl, RB, bwd) <= (size_t)smem_max;
    if (!smemW &&
        (!global_ok || esn_smem_bytes(gru, false, dr4, ncl, RB, bwd) > (size_t)smem_max))
      return -1;
    out->CS = CS;
    out->ncl = ncl;
    out->RB = RB;
    out->nt = ((ncl + 3) / 4) * 4 * ESN_KS;
    out->smemW = smemW;
    out->smem = esn_smem_bytes(gru, smemW, dr4, ncl, RB, bwd);
    out->clusters = (B + RB - 1) / RB;
    *maxc = 0;
    const int st = esn_dispatch(bwd, gru, 0, *out, nullptr, nullptr, maxc);
    if (st != TP_OK) {
      (void)cudaGetLastError();
      return -1;
    }
    return *maxc >= 1 ? 0 : -1;
  };
  // score = waves x (2 + RB): the per-step cost of a wave grows with the rows
  // a cluster carries, and extra waves repeat it (fitted to a sweep on B200
  // of d_reservoir 256/320/640, both recurrences, B=64: it picks the fastest
  // measured (CS, RB) in every case).  Ties: cluster sizes in the order
  // 8, 4, 16, 2, 1 (8 CTAs measured fastest at equal waves), then smaller RB.
  static const int kCsOrder[5] = {8, 4, 16, 2, 1};
  bool have = false;
  EsnPlan best{};
  int64_t best_score = 0;
  int best_rank = 0;
  for (int RB = 1; RB <= ESN_MAX_RB; RB *= 2) {
    for (int r = 0; r < 5; ++r) {
      const int CS = kCsOrder[r];
      if (CS > cs_cap) continue;
      EsnPlan c{};
      int maxc = 0;
      if (make(CS, RB, &c, &maxc) != 0) continue;
      const int64_t waves = (c.clusters + maxc - 1) / maxc;
      const int64_t score = waves * (2 + RB);
      if (!have || score < best_score || (score == best_score && r < best_rank)) {
        best = c;
        best_score = score;
        best_rank = r;
        have = true;
      }
    }
    if (RB >= B) break;  // one cluster already; more rows per cluster cannot help
  }
  if (have) {
    *pl = best;
    return TP_OK;
  }
  return TP_ERR_UNSUPPORTED;
}

// plans are cached per (mode, B, dr, global_ok, device): planning runs
// several occupancy queries
struct EsnPlanKey {
  bool bwd, gru, global_ok;
  int B, dr, dev;
  bool operator==(const EsnPlanKey& o) const {
    return bwd == o.bwd && gru == o.gru && global_ok == o.global_ok && B == o.B && dr == o.dr &&
           dev == o.dev;
  }
};
std::mutex esn_plan_mu;
std::vector<std::pair<EsnPlanKey, EsnPlan>> esn_plan_cache;

int esn_plan_cached(bool bwd, bool gru, int B, int dr, bool global_ok, EsnPlan* pl) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return (int)e;
  const EsnPlanKey key{bwd, gru, global_ok, B, dr, dev};
  {
    std::lock_guard<std::mutex> lk(esn_plan_mu);
    for (auto& kv : esn_plan_cache)
      if (kv.first == key) {
        *pl = kv.second;
        return TP_OK;
      }
  }
  // clusters of 16 CTAs (a non-portable size) when the device schedules
  // them, else at most 8
  int st = esn_plan(bwd, gru, B, dr, global_ok, 16, pl);
  if (st != TP_OK) {
    (void)cudaGetLastError();
    st = esn_plan(bwd, gru, B, dr, global_ok, 8, pl);
  }
  if (st != TP_OK) return st;
  std::lock_guard<std::mutex> lk(esn_plan_mu);
  if (esn_plan_cache.size() >= 64) esn_plan_cache.clear();
  esn_plan_cache.emplace_back(key, *pl);
  return TP_OK;
}

bool esn_vec_ok(const float* w, int64_t ld, int dr) {
  return (dr % 4) == 0 && (ld % 4) == 0 && ((uintptr_t)w & 15u) == 0;
}

}  // namespace

int launch_esn_fwd(bool gru, int64_t B, int64_t T, int64_t dr, const float* U, const float* Uz,
                   const float* Ur, const float* const W[3], const int64_t ld[3],
                   const float* leak, float* H, cudaStream_t stream, int64_t ts,
                   const float* h0, int64_t ld_h0) {
  if (B * T * dr == 0) return TP_OK;
  if (B > INT32_MAX / 2 || T > INT32_MAX / 2) return TP_ERR_TOO_LARGE;
  if (ts < T) ts = T;
  if (dr > 16 * ESN_MAX_NCL) return TP_ERR_UNSUPPORTED;
  const int G = gru ? 3 : 1;
  bool global_ok = true;
  for (int g = 0; g < G; ++g) global_ok = global_ok && esn_vec_ok(W[g], ld[g], (int)dr);
  EsnPlan pl{};
  const int st = esn_plan_cached(false, gru, (int)B, (int)dr, global_ok, &pl);
  if (st != TP_OK) return st;
  if ((int64_t)pl.clusters * pl.CS > INT32_MAX) return TP_ERR_TOO_LARGE;
  EsnParams p{};
  p.B = (int)B;
  p.T = (int)T;
  p.ts = ts;
  p.h0 = h0;
  p.ld_h0 = ld_h0;
  p.dr = (int)dr;
  p.dr4 = ((int)dr + 3) & ~3;
  p.U = U;
  p.Uz = Uz;
  p.Ur = Ur;
  for (int g = 0; g < 3; ++g) {
    p.W[g] = g < G ? W[g] : nullptr;
    p.ld[g] = g < G ? ld[g] : 0;
  }
  p.leak = leak;
  p.H = H;
  p.err = device_error_ptr();
  p.ncl = pl.ncl;
  p.off_h = pl.smemW ? G * pl.ncl * p.dr4 : 0;
  p.off_pre = p.off_h + 2 * pl.RB * p.dr4;
  return esn_dispatch(false, gru, 1, pl, &p, stream, nullptr);
}

int launch_esn_bwd(bool gru, int64_t B, int64_t T, int64_t dr, const float* dH,
                   const float* const F[5], const float* const WT[3], const int64_t ld[3],
                   const float* leak, float* const out[3], cudaStream_t stream) {
  if (B * T * dr == 0) return TP_OK;
  if (B > INT32_MAX / 2 || T > INT32_MAX / 2) return TP_ERR_TOO_LARGE;
  if (dr > 16 * ESN_MAX_NCL) return TP_ERR_UNSUPPORTED;
  const int G = gru ? 3 : 1;
  bool global_ok = true;
  for (int g = 0; g < G; ++g) global_ok = global_ok && esn_vec_ok(WT[g], ld[g], (int)dr);
  EsnPlan pl{};
  const int st = esn_plan_cached(true, gru, (int)B, (int)dr, global_ok, &pl);
  if (st != TP_OK) return st;
  if ((int64_t)pl.clusters * pl.CS > INT32_MAX) return TP_ERR_TOO_LARGE;
  EsnBwdParams p{};
  p.B = (int)B;
  p.T = (int)T;
  p.dr = (int)dr;
  p.dr4 = ((int)dr + 3) & ~3;
  p.dH = dH;
  for (int q = 0; q < 5; ++q) p.F[q] = (gru || q == 0) ? F[q] : nullptr;
  for (int g = 0; g < 3; ++g) {
    p.W[g] = g < G ? WT[g] : nullptr;
    p.ld[g] = g < G ? ld[g] : 0;
  }
  p.leak = leak;
  for (int q = 0; q < 3; ++q) p.out[q] = (gru || q < 2) ? out[q] : nullptr;
  p.err = device_error_ptr();
  p.ncl = pl.ncl;
  p.off_x = pl.smemW ? G * pl.ncl * p.dr4 : 0;
  p.off_pre = p.off_x + 3 * pl.RB * p.dr4;
  return esn_dispatch(true, gru, 1, pl, &p, stream, nullptr);
}

}  // namespace tp
