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

constexpr int ESN_KS = 8;          // lanes per column (k split)
constexpr int ESN_MAX_NCL = 64;    // columns per CTA
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

struct EsnPlan {
  int CS, ncl, RB, nt;
  bool smemW;
  size_t smem;
  int clusters;
};

size_t esn_smem_bytes(bool gru, bool smemW, int dr4, int ncl, int RB) {
  const int G = gru ? 3 : 1, P = gru ? 3 : 1;
  const size_t w = smemW ? (size_t)G * ncl * dr4 : 0;
  const size_t state = (size_t)2 * RB * dr4;
  const size_t pre = (size_t)3 * P * RB * ncl;
  return (w + state + pre) * sizeof(float);
}

template <bool kGru, bool kSmemW, int RB>
int esn_configure(const EsnPlan& pl, cudaLaunchConfig_t* cfg, cudaLaunchAttribute* attr) {
  auto kern = esn_kernel<kGru, kSmemW, RB>;
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
template <bool kGru, bool kSmemW, int RB>
int esn_run(int kind, const EsnPlan& pl, const EsnParams& p, cudaStream_t stream, int* out) {
  cudaLaunchConfig_t cfg;
  cudaLaunchAttribute attr[1];
  int st = esn_configure<kGru, kSmemW, RB>(pl, &cfg, attr);
  if (st != TP_OK) return st;
  if (kind == 0) {
    cfg.gridDim = dim3((unsigned)pl.CS);
    return (int)cudaOccupancyMaxActiveClusters(out, (const void*)esn_kernel<kGru, kSmemW, RB>,
                                               &cfg);
  }
  cfg.stream = stream;
  cudaError_t e = cudaLaunchKernelEx(&cfg, esn_kernel<kGru, kSmemW, RB>, p);
  if (e != cudaSuccess) return (int)e;
  return launch_status();
}

template <bool kGru, bool kSmemW>
int esn_run_rb(int kind, const EsnPlan& pl, const EsnParams& p, cudaStream_t s, int* out) {
  switch (pl.RB) {
    case 1: return esn_run<kGru, kSmemW, 1>(kind, pl, p, s, out);
    case 2: return esn_run<kGru, kSmemW, 2>(kind, pl, p, s, out);
    case 4: return esn_run<kGru, kSmemW, 4>(kind, pl, p, s, out);
    default: return esn_run<kGru, kSmemW, 8>(kind, pl, p, s, out);
  }
}

int esn_dispatch(bool gru, int kind, const EsnPlan& pl, const EsnParams& p, cudaStream_t s,
                 int* out) {
  if (gru) return pl.smemW ? esn_run_rb<true, true>(kind, pl, p, s, out)
                           : esn_run_rb<true, false>(kind, pl, p, s, out);
  return pl.smemW ? esn_run_rb<false, true>(kind, pl, p, s, out)
                  : esn_run_rb<false, false>(kind, pl, p, s, out);
}

// Plan: over cluster sizes CS (at most cs_cap CTAs, <= 64 columns each) and
// rows per cluster RB (power of two <= 8), the candidate with the lowest
// waves x (2 + RB) score (below); weights stay in shared memory when they
// fit, else they are read from L2 (global_ok).
int esn_plan(bool gru, int B, int dr, bool global_ok, int cs_cap, EsnPlan* pl) {
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
    bool smemW = esn_smem_bytes(gru, true, dr4, ncl, RB) <= (size_t)smem_max;
    if (!smemW && (!global_ok || esn_smem_bytes(gru, false, dr4, ncl, RB) > (size_t)smem_max))
      return -1;
    out->CS = CS;
    out->ncl = ncl;
    out->RB = RB;
    out->nt = ((ncl + 3) / 4) * 4 * ESN_KS;
    out->smemW = smemW;
    out->smem = esn_smem_bytes(gru, smemW, dr4, ncl, RB);
    out->clusters = (B + RB - 1) / RB;
    EsnParams dummy{};
    *maxc = 0;
    const int st = esn_dispatch(gru, 0, *out, dummy, nullptr, maxc);
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
  bool gru, global_ok;
  int B, dr, dev;
  bool operator==(const EsnPlanKey& o) const {
    return gru == o.gru && global_ok == o.global_ok && B == o.B && dr == o.dr && dev == o.dev;
  }
};
std::mutex esn_plan_mu;
std::vector<std::pair<EsnPlanKey, EsnPlan>> esn_plan_cache;

int esn_plan_cached(bool gru, int B, int dr, bool global_ok, EsnPlan* pl) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return (int)e;
  const EsnPlanKey key{gru, global_ok, B, dr, dev};
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
  int st = esn_plan(gru, B, dr, global_ok, 16, pl);
  if (st != TP_OK) {
    (void)cudaGetLastError();
    st = esn_plan(gru, B, dr, global_ok, 8, pl);
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
  const int st = esn_plan_cached(gru, (int)B, (int)dr, global_ok, &pl);
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
  return esn_dispatch(gru, 1, pl, p, stream, nullptr);
}

}  // namespace tp
