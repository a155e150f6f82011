// tsrn_attention_tc.cu -- the fused TSRN tropical top-k attention forward
// (research/tsrn_dml.py:438-460 score, :509-524 ALiBi / causal mask / top-k /
// softmax / V) with the score contraction on the 5th-generation tensor cores.
//
// The log-sum-exp over channels factorises into a dot product of exp features
// (each in (0, 1]; see tsrn_attention.cu):
//   S[i,j] = log( F_Q[i,:] . F_K[j,:] ) + qmax_i + kmax_j - slope_h |i - (j - Tc)|
// so the scores of a 128-query tile against a 64-key tile are one 128 x 64
// GEMM with K = dh.  fp32 accuracy from TF32 operands by the 3xTF32 split:
// F = hi + lo with hi = F with its low 13 mantissa bits cleared (exact in
// TF32) and lo = F - hi (exact in fp32; its TF32 rounding costs ~2^-22 of F),
//   F_Q . F_K ~= hi_Q . hi_K + hi_Q . lo_K + lo_Q . hi_K
// (the dropped lo . lo term is below 2^-22 of the product): three
// tcgen05.mma kind::tf32 chains into one fp32 accumulator in tensor memory.
//
// Pre-pass: one warp per row writes hi and lo as row-major [rows_pad, 96]
// planes (channels past dh and rows past the sequence are zero) plus the row
// maxima.  Main kernel: one CTA per (b, h, 128-query tile), 10 warps:
//   warp 0   TMA producer: the query tile once (hi, lo: 96 KB), then key tiles
//            (hi, lo: 48 KB) through a 2-stage ring; 128-byte swizzle, the
//            K-major layout tcgen05 reads;
//   warp 1   allocates 128 TMEM columns and issues the MMAs of each key tile
//            (M = 128, N = 64, K = 8 per instruction) into one of two
//            64-column accumulators; tcgen05.commit frees the key stage and
//            publishes the accumulator;
//   warps 2-9 two threads per query row (TMEM lane = row; a warp reads the
//            lanes of its quarter, warp % 4): the thread of half h takes the
//            tile's columns 2c + h (interleaved, so that keys clustered near
//            the diagonal split evenly), tcgen05.ld's the 64 scores, releases
//            the accumulator and finishes its 32.
// Selection in two passes over the key tiles:
//   pass 1 (keys nearest the diagonal first: tiles in descending order, a
//          tile's columns too): each thread keeps the 16 largest of its scores
//          (a sorted register list, NaN never enters);
//          the two lists of a row are merged in shared memory: rowmax = the
//          first, thr = the top_k-th, ties counted as torch.topk counts them;
//          every score that reached the list's last entry when it was seen is
//          also logged (key, score) in global memory: a superset of the kept
//          keys {j : !(S < thr), S != -inf}, which are then listed from the
//          log with the softmax normaliser, in logged order;
//   pass 2 runs only when a log overflowed (or a score was NaN): it
//          recomputes the same MMAs (same operands, same order: the same bits)
//          and lists each half's kept keys in ascending j.
// Then each warp gathers the V rows of 16 rows' kept keys (lanes split the
// channels).  Kept keys beyond a half's TC_KCAP list entries (ties at the
// threshold) are accumulated by their thread into a scratch row -- the
// output row for half 0, the CTA's own (already consumed) query-feature row
// for half 1 -- and added in by the gather.
// A dot below 1e-30 is recomputed exactly from the raw rows, as in the
// CUDA-core kernel (out of line: rare).
#include "maxplus_internal.cuh"

namespace tp {

namespace {

constexpr int TC_M = 128;           // query rows per CTA = TMEM lanes
constexpr int TC_N = 64;            // keys per tile = accumulator columns
constexpr int TC_KP = 96;           // feature channels, padded: 3 swizzle atoms
constexpr int TC_ATOM = 32;         // fp32 channels per 128-byte swizzled row
constexpr int TC_LIST = 16;         // per-thread score list (top_k <= 16)
constexpr int TC_KCAP = 16;         // kept keys listed per row half in shared memory (>= top_k)
constexpr int TC_EPI_WARPS = 8;     // two per TMEM lane quarter
constexpr int TC_THREADS = 64 + 32 * TC_EPI_WARPS;
constexpr int TC_TMEM_COLS = 128;   // two accumulators of TC_N columns
constexpr int TC_MAX_DH = 96;
constexpr int TC_LISTS_OUT = 2 * TC_KCAP;   // kept keys per row saved for the backward
constexpr int TC_LOGCAP = 48;      // pass-1 candidates logged per row half (else pass 2 runs)
static_assert(TC_LISTS_OUT == TSRN_ATT_LIST, "saved list width");

constexpr uint32_t TC_Q_ATOM_FLOATS = TC_M * TC_ATOM;     // 16 KB
constexpr uint32_t TC_K_ATOM_FLOATS = TC_N * TC_ATOM;     // 8 KB
constexpr uint32_t TC_Q_BYTES = 2 * 3 * TC_Q_ATOM_FLOATS * 4;   // hi + lo
constexpr uint32_t TC_K_STAGE_BYTES = 2 * 3 * TC_K_ATOM_FLOATS * 4;
constexpr size_t TC_LIST_BYTES = (size_t)2 * TC_KCAP * TC_M * 8;   // kept lists (j, S) per half
static_assert((size_t)2 * TC_LIST * TC_M * 4 <= TC_LIST_BYTES,
              "pass-1 score lists are merged in the kept-list space");
// (the per-row counts, normalisers and maxima of the gather live in the query
// tile's space, free once the last MMA has read it)
static_assert((size_t)TC_M * 4 * 5 <= TC_Q_BYTES, "gather state fits the query tile");
constexpr size_t TC_SMEM_BYTES = 1024                          // alignment slack
                                 + TC_Q_BYTES + 2 * TC_K_STAGE_BYTES + TC_LIST_BYTES
                                 + 16 * 8;                     // barriers, TMEM address, flags

// instruction descriptor of tcgen05.mma kind::tf32: fp32 accumulator, TF32 A
// and B, both K-major, N = TC_N, M = TC_M
constexpr uint32_t TC_IDESC = (1u << 4) | (2u << 7) | (2u << 10) |
                              ((uint32_t)(TC_N >> 3) << 17) | ((uint32_t)(TC_M >> 4) << 24);

// shared-memory matrix descriptor: K-major, 128-byte swizzle (8-row groups
// 1024 bytes apart), descriptor version 1
__device__ __forceinline__ uint64_t tc_desc(const float* p) {
  const uint32_t a = tp_smem_addr(p);
  return (uint64_t)((a >> 4) & 0x3FFFu) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
         ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}

__device__ __forceinline__ void tc_mma(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc,
                                       uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(TC_IDESC), "r"(accumulate)
      : "memory");
}

__device__ __forceinline__ void tc_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   tp_smem_addr(bar))
               : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// 32 consecutive accumulator columns of this warp's 32 TMEM lanes
__device__ __forceinline__ void tc_ld32(uint32_t taddr, uint32_t (&v)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]),
        "=r"(v[7]), "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]),
        "=r"(v[14]), "=r"(v[15]), "=r"(v[16]), "=r"(v[17]), "=r"(v[18]), "=r"(v[19]),
        "=r"(v[20]), "=r"(v[21]), "=r"(v[22]), "=r"(v[23]), "=r"(v[24]), "=r"(v[25]),
        "=r"(v[26]), "=r"(v[27]), "=r"(v[28]), "=r"(v[29]), "=r"(v[30]), "=r"(v[31])
      : "r"(taddr));
}

__device__ __forceinline__ void tc_wait_ld() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// ---------------------------------------------------------------------------
// pre-pass: exp features split into TF32 hi / lo planes [S][rows_pad][96]
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(256) att_tc_feat_kernel(const float* __restrict__ X,
                                                          int64_t rows, int64_t rows_pad, int dh,
                                                          float* __restrict__ Fhi,
                                                          float* __restrict__ Flo,
                                                          float* __restrict__ mx,
                                                          int64_t mx_ld) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t slice = blockIdx.y;
  const int64_t r = (int64_t)blockIdx.x * 8 + warp;
  if (r >= rows_pad) return;
  const float NEG_INF = -__int_as_float(0x7f800000);
  const bool live = r < rows;
  const float* xr = X + (slice * rows + (live ? r : 0)) * dh;
  float v[3];
  float m = NEG_INF;
#pragma unroll
  for (int u = 0; u < 3; ++u) {
    const int c = lane + 32 * u;
    v[u] = (live && c < dh) ? xr[c] : NEG_INF;
    m = fmaxf(m, v[u]);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  const int64_t o = (slice * rows_pad + r) * TC_KP;
#pragma unroll
  for (int u = 0; u < 3; ++u) {
    const int c = lane + 32 * u;
    const float f = (live && c < dh) ? expf(v[u] - m) : 0.0f;
    const float hi = __uint_as_float(__float_as_uint(f) & 0xffffe000u);
    Fhi[o + c] = hi;
    Flo[o + c] = f - hi;
  }
  if (lane == 0 && r < mx_ld) mx[slice * mx_ld + r] = live ? m : 0.0f;
}

struct TcArgs {
  int64_t S, H, T, Tkv, Tc;
  int64_t Tp, Kp;         // query rows / keys per slice in the feature planes
  int dh, top_k, causal, nk;
  const float* Q;
  const float* K;
  const float* V;
  const float* slopes;
  const float* qmx;       // [S][T]
  const float* kmx;       // [S][Kp]
  float* out;             // [S][T][dh]
  float* qlo;             // [S][Tp][TC_KP]: query-feature lo plane (overflow scratch of half 1)
  // optional (training): each row's kept keys and softmax weights, half 0's
  // list then half 1's, [S][T][TC_LISTS_OUT] (j = -1 past the end), and the
  // count per row [S][T] (-1 when a half overflowed its list)
  int* kj;
  float* kp;
  float* kl;              // [S][T][TC_LISTS_OUT]: the entry's log-sum-exp score before ALiBi
  int* kn;
  float2* log;            // [grid][2][TC_LOGCAP][TC_M]: pass-1 candidates (key bits, score)
  int* err;
};

// exact max-shifted log-sum-exp of query row i and key j from the raw rows,
// for dots below 1e-30 (out of line: rare)
__device__ __noinline__ float tc_exact_lse(const float* qr, const float* kr, int dh) {
  const float NEG_INF = -__int_as_float(0x7f800000);
  float m = NEG_INF;
  for (int c = 0; c < dh; ++c) m = fmaxf(m, qr[c] + kr[c]);
  float z = 0.0f;
  if (m > NEG_INF)
    for (int c = 0; c < dh; ++c) z += expf(qr[c] + kr[c] - m);
  return (m > NEG_INF) ? m + logf(z) : NEG_INF;
}

// insert s into the descending list L (drops the smallest); s > L[TC_LIST-1]
__device__ __forceinline__ void tc_insert(float (&L)[TC_LIST], float s) {
#pragma unroll
  for (int k = TC_LIST - 1; k >= 1; --k) L[k] = fmaxf(L[k], fminf(L[k - 1], s));
  L[0] = fmaxf(L[0], s);
}

// a kept key beyond the half's list: weight e times V row j into the
// scratch row (zeroed at the first such key)
__device__ __noinline__ void tc_overflow_add(float* dst, bool first, float e, const float* vr,
                                             int dh) {
  for (int c = 0; c < dh; ++c) dst[c] = fmaf(e, vr[c], first ? 0.0f : dst[c]);
}

__device__ __forceinline__ void tc_epi_sync() {
  asm volatile("bar.sync 1, %0;" ::"n"(32 * TC_EPI_WARPS) : "memory");
}

__global__ void __launch_bounds__(TC_THREADS, 1)
    att_tc_kernel(const __grid_constant__ CUtensorMap map_qh,
                  const __grid_constant__ CUtensorMap map_ql,
                  const __grid_constant__ CUtensorMap map_kh,
                  const __grid_constant__ CUtensorMap map_kl, const TcArgs p) {
  extern __shared__ uint8_t tc_raw[];
  float* sQ = reinterpret_cast<float*>((reinterpret_cast<uintptr_t>(tc_raw) + 1023) &
                                       ~(uintptr_t)1023);
  float* sK = sQ + 2 * 3 * TC_Q_ATOM_FLOATS;                       // [stage][hi/lo][atom]
  uint8_t* lists = reinterpret_cast<uint8_t*>(sK + 2 * 2 * 3 * TC_K_ATOM_FLOATS);
  int* s_kj = reinterpret_cast<int*>(lists);                       // [half][TC_KCAP][TC_M]
  float* s_ks = reinterpret_cast<float*>(s_kj + 2 * TC_KCAP * TC_M);   // [half][TC_KCAP][TC_M]
  float* s_lst = reinterpret_cast<float*>(lists);                  // pass 1: [half][TC_LIST][TC_M]
  // gather state, written after the last MMA: in the query tile's space
  int* s_cnt = reinterpret_cast<int*>(sQ);                         // [half][TC_M]
  float* s_z = reinterpret_cast<float*>(s_cnt + 2 * TC_M);         // [half][TC_M]
  float* s_rmax = s_z + 2 * TC_M;                                  // [TC_M]
  uint64_t* bars = reinterpret_cast<uint64_t*>(lists + TC_LIST_BYTES);
  uint64_t* q_full = bars;
  uint64_t* k_full = bars + 1;        // [2]
  uint64_t* k_empty = bars + 3;       // [2]
  uint64_t* acc_full = bars + 5;      // [2]
  uint64_t* acc_empty = bars + 7;     // [2]
  uint32_t* s_tmem = reinterpret_cast<uint32_t*>(bars + 9);
  int* s_flag = reinterpret_cast<int*>(bars + 10);     // [1]: a bounded wait gave up

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t nqt = p.Tp / TC_M;
  const int64_t cta = blockIdx.x;
  const int64_t qt = nqt - 1 - cta / p.S;                // heaviest (causal) tiles first
  const int64_t slice = cta % p.S;
  const int i0 = (int)(qt * TC_M);
  int kv_end = (int)p.Tkv;
  if (p.causal) {
    const int last = (i0 + TC_M - 1 < p.T) ? i0 + TC_M - 1 : (int)p.T - 1;
    kv_end = last + (int)p.Tc + 1 < p.Tkv ? last + (int)p.Tc + 1 : (int)p.Tkv;
  }
  const int nt = (kv_end + TC_N - 1) / TC_N;

  if (threadIdx.x == 0) {
    tp_mbar_init(q_full, 1);
    for (int s = 0; s < 2; ++s) {
      tp_mbar_init(&k_full[s], 1);
      tp_mbar_init(&k_empty[s], 1);
      tp_mbar_init(&acc_full[s], 1);
      tp_mbar_init(&acc_empty[s], TC_EPI_WARPS);
    }
    s_flag[0] = 0;
    s_flag[1] = 0;
    tp_fence_mbar_init();
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     tp_smem_addr(s_tmem)),
                 "r"(TC_TMEM_COLS)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *s_tmem;

  // epilogue state (warps 2-9): row r of the tile, columns 2c + half of each key tile
  const int quarter = warp & 3;
  const int half = (warp - 2) >> 2;
  const int r = quarter * 32 + lane;
  const int i = i0 + r;
  const bool row_ok = warp >= 2 && i < p.T;
  const float NEG_INF = -__int_as_float(0x7f800000);
  const float slope = p.slopes[slice % p.H];
  const float qm = row_ok ? p.qmx[slice * p.T + i] : 0.0f;
  // keys this row may see: j < jlim
  int jlim = (int)p.Tkv;
  if (p.causal) jlim = (i + (int)p.Tc + 1 < p.Tkv) ? i + (int)p.Tc + 1 : (int)p.Tkv;
  float L[TC_LIST];
#pragma unroll
  for (int k = 0; k < TC_LIST; ++k) L[k] = NEG_INF;
  float thr = NEG_INF, rowmax = NEG_INF, z = 0.0f;
  int cnt = 0;
  // pass-1 candidate log of this thread (row r, its half of the key columns):
  // every score that reached the list's last entry when it was seen -- a
  // superset of the kept keys, since that entry only grows up to the
  // threshold.  A log that overflows, or a NaN score, sends the CTA through
  // pass 2 instead.
  float2* lg = p.log + ((int64_t)blockIdx.x * 2 + (half > 0 ? 1 : 0)) * TC_LOGCAP * TC_M + r;
  int lcnt = 0;
  bool lbad = false;
  // scratch row of this thread's kept keys beyond its list
  float* ovf_row = half == 0 ? p.out + (slice * p.T + (row_ok ? i : 0)) * p.dh
                             : p.qlo + (slice * p.Tp + i0 + r) * TC_KP;
  const float* Vs = p.V + slice * p.Tkv * p.dh;

  // the producer and MMA threads remember what they issued last, so that an
  // aborted CTA can wait for its own copies and MMAs before it exits
  int last_load = -1, last_mma = -1;

  for (int round = 0; round < 2; ++round) {
    if (round == 1) {
      __syncthreads();
      // pass 2 only when some thread could not log all its candidates
      if (s_flag[1] != 0 || s_flag[0] == 0) break;
      cnt = 0;            // it rebuilds every row's kept list
      z = 0.0f;
    }
    const int it0 = round * nt;
    if (warp == 0) {
      if (lane == 0 && s_flag[1] == 0) {
        if (round == 0) {
          tp_prefetch_tensormap(&map_qh);
          tp_prefetch_tensormap(&map_ql);
          tp_prefetch_tensormap(&map_kh);
          tp_prefetch_tensormap(&map_kl);
          tp_mbar_arrive_expect_tx(q_full, TC_Q_BYTES);
          const int32_t y = (int32_t)(slice * p.Tp + i0);
          for (int a = 0; a < 3; ++a) {
            tp_tma_load_2d(sQ + a * TC_Q_ATOM_FLOATS, &map_qh, a * TC_ATOM, y, q_full);
            tp_tma_load_2d(sQ + (3 + a) * TC_Q_ATOM_FLOATS, &map_ql, a * TC_ATOM, y, q_full);
          }
        }
        for (int n = 0; n < nt; ++n) {
          const int it = it0 + n, st = it & 1, use = it >> 1;
          const int t = round == 0 ? nt - 1 - n : n;
          if (!tp_mbar_wait(&k_empty[st], (use & 1) ^ 1, p.err)) {
            s_flag[1] = 1;
            break;
          }
          tp_mbar_arrive_expect_tx(&k_full[st], TC_K_STAGE_BYTES);
          const int32_t y = (int32_t)(slice * p.Kp + (int64_t)t * TC_N);
          float* dst = sK + st * 2 * 3 * TC_K_ATOM_FLOATS;
          for (int a = 0; a < 3; ++a) {
            tp_tma_load_2d(dst + a * TC_K_ATOM_FLOATS, &map_kh, a * TC_ATOM, y, &k_full[st]);
            tp_tma_load_2d(dst + (3 + a) * TC_K_ATOM_FLOATS, &map_kl, a * TC_ATOM, y,
                           &k_full[st]);
          }
          last_load = it;
        }
      }
      __syncwarp();
    } else if (warp == 1) {
      if (lane == 0 && s_flag[1] == 0) {
        bool ok = round == 1 || tp_mbar_wait(q_full, 0, p.err);
        if (!ok) s_flag[1] = 1;
        for (int n = 0; ok && n < nt; ++n) {
          const int it = it0 + n, st = it & 1, use = it >> 1;
          if (!tp_mbar_wait(&acc_empty[st], (use & 1) ^ 1, p.err) ||
              !tp_mbar_wait(&k_full[st], use & 1, p.err)) {
            s_flag[1] = 1;
            break;
          }
          tc_fence_after();
          const uint32_t d = tmem + (uint32_t)(st * TC_N);
          const float* kb = sK + st * 2 * 3 * TC_K_ATOM_FLOATS;
          uint32_t acc = 0;
          // hi.hi, hi.lo, lo.hi
#pragma unroll 1
          for (int prod = 0; prod < 3; ++prod) {
            const float* qa = sQ + (prod == 2 ? 3 : 0) * TC_Q_ATOM_FLOATS;
            const float* kbb = kb + (prod == 1 ? 3 : 0) * TC_K_ATOM_FLOATS;
            for (int ks = 0; ks < p.nk; ++ks) {
              const int a = ks >> 2, kk = (ks & 3) * 8;
              tc_mma(d, tc_desc(qa + a * TC_Q_ATOM_FLOATS + kk),
                     tc_desc(kbb + a * TC_K_ATOM_FLOATS + kk), acc);
              acc = 1;
            }
          }
          tc_commit(&k_empty[st]);
          tc_commit(&acc_full[st]);
          last_mma = it;
        }
      }
      __syncwarp();
    } else {
      // ---- scores: two threads per row, 32 interleaved columns each per tile
      float kmn0 = 0.0f, kmn1 = 0.0f;   // key maxima of the next tile (prefetched)
      {
        const int t = round == 0 ? nt - 1 : 0;
        kmn0 = p.kmx[slice * p.Kp + t * TC_N + lane];
        kmn1 = p.kmx[slice * p.Kp + t * TC_N + 32 + lane];
      }
      for (int n = 0; n < nt; ++n) {
        const int it = it0 + n, st = it & 1, use = it >> 1;
        const int t = round == 0 ? nt - 1 - n : n;
        const float km0 = kmn0, km1 = kmn1;
        if (n + 1 < nt) {
          const int tn = round == 0 ? t - 1 : t + 1;
          kmn0 = p.kmx[slice * p.Kp + tn * TC_N + lane];
          kmn1 = p.kmx[slice * p.Kp + tn * TC_N + 32 + lane];
        }
        // the whole warp leaves together (tcgen05.ld is warp-collective)
        const bool got = tp_mbar_wait(&acc_full[st], use & 1, p.err);
        if (!__all_sync(0xffffffffu, got)) {
          s_flag[1] = 1;
          break;
        }
        tc_fence_after();
        const int j0 = t * TC_N;
        // all 32 scores first (independent: the compiler can overlap them);
        // dots below 1e-30 (or NaN) are marked and recomputed exactly below.
        // The tile's two 32-column halves are read one after the other.
        float sc[32];
        uint32_t slow = 0;
        const float fbase = (float)(i - j0 - half + (int)p.Tc);   // i - j for cc = 0
        const uint32_t ta = tmem + ((uint32_t)(quarter * 32) << 16) + (uint32_t)(st * TC_N);
#pragma unroll
        for (int hv = 0; hv < 2; ++hv) {
          uint32_t v[32];
          tc_ld32(ta + 32 * hv, v);
          tc_wait_ld();
          if (hv == 1) {
            tc_fence_before();
            __syncwarp();
            if (lane == 0) tp_mbar_arrive(&acc_empty[st]);
          }
          const float km = hv == 0 ? km0 : km1;
#pragma unroll
          for (int q = 0; q < 16; ++q) {
            const int cc = 16 * hv + q;
            const int c = 2 * cc + half;
            const float kmc = __shfl_sync(0xffffffffu, km, c & 31);
            const float d = __uint_as_float(half ? v[2 * q + 1] : v[2 * q]);
            const bool valid = row_ok && j0 + c < jlim;
            float l2;
            asm("lg2.approx.f32 %0, %1;" : "=f"(l2) : "f"(d));
            const float s0 = __fadd_rn(__fadd_rn(__fmul_rn(l2, 0.6931471805599453f), qm), kmc);
            const float dist = fabsf(fbase - (float)(2 * cc));
            if (valid && !(d >= 1e-30f)) slow |= 1u << cc;
            sc[cc] = valid ? __fmaf_rn(-slope, dist, s0) : NEG_INF;
          }
        }
        if (__any_sync(0xffffffffu, slow != 0)) {
#pragma unroll
          for (int cc = 0; cc < 32; ++cc)
            if ((slow >> cc) & 1u) {
              const int j = j0 + 2 * cc + half;
              const float e = tc_exact_lse(p.Q + (slice * p.T + i) * p.dh,
                                           p.K + (slice * p.Tkv + j) * p.dh, p.dh);
              sc[cc] = __fmaf_rn(-slope, fabsf(fbase - (float)(2 * cc)), e);
            }
        }
        if (round == 0) {
          // candidates against the list's last entry before this tile (it only
          // grows, so no later candidate is missed); columns where no lane
          // has one are skipped with a warp-uniform branch.  A candidate at
          // least equal to the current last entry is logged (ties included),
          // one strictly above it enters the list.
          const float l15 = L[TC_LIST - 1];
          uint32_t cand = 0;
#pragma unroll
          for (int cc = 0; cc < 32; ++cc) {
            cand |= ((sc[cc] >= l15 && sc[cc] != NEG_INF) ? 1u : 0u) << cc;
            lbad |= sc[cc] != sc[cc];
          }
          const uint32_t wm = __reduce_or_sync(0xffffffffu, cand);
          if (wm != 0) {
            // keys nearest the diagonal first (the tiles run that way too):
            // with ALiBi the large scores come early and later keys rarely
            // reach the list, which keeps both the insertions and the log short
#pragma unroll
            for (int cc = 31; cc >= 0; --cc)
              if ((wm >> cc) & 1u) {
                const float sv = sc[cc];
                if (sv >= L[TC_LIST - 1] && sv != NEG_INF) {
                  if (lcnt < TC_LOGCAP)
                    lg[lcnt * TC_M] = make_float2(__int_as_float(j0 + 2 * cc + half), sv);
                  ++lcnt;
                  if (sv > L[TC_LIST - 1]) tc_insert(L, sv);
                }
              }
          }
        } else {
          uint32_t kept = 0;
#pragma unroll
          for (int cc = 0; cc < 32; ++cc)
            kept |= ((!(sc[cc] < thr) && sc[cc] != NEG_INF) ? 1u : 0u) << cc;
          const uint32_t wm = __reduce_or_sync(0xffffffffu, kept);
          if (wm != 0) {
#pragma unroll
            for (int cc = 0; cc < 32; ++cc)
              if (((wm >> cc) & 1u) && ((kept >> cc) & 1u)) {
                const int j = j0 + 2 * cc + half;
                const float e = expf(sc[cc] - rowmax);
                z += e;
                if (cnt < TC_KCAP) {
                  s_kj[(half * TC_KCAP + cnt) * TC_M + r] = j;
                  s_ks[(half * TC_KCAP + cnt) * TC_M + r] = sc[cc];
                } else {
                  tc_overflow_add(ovf_row, cnt == TC_KCAP, e, Vs + (int64_t)j * p.dh, p.dh);
                }
                ++cnt;
              }
          }
        }
      }
      if (round == 0) {
        // merge the row's two lists: rowmax and the top_k-th largest
#pragma unroll
        for (int k = 0; k < TC_LIST; ++k) s_lst[(half * TC_LIST + k) * TC_M + r] = L[k];
        tc_epi_sync();
        int a = 0, b = 0;
        for (int k = 0; k < p.top_k; ++k) {
          const float x = s_lst[a * TC_M + r], y = s_lst[(TC_LIST + b) * TC_M + r];
          if (x >= y) {
            thr = x;
            ++a;
          } else {
            thr = y;
            ++b;
          }
        }
        rowmax = fmaxf(s_lst[r], s_lst[TC_LIST * TC_M + r]);
        tc_epi_sync();          // the lists' space is the kept-key lists' of pass 2
        // the kept keys from the log, in logged order (pass 2 is not needed
        // unless some thread of the CTA could not log all its candidates)
        if (lbad || lcnt > TC_LOGCAP) {
          s_flag[0] = 1;
        } else if (row_ok) {
          for (int e = 0; e < lcnt; ++e) {
            const float2 ent = lg[e * TC_M];
            const float sv = ent.y;
            if (sv < thr) continue;
            const int j = __float_as_int(ent.x);
            const float ev = expf(sv - rowmax);
            z += ev;
            if (cnt < TC_KCAP) {
              s_kj[(half * TC_KCAP + cnt) * TC_M + r] = j;
              s_ks[(half * TC_KCAP + cnt) * TC_M + r] = sv;
            } else {
              tc_overflow_add(ovf_row, cnt == TC_KCAP, ev, Vs + (int64_t)j * p.dh, p.dh);
            }
            ++cnt;
          }
        }
      }
    }
  }

  // ---- gather: each warp forms the outputs of 16 rows (lanes split the
  // channels), from the kept-key lists
  if (warp >= 2) {
    if (row_ok) {
      s_cnt[half * TC_M + r] = cnt;
      s_z[half * TC_M + r] = z;
      if (half == 0) s_rmax[r] = rowmax;
    }
    tc_epi_sync();
    if (s_flag[1] == 0) {
      const int e8 = warp - 2;
      for (int rr = 0; rr < TC_M / TC_EPI_WARPS; ++rr) {
        const int row = e8 * (TC_M / TC_EPI_WARPS) + rr;
        const int ii = i0 + row;
        if (ii >= p.T) break;
        const int c0 = s_cnt[row], c1 = s_cnt[TC_M + row];
        const float rmax = s_rmax[row];
        const float invz = 1.0f / (s_z[row] + s_z[TC_M + row]);
        float* orr = p.out + (slice * p.T + ii) * p.dh;
        float oacc[3] = {0.0f, 0.0f, 0.0f};
        // each half's listed keys eight at a time: the eight V rows' loads in
        // flight together (one L2 round trip per eight keys); accumulated in
        // list order (the order pass 1 logged them, or ascending key after a
        // pass 2), half 0 first
        for (int hh = 0; hh < 2; ++hh) {
          const int n = min(hh ? c1 : c0, TC_KCAP);
          for (int e0 = 0; e0 < n; e0 += 8) {
            int jj[8];
            float val[8][3];
#pragma unroll
            for (int e = 0; e < 8; ++e) {
              jj[e] = e0 + e < n ? s_kj[(hh * TC_KCAP + e0 + e) * TC_M + row] : -1;
#pragma unroll
              for (int q = 0; q < 3; ++q) {
                const int c = lane + 32 * q;
                val[e][q] =
                    (jj[e] >= 0 && c < p.dh) ? __ldg(Vs + (int64_t)jj[e] * p.dh + c) : 0.0f;
              }
            }
#pragma unroll
            for (int e = 0; e < 8; ++e)
              if (jj[e] >= 0) {
                const float wv = expf(s_ks[(hh * TC_KCAP + e0 + e) * TC_M + row] - rmax) * invz;
#pragma unroll
                for (int q = 0; q < 3; ++q) oacc[q] = fmaf(wv, val[e][q], oacc[q]);
              }
          }
        }
        if (p.kj != nullptr) {
          // the row's kept keys and weights for the backward: lane e writes
          // entry e (half 0's list, then half 1's)
          const int64_t lrow = slice * p.T + ii;
          const bool over = c0 > TC_KCAP || c1 > TC_KCAP;
          if (lane < TC_LISTS_OUT) {
            const int hh = lane >= c0 ? 1 : 0;
            const int e = hh ? lane - c0 : lane;
            const bool ok = !over && e < (hh ? c1 : c0);
            const int slot = (hh * TC_KCAP + (ok ? e : 0)) * TC_M + row;
            const int jk = ok ? s_kj[slot] : -1;
            const float sk = s_ks[slot];
            p.kj[lrow * TC_LISTS_OUT + lane] = jk;
            p.kp[lrow * TC_LISTS_OUT + lane] = ok ? expf(sk - rmax) * invz : 0.0f;
            // the score with its ALiBi term added back: the log-sum-exp of
            // (Q_i + K_j) over the channels, which the backward differentiates
            p.kl[lrow * TC_LISTS_OUT + lane] =
                ok ? __fmaf_rn(slope, fabsf((float)(ii - jk + (int)p.Tc)), sk) : 0.0f;
          }
          if (lane == 0) p.kn[lrow] = over ? -1 : c0 + c1;
        }
        // kept keys past the lists, accumulated (unnormalised) in scratch rows
        const float* ov1 = p.qlo + (slice * p.Tp + ii) * TC_KP;
#pragma unroll
        for (int q = 0; q < 3; ++q) {
          const int c = lane + 32 * q;
          if (c >= p.dh) continue;
          float o = oacc[q];
          if (c0 > TC_KCAP) o = fmaf(orr[c], invz, o);
          if (c1 > TC_KCAP) o = fmaf(ov1[c], invz, o);
          orr[c] = o;
        }
      }
    }
  }

  // ---- teardown: an aborted CTA first waits (bounded) for its own copies and
  // MMAs in flight; then TMEM is released
  if (warp == 0 && lane == 0 && last_load >= 0) {
    for (int it = last_load; it >= 0 && it > last_load - 2; --it)
      tp_mbar_wait(&k_full[it & 1], (it >> 1) & 1, p.err);
  }
  if (warp == 1 && lane == 0 && last_mma >= 0)
    tp_mbar_wait(&acc_full[last_mma & 1], (last_mma >> 1) & 1, p.err);
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem),
                 "r"(TC_TMEM_COLS)
                 : "memory");
  }
}

bool make_feat_map(CUtensorMap* map, const float* base, int64_t rows, uint32_t box_rows) {
  EncodeTiledFn enc = encode_tiled();
  if (!enc) return false;
  cuuint64_t dims[2] = {(cuuint64_t)TC_KP, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)TC_KP * 4};
  cuuint32_t box[2] = {(cuuint32_t)TC_ATOM, box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(base), dims,
                   strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                   CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

inline int64_t round64(int64_t n) { return (n + 63) & ~(int64_t)63; }

struct TcLayout {
  int64_t Tp, Kp;
  int64_t qhi, qlo, khi, klo, qmx, kmx, log, total;   // float offsets
};

TcLayout tc_layout(int64_t B, int64_t H, int64_t T, int64_t Tkv) {
  TcLayout l;
  const int64_t S = B * H;
  l.Tp = ceil_div(T, TC_M) * TC_M;
  l.Kp = ceil_div(Tkv, TC_N) * TC_N;
  l.qhi = 0;
  l.qlo = l.qhi + round64(S * l.Tp * TC_KP);
  l.khi = l.qlo + round64(S * l.Tp * TC_KP);
  l.klo = l.khi + round64(S * l.Kp * TC_KP);
  l.qmx = l.klo + round64(S * l.Kp * TC_KP);
  l.kmx = l.qmx + round64(S * T);
  l.log = l.kmx + round64(S * l.Kp);
  l.total = l.log + round64(S * (l.Tp / TC_M) * 2 * TC_LOGCAP * TC_M * 2);
  return l;
}

}  // namespace

int& tsrn_attention_path() {
  static int mode = TP_ATT_PATH_AUTO;
  return mode;
}

bool tsrn_attention_tc_supported(int64_t dh, int top_k) {
  return dh >= 1 && dh <= TC_MAX_DH && top_k >= 1 && top_k <= TC_LIST;
}

int64_t tsrn_attention_tc_workspace_floats(int64_t B, int64_t H, int64_t T, int64_t Tkv) {
  return tc_layout(B, H, T, Tkv).total;
}

int launch_tsrn_attention_tc(int64_t B, int64_t H, int64_t T, int64_t Tkv, int64_t Tc, int64_t dh,
                             const float* Q, const float* K, const float* V, const float* slopes,
                             int top_k, int causal, float* out, float* ws, cudaStream_t stream,
                             int* kj, float* kp, float* kl, int* kn) {
  const TcLayout l = tc_layout(B, H, T, Tkv);
  const int64_t S = B * H;
  if (S * (l.Tp > l.Kp ? l.Tp : l.Kp) >= ((int64_t)1 << 31)) return TP_ERR_TOO_LARGE;
  if (S * (l.Tp / TC_M) >= ((int64_t)1 << 31)) return TP_ERR_TOO_LARGE;
  if (S > 65535) return TP_ERR_TOO_LARGE;
  float* qhi = ws + l.qhi;
  float* qlo = ws + l.qlo;
  float* khi = ws + l.khi;
  float* klo = ws + l.klo;
  float* qmx = ws + l.qmx;
  float* kmx = ws + l.kmx;
  att_tc_feat_kernel<<<dim3((unsigned)ceil_div(l.Tp, 8), (unsigned)S), 256, 0, stream>>>(
      Q, T, l.Tp, (int)dh, qhi, qlo, qmx, T);
  att_tc_feat_kernel<<<dim3((unsigned)ceil_div(l.Kp, 8), (unsigned)S), 256, 0, stream>>>(
      K, Tkv, l.Kp, (int)dh, khi, klo, kmx, l.Kp);
  int s = launch_status();
  if (s != TP_OK) return s;
  CUtensorMap mqh, mql, mkh, mkl;
  if (!make_feat_map(&mqh, qhi, S * l.Tp, TC_M) || !make_feat_map(&mql, qlo, S * l.Tp, TC_M) ||
      !make_feat_map(&mkh, khi, S * l.Kp, TC_N) || !make_feat_map(&mkl, klo, S * l.Kp, TC_N))
    return TP_ERR_UNSUPPORTED;
  TcArgs a{S, H, T, Tkv, Tc, l.Tp, l.Kp, (int)dh, top_k, causal, (int)ceil_div(dh, 8),
           Q, K, V, slopes, qmx, kmx, out, qlo, kj, kp, kl, kn,
           reinterpret_cast<float2*>(ws + l.log), device_error_ptr()};
  cudaError_t e = cudaFuncSetAttribute(att_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)TC_SMEM_BYTES);
  if (e != cudaSuccess) return cuda_status(e);
  att_tc_kernel<<<(unsigned)(S * (l.Tp / TC_M)), TC_THREADS, TC_SMEM_BYTES, stream>>>(mqh, mql, mkh,
                                                                                     mkl, a);
  return launch_status();
}

}  // namespace tp
