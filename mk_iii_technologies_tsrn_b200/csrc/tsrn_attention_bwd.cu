// tsrn_attention_bwd.cu -- sparse backward of the fused TSRN top-k attention
// (the autograd of research/tsrn_dml.py:438-460 and :509-524, with the top-k
// threshold detached as the reference detaches it).
//
// Only the kept keys of a row carry weight, so the backward runs over the
// lists the forward saved (key j and softmax weight P of each kept (i, j);
// about top_k per row) instead of over T x Tkv scores:
//   dP_ij = dO_i . V_j,   dS_ij = P_ij (dP_ij - sum_k P_ik dP_ik),
//   L_ij  = logsumexp_c(Q_ic + K_jc)  (the score before ALiBi),
//   g_ij[c] = exp(Q_ic + K_jc - L_ij)  (d L_ij / d Q_ic = d L_ij / d K_jc),
//   dQ_i = sum_j dS_ij g_ij,   dK_j = sum_i dS_ij g_ij,   dV_j = sum_i P_ij dO_i.
// Three kernels, all deterministic:
//   rows: one warp per query row (lanes split the channels) forms dP, dS and
//         dQ_i, and stores dS per list entry (L comes with the lists: the
//         forward's own score, its ALiBi term added back);
//   group: one CTA per slice groups the list entries by key, rows ascending
//         inside a key (a stable counting sort in shared memory);
//   keys: one warp per key walks the entries that kept it in that order and
//         forms dK_j and dV_j, recomputing g from Q_i, K_j and L.
#include "maxplus_internal.cuh"

namespace tp {

namespace {

constexpr int AB_L = TSRN_ATT_LIST;   // list entries per row
constexpr int AB_MAX_DH = 96;         // three channels per lane


struct AttBwdArgs {
  int64_t S, T, Tkv;
  int dh;
  const float* Q;     // [S][T][dh]
  const float* K;     // [S][Tkv][dh]
  const float* V;     // [S][Tkv][dh]
  const float* dO;    // [S][T][dh]
  const int* kj;      // [S*T][AB_L]
  const float* kp;    // [S*T][AB_L]
  const float* kl;    // [S*T][AB_L]: L_ij, saved by the forward
  const int* kn;      // [S*T]
  float* dQ;          // [S][T][dh]
  float* eds;         // [S*T][AB_L]
};

// Sums of four per-lane values over the warp, every lane receiving all four:
// two halving exchanges leave each eight-lane group with one of the values,
// three butterflies finish it, four broadcasts return the totals.
__device__ __forceinline__ void warp_sum4(float (&v)[4]) {
  const int lane = threadIdx.x & 31;
  const bool h16 = (lane & 16) != 0, h8 = (lane & 8) != 0;
  float a = h16 ? v[2] : v[0], b = h16 ? v[3] : v[1];
  a += __shfl_xor_sync(0xffffffffu, h16 ? v[0] : v[2], 16);
  b += __shfl_xor_sync(0xffffffffu, h16 ? v[1] : v[3], 16);
  float c = h8 ? b : a;
  c += __shfl_xor_sync(0xffffffffu, h8 ? a : b, 8);
  c += __shfl_xor_sync(0xffffffffu, c, 4);
  c += __shfl_xor_sync(0xffffffffu, c, 2);
  c += __shfl_xor_sync(0xffffffffu, c, 1);
#pragma unroll
  for (int e = 0; e < 4; ++e) v[e] = __shfl_sync(0xffffffffu, c, (e >> 1) * 16 + (e & 1) * 8);
}

__global__ void __launch_bounds__(256) att_bwd_rows_kernel(const AttBwdArgs a) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * 8 + warp;
  if (row >= a.S * a.T) return;
  const int64_t slice = row / a.T;
  const int n = min(max(a.kn[row], 0), AB_L);
  float qi[3], gi[3];
#pragma unroll
  for (int q = 0; q < 3; ++q) {
    const int c = lane + 32 * q;
    qi[q] = c < a.dh ? a.Q[row * a.dh + c] : 0.0f;
    gi[q] = c < a.dh ? a.dO[row * a.dh + c] : 0.0f;
  }
  const int* jr = a.kj + row * AB_L;
  const float* pr = a.kp + row * AB_L;
  const float* lr = a.kl + row * AB_L;
  const float* Ks = a.K + slice * a.Tkv * a.dh;
  const float* Vs = a.V + slice * a.Tkv * a.dh;
  // pass A: dP of every entry, four entries' V rows in flight at a time
  float dpv[AB_L];
#pragma unroll
  for (int e0 = 0; e0 < AB_L; e0 += 4) {
    if (e0 >= n) {
#pragma unroll
      for (int e = 0; e < 4; ++e) dpv[e0 + e] = 0.0f;
      continue;
    }
    float part[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      int j = e0 + e < n ? jr[e0 + e] : -1;
      if (j >= a.Tkv) j = -1;     // a key past the slice (not from the forward): no entry
      float d = 0.0f;
#pragma unroll
      for (int q = 0; q < 3; ++q) {
        const int c = lane + 32 * q;
        if (j >= 0 && c < a.dh) d = fmaf(gi[q], __ldg(Vs + (int64_t)j * a.dh + c), d);
      }
      part[e] = d;
    }
    warp_sum4(part);
#pragma unroll
    for (int e = 0; e < 4; ++e) dpv[e0 + e] = part[e];
  }
  float spd = 0.0f;
#pragma unroll
  for (int e = 0; e < AB_L; ++e)
    if (e < n) spd = fmaf(pr[e], dpv[e], spd);
  // pass B: dS and dQ_i = sum_j dS_ij exp(Q_i + K_j - L_ij)
  float dq[3] = {0.0f, 0.0f, 0.0f};
  float my_ds = 0.0f;
#pragma unroll
  for (int e0 = 0; e0 < AB_L; e0 += 4) {
    if (e0 >= n) break;
    float kv[4][3];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      int j = e0 + e < n ? jr[e0 + e] : -1;
      if (j >= a.Tkv) j = -1;
#pragma unroll
      for (int q = 0; q < 3; ++q) {
        const int c = lane + 32 * q;
        kv[e][q] = (j >= 0 && c < a.dh) ? __ldg(Ks + (int64_t)j * a.dh + c) : 0.0f;
      }
    }
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      if (e0 + e >= n) continue;
      const float ds = pr[e0 + e] * (dpv[e0 + e] - spd);
      const float L = lr[e0 + e];
#pragma unroll
      for (int q = 0; q < 3; ++q)
        if (lane + 32 * q < a.dh) dq[q] = fmaf(ds, expf(qi[q] + kv[e][q] - L), dq[q]);
      if (lane == e0 + e) my_ds = ds;
    }
  }
#pragma unroll
  for (int q = 0; q < 3; ++q) {
    const int c = lane + 32 * q;
    if (c < a.dh) a.dQ[row * a.dh + c] = dq[q];
  }
  if (lane < AB_L) a.eds[row * AB_L + lane] = lane < n ? my_ds : 0.0f;
}

struct AttBwdKeyArgs {
  int64_t S, T, Tkv;
  int dh;
  const float* Q;
  const float* K;
  const float* dO;
  const float* kp;
  const float* eds;
  const float* kl;
  const int* order;        // entry ids (row * AB_L + e) grouped by key, rows ascending
  const int* key_begin;    // [S * Tkv]: key (slice, j)'s entries are order[begin, begin + count)
  const int* key_count;    // [S * Tkv]
  float* dK;
  float* dV;
};

__global__ void __launch_bounds__(256) att_bwd_keys_kernel(const AttBwdKeyArgs a) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t key = (int64_t)blockIdx.x * 8 + warp;
  if (key >= a.S * a.Tkv) return;
  const int64_t beg = a.key_begin[key], end = beg + a.key_count[key];
  float kq[3], dk[3] = {0.0f, 0.0f, 0.0f}, dv[3] = {0.0f, 0.0f, 0.0f};
#pragma unroll
  for (int q = 0; q < 3; ++q) {
    const int c = lane + 32 * q;
    kq[q] = c < a.dh ? a.K[key * a.dh + c] : 0.0f;
  }
  for (int64_t b0 = beg; b0 < end; b0 += 4) {
    float qv[4][3], gv[4][3], ds[4], P[4], L[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const bool ok = b0 + e < end;
      const int ent = ok ? a.order[b0 + e] : 0;
      const int64_t row = ent / AB_L;
      ds[e] = ok ? a.eds[ent] : 0.0f;
      P[e] = ok ? a.kp[ent] : 0.0f;
      L[e] = ok ? a.kl[ent] : 0.0f;
#pragma unroll
      for (int q = 0; q < 3; ++q) {
        const int c = lane + 32 * q;
        const bool in = ok && c < a.dh;
        qv[e][q] = in ? __ldg(a.Q + row * a.dh + c) : 0.0f;
        gv[e][q] = in ? __ldg(a.dO + row * a.dh + c) : 0.0f;
      }
    }
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      if (b0 + e >= end) break;
#pragma unroll
      for (int q = 0; q < 3; ++q) {
        if (lane + 32 * q >= a.dh) continue;
        dk[q] = fmaf(ds[e], expf(qv[e][q] + kq[q] - L[e]), dk[q]);
        dv[q] = fmaf(P[e], gv[e][q], dv[q]);
      }
    }
  }
#pragma unroll
  for (int q = 0; q < 3; ++q) {
    const int c = lane + 32 * q;
    if (c < a.dh) {
      a.dK[key * a.dh + c] = dk[q];
      a.dV[key * a.dh + c] = dv[q];
    }
  }
}

// Groups the list entries of each slice by key, rows ascending inside a key
// (a stable counting sort; deterministic): one CTA of 1024 threads per
// slice.  The slice's entries go to its own segment of `order`
// ([slice * T * AB_L, +T * AB_L)); key_begin / key_count locate each key's run.
// Shared memory: count, cursor and a row mask per key (3 * Tkv words).
constexpr int AB_GROUP_THREADS = 1024;
constexpr int AB_GROUP_ROWS = AB_GROUP_THREADS / AB_L;   // rows per chunk (32)

__global__ void __launch_bounds__(AB_GROUP_THREADS) att_bwd_group_kernel(
    int64_t T, int64_t Tkv, const int* __restrict__ kj, int* __restrict__ order,
    int* __restrict__ key_begin, int* __restrict__ key_count) {
  extern __shared__ int ab_sm[];
  int* cnt = ab_sm;                                   // [Tkv]
  int* cur = ab_sm + Tkv;                             // [Tkv]
  unsigned* msk = reinterpret_cast<unsigned*>(ab_sm + 2 * Tkv);   // [Tkv]
  __shared__ int part[AB_GROUP_THREADS / 32];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int64_t slice = blockIdx.x;
  const int* kjs = kj + slice * T * AB_L;
  for (int64_t k = tid; k < Tkv; k += AB_GROUP_THREADS) cnt[k] = 0;
  __syncthreads();
  for (int64_t e = tid; e < T * AB_L; e += AB_GROUP_THREADS) {
    const int j = kjs[e];
    if (j >= 0 && j < Tkv) atomicAdd(&cnt[j], 1);   // counts do not depend on the order
  }
  __syncthreads();
  // exclusive scan of cnt: each thread a contiguous run of keys, then the
  // threads' totals across the block
  const int64_t per = (Tkv + AB_GROUP_THREADS - 1) / AB_GROUP_THREADS;
  const int64_t k0 = tid * per, k1 = min(k0 + per, Tkv);
  int run = 0;
  for (int64_t k = k0; k < k1; ++k) run += cnt[k];
  int incl = run;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int v = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += v;
  }
  if (lane == 31) part[warp] = incl;
  __syncthreads();
  if (warp == 0) {
    int v = part[lane];
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int u = __shfl_up_sync(0xffffffffu, v, o);
      if (lane >= o) v += u;
    }
    part[lane] = v;                          // inclusive over warps
  }
  __syncthreads();
  int base = incl - run + (warp > 0 ? part[warp - 1] : 0);
  const int seg = (int)(slice * T * AB_L);
  for (int64_t k = k0; k < k1; ++k) {
    cur[k] = base;
    key_begin[slice * Tkv + k] = seg + base;
    key_count[slice * Tkv + k] = cnt[k];
    base += cnt[k];
  }
  __syncthreads();
  // stable placement, AB_GROUP_ROWS rows at a time: a key's rank among the
  // chunk's rows that kept it is the number of lower rows in its row mask
  const int rr = tid / AB_L, slot = tid % AB_L;
  for (int64_t r0 = 0; r0 < T; r0 += AB_GROUP_ROWS) {
    for (int64_t k = tid; k < Tkv; k += AB_GROUP_THREADS) msk[k] = 0u;
    __syncthreads();
    const int64_t row = r0 + rr;
    int j = row < T ? kjs[row * AB_L + slot] : -1;
    if (j >= Tkv) j = -1;               // a key past the slice: not an entry
    if (j >= 0) atomicOr(&msk[j], 1u << rr);
    __syncthreads();
    unsigned m = 0u;
    if (j >= 0) {
      m = msk[j];
      const int rank = __popc(m & ((1u << rr) - 1u));
      order[seg + cur[j] + rank] = (int)((slice * T + row) * AB_L + slot);
    }
    __syncthreads();
    if (j >= 0 && (m & ((1u << rr) - 1u)) == 0u) cur[j] += __popc(m);   // the chunk's lowest row
    __syncthreads();
  }
}

}  // namespace

int launch_tsrn_attention_bwd_rows(int64_t S, int64_t T, int64_t Tkv, int64_t dh, const float* Q,
                                   const float* K, const float* V, const float* dO,
                                   const int* kj, const float* kp, const float* kl,
                                   const int* kn, float* dQ, float* eds, cudaStream_t stream) {
  if (S * T == 0) return TP_OK;
  if (dh < 1 || dh > AB_MAX_DH) return TP_ERR_UNSUPPORTED;
  const int64_t blocks = ceil_div(S * T, (int64_t)8);
  if (blocks > INT32_MAX || S * T * AB_L > INT32_MAX) return TP_ERR_TOO_LARGE;
  AttBwdArgs a{S, T, Tkv, (int)dh, Q, K, V, dO, kj, kp, kl, kn, dQ, eds};
  att_bwd_rows_kernel<<<(unsigned)blocks, 256, 0, stream>>>(a);
  return launch_status();
}

int launch_tsrn_attention_bwd_group(int64_t S, int64_t T, int64_t Tkv, const int* kj, int* order,
                                    int* key_begin, int* key_count, cudaStream_t stream) {
  if (S * Tkv == 0) return TP_OK;
  if (S > INT32_MAX || S * T * AB_L > INT32_MAX) return TP_ERR_TOO_LARGE;
  const size_t smem = (size_t)3 * Tkv * sizeof(int);
  if (smem > 200 * 1024) return TP_ERR_TOO_LARGE;   // Tkv up to ~17000 keys
  cudaError_t e = cudaFuncSetAttribute(att_bwd_group_kernel,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return cuda_status(e);
  att_bwd_group_kernel<<<(unsigned)S, AB_GROUP_THREADS, smem, stream>>>(T, Tkv, kj, order,
                                                                      key_begin, key_count);
  return launch_status();
}

int launch_tsrn_attention_bwd_keys(int64_t S, int64_t T, int64_t Tkv, int64_t dh, const float* Q,
                                   const float* K, const float* dO, const float* kp,
                                   const float* eds, const float* kl, const int* order,
                                   const int* key_begin, const int* key_count, float* dK,
                                   float* dV, cudaStream_t stream) {
  if (S * Tkv == 0) return TP_OK;
  if (dh < 1 || dh > AB_MAX_DH) return TP_ERR_UNSUPPORTED;
  const int64_t blocks = ceil_div(S * Tkv, (int64_t)8);
  if (blocks > INT32_MAX || S * T * AB_L > INT32_MAX) return TP_ERR_TOO_LARGE;
  AttBwdKeyArgs a{S, T, Tkv, (int)dh, Q, K, dO, kp, eds, kl, order, key_begin, key_count, dK, dV};
  att_bwd_keys_kernel<<<(unsigned)blocks, 256, 0, stream>>>(a);
  return launch_status();
}

}  // namespace tp
