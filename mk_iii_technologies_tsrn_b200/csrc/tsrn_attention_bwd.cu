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
// Two kernels, both deterministic:
//   rows: one warp per query row (lanes split the channels) forms dP, dS, L
//         and dQ_i, and stores dS and L per list entry;
//   keys: one warp per key walks the entries that kept it in ascending row
//         order (the host sorts the entries by key, stably) and forms dK_j
//         and dV_j, recomputing g from Q_i, K_j and L.
#include "maxplus_internal.cuh"

namespace tp {

namespace {

constexpr int AB_L = TSRN_ATT_LIST;   // list entries per row
constexpr int AB_MAX_DH = 96;         // three channels per lane

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

struct AttBwdArgs {
  int64_t S, T, Tkv;
  int dh;
  const float* Q;     // [S][T][dh]
  const float* K;     // [S][Tkv][dh]
  const float* V;     // [S][Tkv][dh]
  const float* dO;    // [S][T][dh]
  const int* kj;      // [S*T][AB_L]
  const float* kp;    // [S*T][AB_L]
  const int* kn;      // [S*T]
  float* dQ;          // [S][T][dh]
  float* eds;         // [S*T][AB_L]
  float* eL;          // [S*T][AB_L]
};

__global__ void __launch_bounds__(256) att_bwd_rows_kernel(const AttBwdArgs a) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t row = (int64_t)blockIdx.x * 8 + warp;
  if (row >= a.S * a.T) return;
  const int64_t slice = row / a.T;
  const float NEG_INF = -__int_as_float(0x7f800000);
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
  const float* Ks = a.K + slice * a.Tkv * a.dh;
  const float* Vs = a.V + slice * a.Tkv * a.dh;
  // pass A: dP and L of every entry (four entries' rows in flight at a time)
  float dpv[AB_L], Lv[AB_L];
#pragma unroll
  for (int e0 = 0; e0 < AB_L; e0 += 4) {
    if (e0 >= n) {
#pragma unroll
      for (int e = 0; e < 4; ++e) dpv[e0 + e] = Lv[e0 + e] = 0.0f;
      continue;
    }
    float kv[4][3], vv[4][3];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int j = e0 + e < n ? jr[e0 + e] : -1;
#pragma unroll
      for (int q = 0; q < 3; ++q) {
        const int c = lane + 32 * q;
        const bool ok = j >= 0 && c < a.dh;
        kv[e][q] = ok ? __ldg(Ks + (int64_t)j * a.dh + c) : 0.0f;
        vv[e][q] = ok ? __ldg(Vs + (int64_t)j * a.dh + c) : 0.0f;
      }
    }
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      float dp = 0.0f, m = NEG_INF;
#pragma unroll
      for (int q = 0; q < 3; ++q) {
        dp = fmaf(gi[q], vv[e][q], dp);
        if (lane + 32 * q < a.dh) m = fmaxf(m, qi[q] + kv[e][q]);
      }
      dp = warp_sum(dp);
      m = warp_max(m);
      float z = 0.0f;
#pragma unroll
      for (int q = 0; q < 3; ++q)
        if (lane + 32 * q < a.dh) z += expf(qi[q] + kv[e][q] - m);
      z = warp_sum(z);
      dpv[e0 + e] = dp;
      Lv[e0 + e] = m + logf(z);
    }
  }
  float spd = 0.0f;
#pragma unroll
  for (int e = 0; e < AB_L; ++e)
    if (e < n) spd = fmaf(pr[e], dpv[e], spd);
  // pass B: dS and dQ_i
  float dq[3] = {0.0f, 0.0f, 0.0f};
  float my_ds = 0.0f, my_L = 0.0f;
#pragma unroll
  for (int e0 = 0; e0 < AB_L; e0 += 4) {
    if (e0 >= n) break;
    float kv[4][3];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int j = e0 + e < n ? jr[e0 + e] : -1;
#pragma unroll
      for (int q = 0; q < 3; ++q) {
        const int c = lane + 32 * q;
        kv[e][q] = (j >= 0 && c < a.dh) ? __ldg(Ks + (int64_t)j * a.dh + c) : 0.0f;
      }
    }
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      if (e0 + e >= n) continue;
      const float P = pr[e0 + e];
      const float ds = P * (dpv[e0 + e] - spd);
#pragma unroll
      for (int q = 0; q < 3; ++q)
        if (lane + 32 * q < a.dh) dq[q] = fmaf(ds, expf(qi[q] + kv[e][q] - Lv[e0 + e]), dq[q]);
      if (lane == e0 + e) {
        my_ds = ds;
        my_L = Lv[e0 + e];
      }
    }
  }
#pragma unroll
  for (int q = 0; q < 3; ++q) {
    const int c = lane + 32 * q;
    if (c < a.dh) a.dQ[row * a.dh + c] = dq[q];
  }
  if (lane < AB_L) {
    a.eds[row * AB_L + lane] = lane < n ? my_ds : 0.0f;
    a.eL[row * AB_L + lane] = lane < n ? my_L : 0.0f;
  }
}

struct AttBwdKeyArgs {
  int64_t S, T, Tkv;
  int dh;
  const float* Q;
  const float* K;
  const float* dO;
  const float* kp;
  const float* eds;
  const float* eL;
  const int* order;        // entry ids (row * AB_L + e) sorted by key, rows ascending
  const int64_t* offsets;  // [S * Tkv + 1]: entries of key (slice, j) in order[off[k], off[k+1])
  float* dK;
  float* dV;
};

__global__ void __launch_bounds__(256) att_bwd_keys_kernel(const AttBwdKeyArgs a) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t key = (int64_t)blockIdx.x * 8 + warp;
  if (key >= a.S * a.Tkv) return;
  const int64_t beg = a.offsets[key], end = a.offsets[key + 1];
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
      L[e] = ok ? a.eL[ent] : 0.0f;
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

}  // namespace

int launch_tsrn_attention_bwd_rows(int64_t S, int64_t T, int64_t Tkv, int64_t dh, const float* Q,
                                   const float* K, const float* V, const float* dO,
                                   const int* kj, const float* kp, const int* kn, float* dQ,
                                   float* eds, float* eL, cudaStream_t stream) {
  if (S * T == 0) return TP_OK;
  if (dh < 1 || dh > AB_MAX_DH) return TP_ERR_UNSUPPORTED;
  const int64_t blocks = ceil_div(S * T, (int64_t)8);
  if (blocks > INT32_MAX || S * T * AB_L > INT32_MAX) return TP_ERR_TOO_LARGE;
  AttBwdArgs a{S, T, Tkv, (int)dh, Q, K, V, dO, kj, kp, kn, dQ, eds, eL};
  att_bwd_rows_kernel<<<(unsigned)blocks, 256, 0, stream>>>(a);
  return launch_status();
}

int launch_tsrn_attention_bwd_keys(int64_t S, int64_t T, int64_t Tkv, int64_t dh, const float* Q,
                                   const float* K, const float* dO, const float* kp,
                                   const float* eds, const float* eL, const int* order,
                                   const int64_t* offsets, float* dK, float* dV,
                                   cudaStream_t stream) {
  if (S * Tkv == 0) return TP_OK;
  if (dh < 1 || dh > AB_MAX_DH) return TP_ERR_UNSUPPORTED;
  const int64_t blocks = ceil_div(S * Tkv, (int64_t)8);
  if (blocks > INT32_MAX || S * T * AB_L > INT32_MAX) return TP_ERR_TOO_LARGE;
  AttBwdKeyArgs a{S, T, Tkv, (int)dh, Q, K, dO, kp, eds, eL, order, offsets, dK, dV};
  att_bwd_keys_kernel<<<(unsigned)blocks, 256, 0, stream>>>(a);
  return launch_status();
}

}  // namespace tp
