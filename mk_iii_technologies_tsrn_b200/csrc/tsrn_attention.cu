// tsrn_attention.cu -- fused TSRN tropical top-k attention forward (inference).
//
// Replaces, for one TropicalAttention call (research/tsrn_dml.py:462-548), the
// score and attention steps after the Q/K/V projections, QK-norm and RoPE:
//   S[i,j]  = logsumexp_c(Q[i,c] + K[j,c])                      (:438-460)
//           - slope[h] * |i - (j - Tc)|                         ALiBi (:509-514)
//           = -inf where causal and j - Tc > i                  (:516-518)
//   thr_i   = top_k-th largest S[i,:] (ties counted)            (:520-521)
//   out[i]  = softmax over {j : S[i,j] >= thr_i} of S  @ V      (:522-524)
// Keys j < Tc are cached keys at positions j - Tc < 0 (cross-window memory).
//
// The log-sum-exp over channels factorises: with qmax_i = max_c Q[i,c] and
// kmax_j = max_c K[j,c],
//   S[i,j] = log( sum_c exp(Q[i,c]-qmax_i) * exp(K[j,c]-kmax_j) ) + qmax_i + kmax_j,
// an fp32 dot product of "exp features" (each factor in (0, 1], one of them 1
// per row).  A pre-pass computes the features once per row (2*(T+Tkv)*dh
// exps per head instead of T*Tkv*dh); the main kernel forms the dots on CUDA
// cores.  A dot below 1e-30 (possible only when every channel pair is far
// below its row maxima) is recomputed exactly with a max-shifted sum.
//
// Main kernel: one CTA per R (16, or 8 when shared memory is short) query
// rows of one (b, h).  Key tiles of 64
// feature columns are double-buffered with cp.async; the CTA keeps its R x Tkv
// score block in shared memory.  Then each warp takes R/8 rows: each lane
// keeps its 4 largest scores and the warp pops the overall largest top_k times
// (the last popped value is the k-th largest, ties counted); a row where one
// lane held more than 4 of the top_k falls back to exact rounds (count the
// current value, find the next smaller one).  The kept scores' softmax
// weights are formed and the weighted V rows gathered (the kept entries are
// broadcast one at a time; lanes split the dh channels).
#include "maxplus_internal.cuh"

namespace tp {

namespace {

constexpr int ATT_THREADS = 256;
constexpr int ATT_KT = 64;          // keys per feature tile
constexpr int ATT_MAX_DH = 128;
constexpr int ATT_MAX_TOPK = 64;
constexpr int ATT_MAX_TKV = 6144;   // scores held in shared memory

// exp features of one [rows x dh] matrix: F^T[c][r] = exp(X[r,c] - max_c X[r,:]),
// mx[r] = that max.  Block: 32 rows of one (b,h) slice; transposed through smem.
__global__ void __launch_bounds__(ATT_THREADS)
    att_expfeat_kernel(const float* __restrict__ X, int64_t rows, int dh, float* __restrict__ FT,
                       float* __restrict__ mx) {
  __shared__ float tile[32][ATT_MAX_DH + 1];
  const int64_t slice = blockIdx.y;                       // (b, h)
  const int64_t r0 = (int64_t)blockIdx.x * 32;
  const float* Xs = X + slice * rows * dh;
  float* Fs = FT + slice * rows * dh;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const float NEG_INF = -__int_as_float(0x7f800000);
  for (int rr = warp; rr < 32; rr += ATT_THREADS / 32) {
    const int64_t r = r0 + rr;
    float v[ATT_MAX_DH / 32];
    float m = NEG_INF;
#pragma unroll
    for (int u = 0; u < ATT_MAX_DH / 32; ++u) {
      const int c = lane + 32 * u;
      v[u] = (r < rows && c < dh) ? Xs[r * dh + c] : NEG_INF;
      m = fmaxf(m, v[u]);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
#pragma unroll
    for (int u = 0; u < ATT_MAX_DH / 32; ++u) {
      const int c = lane + 32 * u;
      if (c < dh) tile[rr][c] = (r < rows) ? expf(v[u] - m) : 0.0f;
    }
    if (lane == 0 && r < rows) mx[slice * rows + r] = m;
  }
  __syncthreads();
  // transposed store: for each channel, 32 consecutive rows
  for (int e = threadIdx.x; e < dh * 32; e += ATT_THREADS) {
    const int c = e / 32, rr = e % 32;
    const int64_t r = r0 + rr;
    if (r < rows) Fs[(int64_t)c * rows + r] = tile[rr][c];
  }
}

struct AttArgs {
  int64_t B, H, T, Tkv, Tc;
  int dh, top_k, causal;
  const float* Q;      // raw, for the exact fallback
  const float* K;
  const float* V;
  const float* slopes;
  const float* AT;     // [B*H][dh][T]   query exp features (transposed)
  const float* qmx;    // [B*H][T]
  const float* BT;     // [B*H][dh][Tkv] key exp features (transposed)
  const float* kmx;    // [B*H][Tkv]
  float* out;          // [B*H][T][dh]
};

// R query rows per CTA; thread tile RM rows x KN keys (8 x 32 thread grid).
// PL > 0: each lane holds its PL scores of a row in registers for the selection
// (Tkv <= 32*PL); PL == 0 reads them from shared memory.
template <int R, int PL>
__global__ void __launch_bounds__(ATT_THREADS) att_fwd_kernel(AttArgs p) {
  constexpr int RM = R / 8;       // rows per thread in the score tile
  constexpr int KN = ATT_KT / 32; // keys per thread (2)
  extern __shared__ __align__(16) float att_smem[];
  const int dh = p.dh;
  const int64_t Tkv = p.Tkv;
  const int tkv_pad = (int)((Tkv + 3) & ~(int64_t)3);
  float* At = att_smem;                                  // [dh][R]
  float* Bt = At + dh * R;                               // [2][dh][ATT_KT]
  float* S = Bt + 2 * dh * ATT_KT;                       // [R][tkv_pad]

  const int64_t slice = (int64_t)blockIdx.z * p.H + blockIdx.y;
  const int h = blockIdx.y;
  const int64_t i0 = (int64_t)blockIdx.x * R;
  const float* AT = p.AT + slice * dh * p.T;
  const float* BT = p.BT + slice * dh * Tkv;
  const float* qmx = p.qmx + slice * p.T;
  const float* kmx = p.kmx + slice * Tkv;
  const float slope = p.slopes[h];
  const float NEG_INF = -__int_as_float(0x7f800000);
  const int tid = threadIdx.x;

  // query features of this CTA's rows
  for (int e = tid; e < dh * R; e += ATT_THREADS) {
    const int c = e / R, rr = e % R;
    At[e] = (i0 + rr < p.T) ? AT[(int64_t)c * p.T + i0 + rr] : 0.0f;
  }
  // keys this CTA needs: all, or (causal) up to the last row's position
  int64_t kv_end = Tkv;
  if (p.causal) {
    const int64_t last_row = (i0 + R - 1 < p.T) ? i0 + R - 1 : p.T - 1;
    kv_end = last_row + p.Tc + 1 < Tkv ? last_row + p.Tc + 1 : Tkv;
  }
  const int ntiles = (int)((kv_end + ATT_KT - 1) / ATT_KT);

  // feature tile of keys [k0, k0+64) -> buffer b: 16-byte cp.async when the
  // feature rows are 16-byte aligned (Tkv % 4 == 0), 4-byte copies otherwise
  const bool vec = (Tkv % 4) == 0;
  auto issue = [&](int b, int t) {
    const int64_t k0 = (int64_t)t * ATT_KT;
    float* dst = Bt + b * dh * ATT_KT;
    if (vec) {
      for (int e = tid; e < dh * (ATT_KT / 4); e += ATT_THREADS) {
        const int c = e / (ATT_KT / 4), kv = e % (ATT_KT / 4);
        const int64_t k = k0 + 4 * kv;
        const bool ok = k < Tkv;
        tp_cp_async16(dst + c * ATT_KT + 4 * kv, ok ? BT + (int64_t)c * Tkv + k : BT,
                      ok ? 16 : 0);
      }
    } else {
      for (int e = tid; e < dh * ATT_KT; e += ATT_THREADS) {
        const int c = e / ATT_KT, kv = e % ATT_KT;
        const int64_t k = k0 + kv;
        const bool ok = k < Tkv;
        tp_cp_async4(dst + c * ATT_KT + kv, ok ? BT + (int64_t)c * Tkv + k : BT, ok ? 4 : 0);
      }
    }
    tp_cp_async_commit();
  };

  const int ty = tid / 32;         // row group: rows RM*ty .. RM*ty+RM-1
  const int tx = tid % 32;         // keys KN*tx .. KN*tx+KN-1 of the tile
  if (ntiles > 0) issue(0, 0);
  for (int t = 0; t < ntiles; ++t) {
    const int b = t & 1;
    if (t + 1 < ntiles) {
      issue(b ^ 1, t + 1);
      tp_cp_async_wait<1>();
    } else {
      tp_cp_async_wait<0>();
    }
    __syncthreads();
    const float* Bb = Bt + b * dh * ATT_KT;
    float acc[RM][KN];
#pragma unroll
    for (int r = 0; r < RM; ++r)
#pragma unroll
      for (int q = 0; q < KN; ++q) acc[r][q] = 0.0f;
#pragma unroll 4
    for (int c = 0; c < dh; ++c) {
      float a[RM];
#pragma unroll
      for (int r = 0; r < RM; ++r) a[r] = At[c * R + RM * ty + r];
      const float2 bb = *reinterpret_cast<const float2*>(Bb + c * ATT_KT + KN * tx);
      const float bv[KN] = {bb.x, bb.y};
#pragma unroll
      for (int r = 0; r < RM; ++r)
#pragma unroll
        for (int q = 0; q < KN; ++q) acc[r][q] = fmaf(a[r], bv[q], acc[r][q]);
    }
    // scores -> shared memory
#pragma unroll
    for (int r = 0; r < RM; ++r) {
      const int rr = RM * ty + r;
      const int64_t i = i0 + rr;
#pragma unroll
      for (int q = 0; q < KN; ++q) {
        const int64_t j = (int64_t)t * ATT_KT + KN * tx + q;
        if (j >= Tkv || i >= p.T) continue;
        const int64_t kpos = j - p.Tc;
        float s;
        if (p.causal && kpos > i) {
          s = NEG_INF;
        } else {
          const float d = acc[r][q];
          if (d >= 1e-30f) {
            // fast log: absolute error ~1e-7 here, far inside the scores'
            // 1e-5 tolerance (one per score: the epilogue bounds this kernel)
            s = __logf(d) + qmx[i] + kmx[j];
          } else {
            // exact max-shifted log-sum-exp from the raw rows (rare)
            const float* qr = p.Q + (slice * p.T + i) * dh;
            const float* kr = p.K + (slice * Tkv + j) * dh;
            float m = NEG_INF;
            for (int c = 0; c < dh; ++c) m = fmaxf(m, qr[c] + kr[c]);
            float z = 0.0f;
            if (m > NEG_INF)
              for (int c = 0; c < dh; ++c) z += expf(qr[c] + kr[c] - m);
            s = (m > NEG_INF) ? m + logf(z) : NEG_INF;
          }
          const float dist = fabsf((float)(i - kpos));
          s = s - slope * dist;
        }
        S[rr * tkv_pad + j] = s;
      }
    }
    __syncthreads();   // buffer b is refilled by the next iteration's issue
  }

  // ---- per row: k-th largest, kept softmax weights, gather of V rows.  Lane
  // `lane` owns keys lane, lane+32, ...; keys at or past kv_end were not
  // computed and are masked by causality (-inf).
  const int warp = tid >> 5, lane = tid & 31;
  for (int rr = warp; rr < R; rr += ATT_THREADS / 32) {
    const int64_t i = i0 + rr;
    if (i >= p.T) break;
    const float* Sr = S + rr * tkv_pad;
    auto sval = [&](int64_t j) { return j < kv_end ? Sr[j] : NEG_INF; };
    const int kk = (int)((int64_t)p.top_k < Tkv ? p.top_k : Tkv);
    float thr = NEG_INF, rowmax = NEG_INF;
    float oacc[ATT_MAX_DH / 32];
#pragma unroll
    for (int u = 0; u < ATT_MAX_DH / 32; ++u) oacc[u] = 0.0f;
    const float* Vs = p.V + slice * Tkv * dh;
    // out += sum over the kept keys j = jbase + (bits of mask) of weight * V[j]:
    // four kept keys at a time, their V rows loaded before any is accumulated
    // (same order of accumulation as one key at a time)
    auto gather = [&](unsigned mask, float wl, int64_t jbase) {
      while (mask) {
        int src[4];
        float wv[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          src[e] = mask ? __ffs(mask) - 1 : -1;
          if (mask) mask &= mask - 1;
          wv[e] = __shfl_sync(0xffffffffu, wl, src[e] < 0 ? 0 : src[e]);
        }
        float val[4][ATT_MAX_DH / 32];
#pragma unroll
        for (int e = 0; e < 4; ++e)
#pragma unroll
          for (int q = 0; q < ATT_MAX_DH / 32; ++q) {
            const int c = lane + 32 * q;
            val[e][q] = (src[e] >= 0 && c < dh) ? __ldg(Vs + (jbase + src[e]) * dh + c) : 0.0f;
          }
#pragma unroll
        for (int e = 0; e < 4; ++e)
          if (src[e] >= 0)
#pragma unroll
            for (int q = 0; q < ATT_MAX_DH / 32; ++q) oacc[q] = fmaf(wv[e], val[e][q], oacc[q]);
      }
    };
    if constexpr (PL > 0) {
      // the row in registers (slots past Tkv read -inf: with at least top_k
      // real keys, extra -inf entries never change the threshold)
      float v[PL];
#pragma unroll
      for (int u = 0; u < PL; ++u) v[u] = sval(lane + 32 * (int64_t)u);
      // Fast selection: each lane keeps its 4 largest scores (sorted, NaN
      // dropped); the warp pops the overall largest top_k times, one instance
      // per pop, so the last popped value is the top_k-th largest counting
      // ties.  If a lane runs out of candidates before the last pop (it held
      // more than 4 of the top_k), the row falls back to the exact rounds below.
      constexpr int NC = 4;
      float cand[NC];
#pragma unroll
      for (int c = 0; c < NC; ++c) cand[c] = NEG_INF;
#pragma unroll
      for (int u = 0; u < PL; ++u) {
        float x = v[u];
        if (x == x) {
#pragma unroll
          for (int c = 0; c < NC; ++c) {
            const float hi = fmaxf(cand[c], x);
            x = fminf(cand[c], x);
            cand[c] = hi;
          }
        }
      }
      int popped = 0;
      bool exhausted = false;
      for (int round = 0; round < kk; ++round) {
        float wm = cand[0];
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) wm = fmaxf(wm, __shfl_xor_sync(0xffffffffu, wm, o));
        if (round == 0) rowmax = wm;
        thr = wm;
        if (wm == NEG_INF) break;                 // everything left is -inf
        const unsigned hold = __ballot_sync(0xffffffffu, cand[0] == wm);
        const int win = __ffs(hold) - 1;
        if (lane == win) {
#pragma unroll
          for (int c = 0; c < NC - 1; ++c) cand[c] = cand[c + 1];
          cand[NC - 1] = NEG_INF;
          ++popped;
        }
        // a lane that gave up all its candidates may hold more: exact path
        if (round + 1 < kk && __any_sync(0xffffffffu, popped == NC)) {
          exhausted = true;
          break;
        }
      }
      // exact rounds: count the current value, find the next smaller one; the
      // threshold is the value at which the running count reaches top_k
      float cur = NEG_INF;
      int need = kk;
      if (exhausted) {
#pragma unroll
        for (int u = 0; u < PL; ++u) cur = fmaxf(cur, v[u]);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) cur = fmaxf(cur, __shfl_xor_sync(0xffffffffu, cur, o));
        rowmax = cur;
        thr = cur;
      }
      for (int round = 0; exhausted && round < kk; ++round) {
        int cnt = 0;
        float nxt = NEG_INF;
        bool below = false;
#pragma unroll
        for (int u = 0; u < PL; ++u) {
          cnt += (v[u] == cur) ? 1 : 0;
          if (v[u] < cur) {
            nxt = fmaxf(nxt, v[u]);
            below = true;
          }
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
          cnt += __shfl_xor_sync(0xffffffffu, cnt, o);
          nxt = fmaxf(nxt, __shfl_xor_sync(0xffffffffu, nxt, o));
        }
        const bool any_below = __any_sync(0xffffffffu, below);
        thr = cur;
        if (cnt >= need || !any_below) break;
        need -= cnt;
        cur = nxt;
      }
      // kept keys (ascending j): count them; when at most ATT_MAX_TOPK, list
      // them (index, score) in this row's own score slots -- the row is in
      // registers, so the slots are free -- and form the softmax and the V
      // gather over the list only
      int nk = 0;
#pragma unroll
      for (int u = 0; u < PL; ++u) {
        const int64_t jl = lane + 32 * (int64_t)u;
        nk += __popc(__ballot_sync(0xffffffffu,
                                   jl < Tkv && !(v[u] < thr) && v[u] != NEG_INF));
      }
      if (nk <= ATT_MAX_TOPK && tkv_pad >= 2 * ATT_MAX_TOPK) {
        float* slot = S + rr * tkv_pad;          // this warp's row
        int* kidx = reinterpret_cast<int*>(slot);
        float* kval = slot + ATT_MAX_TOPK;
        __syncwarp();
        int base = 0;
#pragma unroll
        for (int u = 0; u < PL; ++u) {
          const int64_t jl = lane + 32 * (int64_t)u;
          const bool kept = jl < Tkv && !(v[u] < thr) && v[u] != NEG_INF;
          const unsigned mask = __ballot_sync(0xffffffffu, kept);
          if (kept) {
            const int pos = base + __popc(mask & ((1u << lane) - 1u));
            kidx[pos] = (int)jl;
            kval[pos] = v[u];
          }
          base += __popc(mask);
        }
        __syncwarp();
        float z = 0.0f;
        for (int e = lane; e < nk; e += 32) z += expf(kval[e] - rowmax);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) z += __shfl_xor_sync(0xffffffffu, z, o);
        const float invz = 1.0f / z;
        for (int e0 = 0; e0 < nk; e0 += 4) {
          int jj[4];
          float wv[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const bool ok = e0 + e < nk;
            jj[e] = ok ? kidx[e0 + e] : -1;
            wv[e] = ok ? expf(kval[e0 + e] - rowmax) * invz : 0.0f;
          }
          float val[4][ATT_MAX_DH / 32];
#pragma unroll
          for (int e = 0; e < 4; ++e)
#pragma unroll
            for (int q = 0; q < ATT_MAX_DH / 32; ++q) {
              const int c = lane + 32 * q;
              val[e][q] = (jj[e] >= 0 && c < dh) ? __ldg(Vs + (int64_t)jj[e] * dh + c) : 0.0f;
            }
#pragma unroll
          for (int e = 0; e < 4; ++e)
            if (jj[e] >= 0)
#pragma unroll
              for (int q = 0; q < ATT_MAX_DH / 32; ++q) oacc[q] = fmaf(wv[e], val[e][q], oacc[q]);
        }
      } else {
        float z = 0.0f;
#pragma unroll
        for (int u = 0; u < PL; ++u)
          if (!(v[u] < thr) && v[u] != NEG_INF) z += expf(v[u] - rowmax);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) z += __shfl_xor_sync(0xffffffffu, z, o);
        const float invz = 1.0f / z;
#pragma unroll
        for (int u = 0; u < PL; ++u) {
          const int64_t jl = lane + 32 * (int64_t)u;
          const bool kept = jl < Tkv && !(v[u] < thr) && v[u] != NEG_INF;
          const unsigned mask = __ballot_sync(0xffffffffu, kept);
          const float wl = kept ? expf(v[u] - rowmax) * invz : 0.0f;
          gather(mask, wl, 32 * (int64_t)u);
        }
      }
    } else {
    // threshold: top_k-th largest value, ties counted (torch.topk(k)[..., -1])
    int need = kk;
    float ub = __int_as_float(0x7f800000);     // values strictly below ub remain
    bool first = true;
    for (int round = 0; round < kk; ++round) {
      float m = NEG_INF;
      bool any = false;
      for (int64_t j = lane; j < Tkv; j += 32) {
        const float v = sval(j);
        if (v < ub || (first && v == ub)) {    // (first round: +inf scores count)
          if (!any || v > m) m = v;
          any = true;
        }
      }
      const int wany = __any_sync(0xffffffffu, any);
      float wm = any ? m : NEG_INF;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) wm = fmaxf(wm, __shfl_xor_sync(0xffffffffu, wm, o));
      if (!wany) break;                         // only NaN left
      int cnt = 0;
      for (int64_t j = lane; j < Tkv; j += 32) cnt += (sval(j) == wm) ? 1 : 0;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) cnt += __shfl_xor_sync(0xffffffffu, cnt, o);
      if (first) rowmax = wm;
      first = false;
      thr = wm;
      if (cnt >= need) break;
      need -= cnt;
      ub = wm;
      if (wm == NEG_INF) break;                 // everything left is -inf
    }
    // softmax over kept scores (kept: not below thr, so NaN is kept as with
    // masked_fill(scores < thr, -inf)); -inf scores have zero weight
    float z = 0.0f;
    for (int64_t j = lane; j < Tkv; j += 32) {
      const float v = sval(j);
      if (!(v < thr) && v != NEG_INF) z += expf(v - rowmax);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) z += __shfl_xor_sync(0xffffffffu, z, o);
    const float invz = 1.0f / z;
    for (int64_t jb = 0; jb < Tkv; jb += 32) {
      const int64_t jl = jb + lane;
      const float v = jl < Tkv ? sval(jl) : NEG_INF;
      const bool kept = jl < Tkv && !(v < thr) && v != NEG_INF;
      const unsigned mask = __ballot_sync(0xffffffffu, kept);
      const float wl = kept ? expf(v - rowmax) * invz : 0.0f;
      gather(mask, wl, jb);
    }
    }
    float* orow = p.out + (slice * p.T + i) * dh;
#pragma unroll
    for (int q = 0; q < ATT_MAX_DH / 32; ++q) {
      const int c = lane + 32 * q;
      if (c < dh) orow[c] = oacc[q];
    }
  }
}

template <int R, int PL>
int launch_att(const AttArgs& a, cudaStream_t stream) {
  const int tkv_pad = (int)((a.Tkv + 3) & ~(int64_t)3);
  const size_t smem = ((size_t)a.dh * R + 2 * (size_t)a.dh * ATT_KT + (size_t)R * tkv_pad) * 4;
  cudaError_t e = cudaFuncSetAttribute(att_fwd_kernel<R, PL>,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return (int)e;
  dim3 grid((unsigned)ceil_div(a.T, (int64_t)R), (unsigned)a.H, (unsigned)a.B);
  att_fwd_kernel<R, PL><<<grid, ATT_THREADS, smem, stream>>>(a);
  return launch_status();
}

template <int R>
int launch_att_pl(const AttArgs& a, cudaStream_t stream) {
  if (a.Tkv <= 32 * 16) return launch_att<R, 16>(a, stream);
  if (a.Tkv <= 32 * 32) return launch_att<R, 32>(a, stream);
  if (a.Tkv <= 32 * 48) return launch_att<R, 48>(a, stream);
  return launch_att<R, 0>(a, stream);
}

constexpr size_t ATT_SMEM_LIMIT = 227 * 1024;

size_t att_smem_bytes(int R, int64_t Tkv, int dh) {
  const int64_t tkv_pad = (Tkv + 3) & ~(int64_t)3;
  return ((size_t)dh * R + 2 * (size_t)dh * ATT_KT + (size_t)R * tkv_pad) * 4;
}

}  // namespace

static inline int64_t round4(int64_t n) { return (n + 3) & ~(int64_t)3; }

// workspace: query features, query maxima, key features, key maxima; each
// region starts on a 16-byte boundary
// (the larger of this kernel's and the tensor-core kernel's, so that one
// workspace serves whichever path runs)
int64_t tsrn_attention_workspace_floats(int64_t B, int64_t H, int64_t T, int64_t Tkv, int64_t dh) {
  const int64_t cc =
      round4(B * H * T * dh) + round4(B * H * T) + round4(B * H * Tkv * dh) + round4(B * H * Tkv);
  const int64_t tc = tsrn_attention_tc_workspace_floats(B, H, T, Tkv);
  return cc > tc ? cc : tc;
}

int launch_tsrn_attention_fwd(int64_t B, int64_t H, int64_t T, int64_t Tkv, int64_t Tc, int64_t dh,
                              const float* Q, const float* K, const float* V,
                              const float* slopes, int top_k, int causal, float* out,
                              float* ws, cudaStream_t stream) {
  if (B * H * T == 0) return TP_OK;
  const int path = tsrn_attention_path();
  const bool tc_ok = tsrn_attention_tc_supported(dh, top_k);
  if (path == TP_ATT_PATH_TENSOR_CORES && !tc_ok) return TP_ERR_UNSUPPORTED;
  // auto: the tensor-core kernel where it applies and its 128-query tiles
  // are filled (T >= 128; at B = 64, T = 1024, dh = 80 it measured 3.27 ms
  // against 5.16 ms on CUDA cores), else the CUDA-core kernel (16-row tiles),
  // and the tensor-core kernel again beyond the CUDA-core key limit
  const bool cc_ok = dh >= 1 && dh <= ATT_MAX_DH && top_k >= 1 && top_k <= ATT_MAX_TOPK &&
                     Tkv >= 1 && Tkv <= ATT_MAX_TKV;
  const bool auto_tc = T >= 128 || !cc_ok;
  if (tc_ok && (path == TP_ATT_PATH_TENSOR_CORES || (path == TP_ATT_PATH_AUTO && auto_tc))) {
    if (Tc < 0 || Tc > Tkv || Tkv < 1) return TP_ERR_INVALID_ARG;
    return launch_tsrn_attention_tc(B, H, T, Tkv, Tc, dh, Q, K, V, slopes, top_k, causal, out, ws,
                                    stream);
  }
  if (dh < 1 || dh > ATT_MAX_DH || top_k < 1 || top_k > ATT_MAX_TOPK) return TP_ERR_UNSUPPORTED;
  if (Tkv < 1 || Tkv > ATT_MAX_TKV) return TP_ERR_UNSUPPORTED;
  if (Tc < 0 || Tc > Tkv) return TP_ERR_INVALID_ARG;
  if (B * H > 65535 || H > 65535) return TP_ERR_TOO_LARGE;
  // 16 query rows per CTA: at Tkv = 1024, dh = 80 two CTAs fit an SM (measured
  // 7.2 ms vs 10.0 ms with 32 rows and one CTA per SM, 8.1 ms with 8 rows)
  int R = 16;
  while (R > 8 && att_smem_bytes(R, Tkv, (int)dh) > ATT_SMEM_LIMIT) R /= 2;
  if (att_smem_bytes(R, Tkv, (int)dh) > ATT_SMEM_LIMIT) return TP_ERR_TOO_LARGE;
  float* AT = ws;
  float* qmx = AT + round4(B * H * T * dh);
  float* BT = qmx + round4(B * H * T);
  float* kmx = BT + round4(B * H * Tkv * dh);
  att_expfeat_kernel<<<dim3((unsigned)ceil_div(T, (int64_t)32), (unsigned)(B * H)), ATT_THREADS, 0,
                       stream>>>(Q, T, (int)dh, AT, qmx);
  att_expfeat_kernel<<<dim3((unsigned)ceil_div(Tkv, (int64_t)32), (unsigned)(B * H)), ATT_THREADS,
                       0, stream>>>(K, Tkv, (int)dh, BT, kmx);
  int s = launch_status();
  if (s != TP_OK) return s;
  AttArgs a{B, H, T, Tkv, Tc, (int)dh, top_k, causal, Q, K, V, slopes, AT, qmx, BT, kmx, out};
  if (R == 16) return launch_att_pl<16>(a, stream);
  return launch_att_pl<8>(a, stream);
}

}  // namespace tp
