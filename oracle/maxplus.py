"""Max-plus (tropical) GEMM oracle -- test infrastructure only (see package doc).

Reference expressions restated here:

* forward: ``scores = W.unsqueeze(0) + x.unsqueeze(1)`` then ``scores.max(-1)`` and
  ``+ bias`` -- tropformer.py:131 (broadcast add), :141 (max), :143-144 (bias).
  torch.max(dim=-1) returns the LOWEST index on ties and the first NaN;
  numpy's max/argmax follow the same rules, and each term is one float32 add.
* argmax backward: autograd of ``.max(-1).values`` (tropformer.py:141, and the
  hard branch of ``_tropical_max`` tropformer.py:93-94): the upstream gradient
  goes to the argmax term only, then sums over the broadcast dims.
* STE backward: autograd of tropformer.py:133-139 --
  ``soft = sum(softmax(s/tau) * s)``; d soft/ds = p * (1 + (s - sum(p*s))/tau).
* LSE backward: gradient of ``tau * logsumexp(s/tau)`` = softmax(s/tau)
  (tropformer.py:95-97 with _SMOOTH_MAX_TEMP; cuda/maxplus_gemm.cu:181-259).
* LSE forward: ``tau * logsumexp(s/tau)`` -- research/tsrn_dml.py:438-460 (tau = 1,
  the TSRN attention score) and research/tropical_optimizers.py:750-763.
"""
from __future__ import annotations

import numpy as np

_CHUNK_ELEMS = 1 << 24  # bound the [rows, N, K] broadcast temporary


def _rows_per_chunk(N: int, K: int) -> int:
    return max(1, _CHUNK_ELEMS // max(1, N * K))


def maxplus_fwd(x: np.ndarray, w: np.ndarray, bias: np.ndarray | None = None,
                scale: float = 1.0):
    """y[m,n] = max_k(w[n,k] + x[m,k]) (+bias[n]) (*scale), argmax (int64, lowest k).

    x [M,K], w [N,K] float32 (tropformer.py:131-144)."""
    x = np.asarray(x, dtype=np.float32)
    w = np.asarray(w, dtype=np.float32)
    M, K = x.shape
    N = w.shape[0]
    y = np.empty((M, N), dtype=np.float32)
    idx = np.zeros((M, N), dtype=np.int64)
    if K == 0:
        y.fill(-np.inf)
    else:
        step = _rows_per_chunk(N, K)
        with np.errstate(invalid="ignore"):          # inf + -inf = NaN, as in torch
            for m0 in range(0, M, step):
                s = w[None, :, :] + x[m0:m0 + step, None, :]   # one float32 add per term
                y[m0:m0 + step] = s.max(axis=-1)
                idx[m0:m0 + step] = s.argmax(axis=-1)
    if bias is not None:
        y = (y + np.asarray(bias, dtype=np.float32)[None, :]).astype(np.float32)
    if scale != 1.0:
        y = (y * np.float32(scale)).astype(np.float32)
    return y, idx


def maxplus_matmul(A: np.ndarray, B: np.ndarray):
    """C[i,j] = max_k(A[i,k] + B[k,j]) with B stored [K, N], and the lowest
    maximising k -- ``_tropical_matmul`` (benchmarks/synthetic_scheduling.py:35-38:
    ``(A[:, :, None] + B[None, :, :]).max(axis=1)``).  Each term is one float32
    add (commutative), so this is maxplus_fwd with w = B transposed."""
    return maxplus_fwd(np.asarray(A, np.float32), np.ascontiguousarray(np.asarray(B, np.float32).T))


def tropical_power_chain(A: np.ndarray, steps: int):
    """A^(steps+1) by repeated right-multiplication ``Ak = Ak (x) A`` -- the loop of
    ``_tropical_eigenvalue`` (benchmarks/synthetic_scheduling.py:41-55) -- and the
    eigenvalue estimate max_i Ak[i,i] / (steps + 1) that it returns."""
    Ak = np.asarray(A, np.float32).copy()
    for _ in range(steps):
        Ak, _ = maxplus_matmul(Ak, A)
    return Ak, float(np.diag(Ak).max() / (steps + 1))


def round_bf16(a: np.ndarray) -> np.ndarray:
    """Round float32 values to the nearest bfloat16 (ties to even), returned as
    float32; NaN stays NaN, overflow goes to +-inf."""
    a = np.asarray(a, dtype=np.float32)
    bits = a.view(np.uint32).astype(np.uint64)
    rounded = ((bits + 0x7FFF + ((bits >> 16) & 1)) & 0xFFFF0000).astype(np.uint32)
    out = rounded.view(np.float32)
    return np.where(np.isnan(a), np.float32(np.nan), out).astype(np.float32)


def maxplus_fwd_bf16(x: np.ndarray, w: np.ndarray, bias: np.ndarray | None = None,
                     scale: float = 1.0):
    """The reference expression on bf16 tensors (tropformer.py:131,141 with bf16
    weight and input): every sum w[n,k] + x[m,k] rounded to bf16, exact max,
    lowest-index argmax.  The max is returned as float32; bias and scale are
    then applied in float32 (the library's output convention)."""
    x = round_bf16(x)
    w = round_bf16(w)
    M, K = x.shape
    N = w.shape[0]
    y = np.empty((M, N), dtype=np.float32)
    idx = np.zeros((M, N), dtype=np.int64)
    if K == 0:
        y.fill(-np.inf)
    else:
        step = _rows_per_chunk(N, K)
        with np.errstate(invalid="ignore", over="ignore"):
            for m0 in range(0, M, step):
                s = round_bf16(w[None, :, :] + x[m0:m0 + step, None, :])
                y[m0:m0 + step] = s.max(axis=-1)
                idx[m0:m0 + step] = s.argmax(axis=-1)
    if bias is not None:
        y = (y + np.asarray(bias, dtype=np.float32)[None, :]).astype(np.float32)
    if scale != 1.0:
        y = (y * np.float32(scale)).astype(np.float32)
    return y, idx


def maxplus_bwd_argmax(idx: np.ndarray, gy: np.ndarray, K: int, scale: float = 1.0):
    """(gx [M,K], gw [N,K], gbias [N]) routing gy*scale to the argmax term (float64 sums)."""
    M, N = gy.shape
    g = gy.astype(np.float64) * scale
    gx = np.zeros((M, K), dtype=np.float64)
    gw = np.zeros((N, K), dtype=np.float64)
    if K > 0:
        mm = np.repeat(np.arange(M), N)
        nn = np.tile(np.arange(N), M)
        kk = idx.reshape(-1)
        np.add.at(gx, (mm, kk), g.reshape(-1))
        np.add.at(gw, (nn, kk), g.reshape(-1))
    return gx, gw, g.sum(axis=0)


def maxplus_bwd_smooth(mode: str, tau: float, x: np.ndarray, w: np.ndarray, gy: np.ndarray):
    """STE (tropformer.py:133-139) or LSE (tropformer.py:95-97) backward in float64."""
    x = np.asarray(x, dtype=np.float32)
    w = np.asarray(w, dtype=np.float32)
    M, K = x.shape
    N = w.shape[0]
    gx = np.zeros((M, K), dtype=np.float64)
    gw = np.zeros((N, K), dtype=np.float64)
    step = _rows_per_chunk(N, K)
    for m0 in range(0, M, step):
        s = (w[None, :, :] + x[m0:m0 + step, None, :]).astype(np.float64)
        z = s / tau
        z = z - z.max(axis=-1, keepdims=True)
        p = np.exp(z)
        p /= p.sum(axis=-1, keepdims=True)
        g = gy[m0:m0 + step, :, None].astype(np.float64)
        if mode == "ste":
            sbar = (p * s).sum(axis=-1, keepdims=True)
            dS = g * p * (1.0 + (s - sbar) / tau)
        elif mode == "lse":
            dS = g * p
        else:
            raise ValueError(mode)
        gx[m0:m0 + step] = dS.sum(axis=1)
        gw += dS.sum(axis=0)
    return gx, gw, gy.astype(np.float64).sum(axis=0)


def maxplus_lse_fwd(x: np.ndarray, w: np.ndarray, tau: float = 1.0):
    """tau * logsumexp_k((w[n,k] + x[m,k]) / tau) in float64 (terms rounded to float32 first)."""
    x = np.asarray(x, dtype=np.float32)
    w = np.asarray(w, dtype=np.float32)
    M, K = x.shape
    N = w.shape[0]
    y = np.empty((M, N), dtype=np.float64)
    step = _rows_per_chunk(N, K)
    for m0 in range(0, M, step):
        s = (w[None, :, :] + x[m0:m0 + step, None, :]).astype(np.float64) / tau
        mx = s.max(axis=-1, keepdims=True)
        y[m0:m0 + step] = tau * (mx[..., 0] + np.log(np.exp(s - mx).sum(axis=-1)))
    return y


def tsrn_attention_fwd(Q, K, V, slopes, top_k: int, causal: bool = True, Tc: int = 0):
    """TropicalAttention after RoPE (research/tsrn_dml.py:438-460 score, :505-526
    ALiBi, causal mask, top-k threshold, softmax, @V) in float64.

    Q [B,H,T,dh], K/V [B,H,Tkv,dh], slopes [H].  Returns (out [B,H,T,dh], the
    masked scores before the top-k step [B,H,T,Tkv])."""
    Q = np.asarray(Q, np.float64)
    K = np.asarray(K, np.float64)
    V = np.asarray(V, np.float64)
    slopes = np.asarray(slopes, np.float64)
    B, H, T, dh = Q.shape
    Tkv = K.shape[2]
    raw = Q[:, :, :, None, :] + K[:, :, None, :, :]
    m = raw.max(axis=-1, keepdims=True)
    S = (m + np.log(np.exp(raw - m).sum(axis=-1, keepdims=True)))[..., 0]
    q_pos = np.arange(T)
    k_pos = np.arange(-Tc, Tkv - Tc)
    dist = np.abs(q_pos[:, None] - k_pos[None, :])
    S = S - slopes[None, :, None, None] * dist[None, None]
    if causal:
        S = np.where((k_pos[None, :] > q_pos[:, None])[None, None], -np.inf, S)
    k = min(top_k, Tkv)
    thr = -np.sort(-S, axis=-1)[..., k - 1:k]
    Sm = np.where(S < thr, -np.inf, S)
    mx = Sm.max(axis=-1, keepdims=True)
    with np.errstate(invalid="ignore"):
        w = np.exp(Sm - mx)
        w = w / w.sum(axis=-1, keepdims=True)
    return w @ V, S


def lfdual_act(y, mode: str, slopes, biases, x_grid, blend_gate=None):
    """LFDualActivation (tropformer.py:224-289) in float32, each product and sum
    rounded separately as torch evaluates the reference expressions."""
    y = np.asarray(y, np.float32)
    s = np.asarray(slopes, np.float32)
    b = np.asarray(biases, np.float32)
    xg = np.asarray(x_grid, np.float32)
    with np.errstate(invalid="ignore", over="ignore"):
        primal = (y[..., None] * s + b).max(axis=-1)
        f_at_grid = (xg[:, None] * s + b).max(axis=-1)
        dual = (y[..., None] * xg - f_at_grid).max(axis=-1)
    if mode == "primal":
        return primal
    if mode == "dual":
        return dual
    g = (1.0 / (1.0 + np.exp(-np.asarray(blend_gate, np.float64)))).astype(np.float32)
    return (g * primal + (np.float32(1.0) - g) * dual).astype(np.float32)


def esn_gru_fwd(U, Uz, Ur, Wzh, Wrh, Ws, h0=None):
    """GRU-gated echo-state recurrence (research/tsrn_dml.py:834-840) in float64,
    h_{-1} = h0 (the reference: 0); returns H [B, T, dr]."""
    U, Uz, Ur = (np.asarray(a, np.float64) for a in (U, Uz, Ur))
    Wzh, Wrh, Ws = (np.asarray(a, np.float64) for a in (Wzh, Wrh, Ws))
    B, T, dr = U.shape
    h = np.zeros((B, dr)) if h0 is None else np.asarray(h0, np.float64).copy()
    H = np.empty((B, T, dr))
    sig = lambda v: 1.0 / (1.0 + np.exp(-v))
    for t in range(T):
        z = sig(h @ Wzh.T + Uz[:, t])
        r = sig(h @ Wrh.T + Ur[:, t])
        ht = np.tanh((r * h) @ Ws.T + U[:, t])
        h = (1 - z) * h + z * ht
        H[:, t] = h
    return H


def esn_leaky_fwd(U, Ws, lk, h0=None):
    """Leaky echo-state recurrence h = (1 - lk) h + lk tanh(h Ws^T + U_t)
    (tsrn_gpu.py:480-484) in float64, h_{-1} = h0 (the reference: 0); returns
    H [B, T, dr]."""
    U = np.asarray(U, np.float64)
    Ws = np.asarray(Ws, np.float64)
    lk = float(np.asarray(lk).reshape(()))
    B, T, dr = U.shape
    h = np.zeros((B, dr)) if h0 is None else np.asarray(h0, np.float64).copy()
    H = np.empty((B, T, dr))
    for t in range(T):
        h = (1 - lk) * h + lk * np.tanh(h @ Ws.T + U[:, t])
        H[:, t] = h
    return H
