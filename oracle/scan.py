"""Max-plus SSM scan oracle -- test infrastructure only (see package doc).

The recurrence of record is ``h_t = max(A + h_{t-1}, u_t)`` (module comment
research/tsrn_dml.py:906-916; docstring :918-927), evaluated step by step in
float32: one rounded add, one exact max.  The input wins ties, the rule
``torch.cummax`` applies in the reference's closed form (last index on ties,
research/tsrn_dml.py:968), which routes the reference gradient.

``scan_closed_form`` restates the reference's own vectorised evaluation
(research/tsrn_dml.py:961-972) for comparison; its rounding differs from the
recurrence by O(T * ulp).
"""
from __future__ import annotations

import numpy as np


def scan_fwd(u: np.ndarray, a: np.ndarray, h_init: float = -np.inf,
             h0: np.ndarray | None = None):
    """Sequential recurrence over u [B,T,C] float32 -> (h [B,T,C], win [B,T,C] bool)."""
    u = np.asarray(u, dtype=np.float32)
    a = np.asarray(a, dtype=np.float32)
    B, T, C = u.shape
    h = np.empty_like(u)
    win = np.empty(u.shape, dtype=bool)
    cur = (np.full((B, C), h_init, dtype=np.float32) if h0 is None
           else np.asarray(h0, dtype=np.float32).copy())
    for t in range(T):
        d = (a[None, :] + cur).astype(np.float32)
        wt = u[:, t, :] >= d
        cur = np.where(wt, u[:, t, :], d).astype(np.float32)
        h[:, t, :] = cur
        win[:, t, :] = wt
    return h, win


def scan_bwd(gh: np.ndarray, win: np.ndarray, dtype=np.float64):
    """Argmax-path backward: returns (gu [B,T,C], ga [C], gh0 [B,C]).

    G_t = gh_t + (input lost at t+1 ? G_{t+1} : 0); gu_t = win_t ? G_t : 0;
    ga = sum over b, t of (!win_t ? G_t : 0); gh0 = !win_0 ? G_0 : 0.
    With dtype=float32 the sums run in the same order as the CUDA kernel
    (reverse time per lane, then ascending batch), so results are bit-exact."""
    gh = np.asarray(gh, dtype=dtype)
    B, T, C = gh.shape
    zero = dtype(0.0)
    gu = np.zeros_like(gh)
    ga = np.zeros((B, C), dtype=dtype)
    carry = np.zeros((B, C), dtype=dtype)
    for t in range(T - 1, -1, -1):
        G = (gh[:, t, :] + carry).astype(dtype)
        w = win[:, t, :]
        gu[:, t, :] = np.where(w, G, zero)
        lost = np.where(w, zero, G).astype(dtype)
        ga = (ga + lost).astype(dtype)
        carry = lost
    total = np.zeros(C, dtype=dtype)
    for b in range(B):
        total = (total + ga[b]).astype(dtype)
    return gu, total, carry


def win_mask_words(win: np.ndarray) -> np.ndarray:
    """Pack win [B,T,C] into [B, ceil(T/32), C] uint32 words (bit t%32 of word t//32)."""
    B, T, C = win.shape
    nw = (T + 31) // 32
    out = np.zeros((B, nw, C), dtype=np.uint64)
    for t in range(T):
        out[:, t // 32, :] |= win[:, t, :].astype(np.uint64) << np.uint64(t % 32)
    return out.astype(np.uint32)


def scan_closed_form(u: np.ndarray, A: np.ndarray):
    """research/tsrn_dml.py:961-972: H = t*A_c + cummax([A_c, u_t - t*A_c])[1:], A_c = min(A,0).

    Effective h_{-1} = 0 (the leading A_c row)."""
    u = np.asarray(u, dtype=np.float32)
    A_c = np.minimum(np.asarray(A, dtype=np.float32), np.float32(0.0))
    B, T, C = u.shape
    t_idx = np.arange(T, dtype=np.float32)[:, None]
    shifted = (u - t_idx * A_c).astype(np.float32)
    G = np.concatenate([np.broadcast_to(A_c, (B, 1, C)), shifted], axis=1)
    cm = np.maximum.accumulate(G, axis=1)[:, 1:, :]
    return (t_idx[None] * A_c + cm).astype(np.float32)
