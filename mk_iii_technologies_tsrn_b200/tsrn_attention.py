"""``TropicalAttention`` drop-in for TSRN (research/tsrn_dml.py:355-548) on the B200 kernels.

The module keeps the reference's constructor and its parameter / buffer names
(``Wq``, ``Wk``, ``Wv``, ``Wo``, ``q_norm``, ``k_norm``, ``rope.inv_freq``,
``alibi_slopes``, ``cross_window_mem.cached_k`` / ``cached_v``), so a reference
state dict loads unchanged.  The computation is this library's:

* one GEMM projects Q, K and V together (the three weights stacked; in
  inference the projections run as fp32-accurate 3xTF32 tensor-core GEMMs,
  ``ops.linear``);
* one kernel (``tp_tsrn_attention_prologue``) applies the per-head QK
  LayerNorm and the rotary embedding and lays Q/K/V out head-major;
* one kernel (``tp_tsrn_attention_fwd``) computes the log-sum-exp tropical
  score, ALiBi, the causal mask, the top-k threshold, the softmax and @V
  without materialising the T x T scores;
* in training, :class:`PrologueFunction` runs the same prologue kernel with a
  fused backward, and :class:`TopKAttentionFunction` keeps the attention
  forward (saving each row's kept keys) and supplies a sparse analytic backward over the kept
  (query, key) pairs (``ops.tsrn_attention_sparse_bwd``); with attention
  dropout the forward runs densely so that the dropped weights are the ones
  differentiated, and the backward recomputes the dense scores.
"""
from __future__ import annotations

from typing import Dict, Optional, Tuple

import torch
import torch.nn as nn

from . import ops


def alibi_slopes(n_heads: int) -> torch.Tensor:
    """Slope of head h (0-based): 2^(-8 (h + 1) / H) (research/tsrn_dml.py:329-334)."""
    e = torch.arange(1, n_heads + 1, dtype=torch.float64) * (-8.0 / n_heads)
    return torch.pow(2.0, e).float()


class RotaryTable(nn.Module):
    """Rotary position embedding of research/tsrn_dml.py:284-319: base 500000,
    channel c paired with c + dh/2 and rotated by pos * inv_freq[c].

    Holds the reference's persistent buffer ``inv_freq``.  The cos / sin tables
    ([positions, dh/2]) are computed on the host, as the reference builds its
    cache at construction, and kept per device outside the state dict."""

    def __init__(self, dim: int, max_seq_len: int = 4096, base: float = 500000.0):
        super().__init__()
        self.register_buffer("inv_freq",
                             1.0 / (base ** (torch.arange(0, dim, 2).float() / dim)))
        self.max_seq_len = max_seq_len
        self._tables: Dict[tuple, Tuple[torch.Tensor, torch.Tensor]] = {}

    def tables(self, n: int, device) -> Tuple[torch.Tensor, torch.Tensor]:
        n = max(n, self.max_seq_len)
        inv = self.inv_freq.detach()
        key = (str(device), n, inv.data_ptr(), inv._version)
        hit = self._tables.get(key)
        if hit is None:
            angle = torch.outer(torch.arange(n, dtype=torch.float32), inv.float().cpu())
            hit = (angle.cos().to(device), angle.sin().to(device))
            self._tables = {key: hit}
        return hit

    @staticmethod
    def rotate(t: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor) -> torch.Tensor:
        """Differentiable rotation of t [..., T, dh] by tables [T, dh/2]."""
        lo, hi = t.chunk(2, dim=-1)
        return torch.cat((lo * cos - hi * sin, hi * cos + lo * sin), dim=-1)


class CrossWindowCache(nn.Module):
    """Opt-in K/V of the previous window for autoregressive generation in eval
    mode (research/tsrn_dml.py:994-1047): after a call the last
    ``max_cached_len`` positions of sequence 0's rotated K and V are kept and
    prepended, broadcast over the batch, to the next call's keys."""

    def __init__(self, d_model: int, n_heads: int, max_cached_len: int = 256):
        super().__init__()
        self.max_cached_len = max_cached_len
        self.register_buffer("cached_k", torch.zeros(0))
        self.register_buffer("cached_v", torch.zeros(0))
        self.enabled = False
        self._filled = False          # set by store(), not by loading a state dict

    def has(self) -> bool:
        return self._filled and self.cached_k.numel() > 0

    def store(self, K: torch.Tensor, V: torch.Tensor) -> None:
        keep = slice(max(0, K.shape[2] - self.max_cached_len), None)
        self.cached_k = K[0, :, keep].detach().clone()
        self.cached_v = V[0, :, keep].detach().clone()
        self._filled = True

    def prepend(self, K: torch.Tensor, V: torch.Tensor):
        B = K.shape[0]
        ck = self.cached_k.unsqueeze(0).expand(B, -1, -1, -1)
        cv = self.cached_v.unsqueeze(0).expand(B, -1, -1, -1)
        return torch.cat((ck, K), dim=2), torch.cat((cv, V), dim=2), ck.shape[2]

    def reset(self) -> None:
        self.cached_k = torch.zeros(0, device=self.cached_k.device)
        self.cached_v = torch.zeros(0, device=self.cached_v.device)
        self._filled = False


def _masked_scores(Q, K, slopes, top_k: int, causal: bool, Tc: int) -> torch.Tensor:
    """Dense scores with ALiBi, the causal mask and the top-k cut (-inf outside),
    the score itself from the LSE kernel."""
    T, Tkv = Q.shape[2], K.shape[2]
    S = ops.lse_scores(Q, K)
    qp = torch.arange(T, device=S.device)
    kp = torch.arange(-Tc, Tkv - Tc, device=S.device)
    S = S - slopes.view(-1, 1, 1) * (qp[:, None] - kp[None, :]).abs()
    if causal:
        S = S.masked_fill(kp[None, :] > qp[:, None], float("-inf"))
    cut = S.topk(min(top_k, Tkv), dim=-1).values[..., -1:]
    return S.masked_fill(S < cut, float("-inf"))


class PrologueFunction(torch.autograd.Function):
    """The attention prologue (per-head QK LayerNorm, rotary embedding, head
    layout) with autograd: the fused forward kernel and its fused backward
    (``ops.tsrn_attention_prologue_bwd``): qkv [B*T, 3*H*dh] and the four
    LayerNorm parameters get gradients."""

    @staticmethod
    def forward(ctx, qkv, qg, qb, kg, kb, cos, sin, B: int, T: int, H: int, dh: int, eps: float):
        ctx.dims = (B, T, H, dh, eps)
        ctx.save_for_backward(qkv, qg, kg, cos, sin)
        return ops.tsrn_attention_prologue_raw(qkv, B, T, H, dh, qg, qb, kg, kb, eps, cos, sin)

    @staticmethod
    def backward(ctx, dQ, dK, dV):
        qkv, qg, kg, cos, sin = ctx.saved_tensors
        B, T, H, dh, eps = ctx.dims
        zero = None
        if dQ is None or dK is None or dV is None:
            zero = torch.zeros(B, H, T, dh, device=qkv.device)
        dqkv, dqg, dqb, dkg, dkb = ops.tsrn_attention_prologue_bwd(
            qkv, B, T, H, dh, qg, kg, eps, cos, sin, zero if dQ is None else dQ,
            zero if dK is None else dK, zero if dV is None else dV)
        return dqkv, dqg, dqb, dkg, dkb, None, None, None, None, None, None, None


class TopKAttentionFunction(torch.autograd.Function):
    """Tropical top-k attention core: Q, K, V [B, H, T(kv), dh] (rotated) ->
    context [B, H, T, dh].  The top-k cut is not differentiated (the reference
    detaches its threshold).  ``drop_p`` > 0 draws an attention-dropout mask
    (scaled by 1 / (1 - p)) over the kept weights.

    Without dropout, on shapes the tensor-core kernel takes (dh <= 96,
    top_k <= 16), the forward saves each row's kept keys and weights and the
    backward is sparse: two kernels over the ~top_k kept (i, j) of each row
    (``ops.tsrn_attention_sparse_bwd``).  Otherwise -- dropout, other shapes,
    or ties that kept more keys than the lists hold -- the backward recomputes
    the dense scores."""

    @staticmethod
    def forward(ctx, Q, K, V, slopes, top_k: int, causal: bool, Tc: int, drop_p: float):
        ctx.args = (top_k, causal, Tc, drop_p)
        if drop_p > 0.0:
            P = torch.softmax(_masked_scores(Q, K, slopes, top_k, causal, Tc), dim=-1)
            keep = (torch.rand_like(P) >= drop_p).to(P.dtype) / (1.0 - drop_p)
            ctx.save_for_backward(Q, K, V, slopes, keep, None, None, None, None)
            return (P * keep) @ V
        if ops.tsrn_attention_supports_lists(Q.shape[-1], top_k, K.shape[-2]):
            out, kj, kp, kl, kn = ops.tsrn_attention_train_fwd(Q, K, V, slopes, top_k, causal, Tc)
            ctx.save_for_backward(Q, K, V, slopes, None, kj, kp, kl, kn)
            return out
        ctx.save_for_backward(Q, K, V, slopes, None, None, None, None, None)
        return ops.tsrn_attention(Q, K, V, slopes, top_k, causal, Tc)

    @staticmethod
    def backward(ctx, dO):
        Q, K, V, slopes, keep, kj, kp, kl, kn = ctx.saved_tensors
        top_k, causal, Tc, _ = ctx.args
        if kj is not None and (kn.numel() == 0 or int(kn.min()) >= 0):
            dQ, dK, dV = ops.tsrn_attention_sparse_bwd(Q, K, V, dO, kj, kp, kl, kn)
            return dQ, dK, dV, None, None, None, None, None
        P = torch.softmax(_masked_scores(Q, K, slopes, top_k, causal, Tc), dim=-1)
        Pd = P * keep if keep is not None else P
        dV = Pd.transpose(-1, -2) @ dO
        dP = dO @ V.transpose(-1, -2)
        if keep is not None:
            dP = dP * keep
        # softmax backward: dS = P (dP - sum_j P dP); -inf entries have P = 0
        dS = P * (dP - (P * dP).sum(dim=-1, keepdim=True))
        lead = Q.shape[:-2]
        gQ, gK, _ = ops.maxplus_backward_smooth(
            "lse", 1.0, Q.reshape(-1, *Q.shape[-2:]), K.reshape(-1, *K.shape[-2:]),
            dS.reshape(-1, *dS.shape[-2:]))
        return (gQ.reshape(*lead, *Q.shape[-2:]), gK.reshape(*lead, *K.shape[-2:]), dV,
                None, None, None, None, None)


class TropicalAttention(nn.Module):
    def __init__(self, d_model: int, top_k: int = 8, n_heads: int = 4,
                 dropout: float = 0.0, max_seq_len: int = 4096):
        super().__init__()
        if d_model % n_heads:
            raise ValueError(f"d_model {d_model} is not a multiple of n_heads {n_heads}")
        self.H = n_heads
        self.dh = d_model // n_heads
        self.top_k = top_k
        self.Wq = nn.Linear(d_model, d_model, bias=False)
        self.Wk = nn.Linear(d_model, d_model, bias=False)
        self.Wv = nn.Linear(d_model, d_model, bias=False)
        self.Wo = nn.Linear(d_model, d_model, bias=False)
        for w in (self.Wq, self.Wk, self.Wv):
            nn.init.xavier_uniform_(w.weight, gain=0.5)
        self.drop = nn.Dropout(dropout)
        self.q_norm = nn.LayerNorm(self.dh)
        self.k_norm = nn.LayerNorm(self.dh)
        self.rope = RotaryTable(self.dh, max_seq_len=max_seq_len)
        self.register_buffer("alibi_slopes", alibi_slopes(n_heads))
        self.cross_window_mem = CrossWindowCache(d_model, n_heads, max_cached_len=256)

    def _qkv_weight(self) -> torch.Tensor:
        return torch.cat((self.Wq.weight, self.Wk.weight, self.Wv.weight), dim=0)

    def project(self, x: torch.Tensor):
        """Rotated, normalised Q, K and V [B, H, T, dh] of x [B, T, d] (inference:
        one stacked GEMM and the fused prologue kernel)."""
        B, T, d = x.shape
        qkv = ops.linear(x, self._qkv_weight()).reshape(B * T, 3 * d)
        cos, sin = self.rope.tables(T, x.device)
        return ops.tsrn_attention_prologue(qkv, B, T, self.H, self.dh, self.q_norm, self.k_norm,
                                           cos, sin)

    def _project_train(self, x: torch.Tensor):
        """Q, K, V with autograd: the stacked projection (3xTF32 GEMMs) and the
        fused prologue kernel with its fused backward; the PyTorch chain
        (``_project_differentiable``) where the kernel does not apply."""
        qn, kn = self.q_norm, self.k_norm
        if qn.weight is None or kn.weight is None or qn.eps != kn.eps or self.dh % 2 or \
                self.dh > 128 or not x.is_cuda:
            return self._project_differentiable(x)
        B, T, d = x.shape
        qkv = ops.linear(x, self._qkv_weight()).reshape(B * T, 3 * d)
        cos, sin = self.rope.tables(T, x.device)
        return PrologueFunction.apply(qkv, qn.weight, qn.bias, kn.weight, kn.bias, cos, sin,
                                      B, T, self.H, self.dh, float(qn.eps))

    def _project_differentiable(self, x: torch.Tensor):
        B, T, d = x.shape
        q, k, v = ops.linear(x, self._qkv_weight()).view(B, T, 3, self.H, self.dh).unbind(2)
        cos, sin = self.rope.tables(T, x.device)
        cos, sin = cos[:T], sin[:T]
        heads = lambda t: t.permute(0, 2, 1, 3)   # noqa: E731
        Q = RotaryTable.rotate(self.q_norm(heads(q)), cos, sin)
        K = RotaryTable.rotate(self.k_norm(heads(k)), cos, sin)
        return Q, K, heads(v)

    def forward(self, x: torch.Tensor, causal: bool = True) -> torch.Tensor:
        B, T, d = x.shape
        k = min(self.top_k, T)
        grad = torch.is_grad_enabled() and (x.requires_grad or any(
            p.requires_grad for p in self.parameters()))
        Q, K, V = self._project_train(x) if grad else self.project(x)
        use_cache = not self.training and self.cross_window_mem.enabled
        Kn, Vn, Tc = K, V, 0
        if use_cache and self.cross_window_mem.has():
            K, V, Tc = self.cross_window_mem.prepend(K, V)
        slopes = self.alibi_slopes.to(device=x.device, dtype=torch.float32)
        if grad:
            p = self.drop.p if self.training else 0.0
            ctx = TopKAttentionFunction.apply(Q, K, V, slopes, k, causal, Tc, p)
        else:
            ctx = ops.tsrn_attention(Q, K.contiguous(), V.contiguous(), slopes, k, causal, Tc)
        if use_cache:
            self.cross_window_mem.store(Kn, Vn)
        return ops.linear(ctx.transpose(1, 2).reshape(B, T, d), self.Wo.weight)
