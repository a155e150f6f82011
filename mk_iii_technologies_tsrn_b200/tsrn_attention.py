"""``TropicalAttention`` drop-in for TSRN (research/tsrn_dml.py:355-548).

Same constructor, sub-module and buffer names as the reference (``Wq``, ``Wk``,
``Wv``, ``Wo``, ``q_norm``, ``k_norm``, ``rope``, ``alibi_slopes``,
``cross_window_mem``), so a reference state dict loads unchanged.  The Q/K/V
projections, QK-norm and RoPE stay in PyTorch; in inference (eval mode or no
grad) the tropical score, ALiBi, causal mask, top-k threshold, softmax and
@V run as one fused kernel (``ops.tsrn_attention``).  With gradients enabled
in training the score runs on the LSE kernel (``ops.LSEScoreFunction``) and
the rest in PyTorch, so autograd sees the reference's expression.
"""
from __future__ import annotations

from typing import Optional, Tuple

import torch
import torch.nn as nn

from . import ops


class RotaryPositionEmbedding(nn.Module):
    """RoPE with base 500000 (research/tsrn_dml.py:284-319)."""

    def __init__(self, dim: int, max_seq_len: int = 4096, base: float = 500000.0):
        super().__init__()
        inv_freq = 1.0 / (base ** (torch.arange(0, dim, 2).float() / dim))
        self.register_buffer("inv_freq", inv_freq)
        self._build_cache(max_seq_len)

    def _build_cache(self, seq_len: int):
        t = torch.arange(seq_len, dtype=self.inv_freq.dtype, device=self.inv_freq.device)
        freqs = torch.einsum("i,j->ij", t, self.inv_freq)
        emb = torch.cat([freqs, freqs], dim=-1)
        self.register_buffer("cos_cached", emb.cos(), persistent=False)
        self.register_buffer("sin_cached", emb.sin(), persistent=False)

    @staticmethod
    def _rotate_half(x: torch.Tensor) -> torch.Tensor:
        x1, x2 = x[..., :x.shape[-1] // 2], x[..., x.shape[-1] // 2:]
        return torch.cat([-x2, x1], dim=-1)

    def forward(self, q: torch.Tensor, k: torch.Tensor, offset: int = 0):
        T = q.shape[2]
        if offset + T > self.cos_cached.shape[0]:
            self._build_cache(offset + T)
        cos = self.cos_cached[offset:offset + T].unsqueeze(0).unsqueeze(0)
        sin = self.sin_cached[offset:offset + T].unsqueeze(0).unsqueeze(0)
        return q * cos + self._rotate_half(q) * sin, k * cos + self._rotate_half(k) * sin


def build_alibi_slopes(n_heads: int) -> torch.Tensor:
    """Per-head ALiBi slopes 2^(-8 (h+1) / H) (research/tsrn_dml.py:329-334)."""
    ratio = 2.0 ** (-8.0 / n_heads)
    return torch.tensor([ratio ** (h + 1) for h in range(n_heads)])


class PersistentCrossWindowMemory(nn.Module):
    """Opt-in K/V cache of the previous window (research/tsrn_dml.py:994-1047)."""

    def __init__(self, d_model: int, n_heads: int, max_cached_len: int = 256):
        super().__init__()
        self.H = n_heads
        self.dh = d_model // n_heads
        self.max_cached_len = max_cached_len
        self.register_buffer("cached_k", torch.zeros(0))
        self.register_buffer("cached_v", torch.zeros(0))
        self._has_cache = False
        self.enabled = False

    def cache_kv(self, k: torch.Tensor, v: torch.Tensor):
        with torch.no_grad():
            T = k.shape[2]
            start = max(0, T - self.max_cached_len)
            self.cached_k = k[0, :, start:, :].detach().clone()
            self.cached_v = v[0, :, start:, :].detach().clone()
            self._has_cache = True

    def get_cached_kv(self, B: int) -> Tuple[Optional[torch.Tensor], Optional[torch.Tensor]]:
        if not self._has_cache or self.cached_k.numel() == 0:
            return None, None
        return (self.cached_k.unsqueeze(0).expand(B, -1, -1, -1),
                self.cached_v.unsqueeze(0).expand(B, -1, -1, -1))

    def reset(self):
        self.cached_k = torch.zeros(0, device=self.cached_k.device)
        self.cached_v = torch.zeros(0, device=self.cached_v.device)
        self._has_cache = False


class TropicalAttention(nn.Module):
    def __init__(self, d_model: int, top_k: int = 8, n_heads: int = 4,
                 dropout: float = 0.0, max_seq_len: int = 4096):
        super().__init__()
        assert d_model % n_heads == 0
        self.H = n_heads
        self.dh = d_model // n_heads
        self.top_k = top_k
        self.Wq = nn.Linear(d_model, d_model, bias=False)
        self.Wk = nn.Linear(d_model, d_model, bias=False)
        self.Wv = nn.Linear(d_model, d_model, bias=False)
        self.Wo = nn.Linear(d_model, d_model, bias=False)
        self.drop = nn.Dropout(dropout)
        nn.init.xavier_uniform_(self.Wq.weight, gain=0.5)
        nn.init.xavier_uniform_(self.Wk.weight, gain=0.5)
        nn.init.xavier_uniform_(self.Wv.weight, gain=0.5)
        self.q_norm = nn.LayerNorm(self.dh, elementwise_affine=True)
        self.k_norm = nn.LayerNorm(self.dh, elementwise_affine=True)
        self.rope = RotaryPositionEmbedding(self.dh, max_seq_len=max_seq_len)
        self.register_buffer("alibi_slopes", build_alibi_slopes(n_heads))
        self.cross_window_mem = PersistentCrossWindowMemory(d_model, n_heads, max_cached_len=256)

    def _unfused(self, Q, K, V, causal: bool, T_c: int, k: int):
        # the reference expression (research/tsrn_dml.py:505-526) on the LSE kernel
        T, T_kv = Q.shape[2], K.shape[2]
        scores = ops.LSEScoreFunction.apply(Q.contiguous(), K.contiguous(), 1.0)
        q_pos = torch.arange(T, device=scores.device)
        k_pos = torch.arange(-T_c, T_kv - T_c, device=scores.device)
        dist = (q_pos.unsqueeze(1) - k_pos.unsqueeze(0)).abs()
        alibi = -self.alibi_slopes.to(scores.device).view(-1, 1, 1) * dist.unsqueeze(0)
        scores = scores + alibi.unsqueeze(0)
        if causal:
            mask = k_pos.unsqueeze(0) > q_pos.unsqueeze(1)
            scores = scores.masked_fill(mask.unsqueeze(0).unsqueeze(0), float("-inf"))
        topk_v, _ = scores.topk(min(k, T_kv), dim=-1)
        thr = topk_v[:, :, :, -1:].detach()
        scores = scores.masked_fill(scores < thr, float("-inf"))
        w = self.drop(torch.softmax(scores, dim=-1))
        return w @ V

    def forward(self, x: torch.Tensor, causal: bool = True) -> torch.Tensor:
        B, T, d = x.shape
        H, dh = self.H, self.dh
        k = min(self.top_k, T)
        Q = self.Wq(x).view(B, T, H, dh).permute(0, 2, 1, 3)
        K = self.Wk(x).view(B, T, H, dh).permute(0, 2, 1, 3)
        V = self.Wv(x).view(B, T, H, dh).permute(0, 2, 1, 3)
        Q = self.q_norm(Q)
        K = self.k_norm(K)
        Q, K = self.rope(Q, K)
        K_orig, V_orig = K, V
        T_c = 0
        if not self.training and self.cross_window_mem.enabled:
            ck, cv = self.cross_window_mem.get_cached_kv(B)
            if ck is not None:
                K = torch.cat([ck, K], dim=2)
                V = torch.cat([cv, V], dim=2)
                T_c = ck.shape[2]
        if self.training and torch.is_grad_enabled():
            ctx = self._unfused(Q, K, V, causal, T_c, k)
        else:
            ctx = ops.tsrn_attention(Q, K, V, self.alibi_slopes, k, causal, T_c)
        ctx = ctx.permute(0, 2, 1, 3).contiguous().reshape(B, T, d)
        if not self.training and self.cross_window_mem.enabled:
            self.cross_window_mem.cache_kv(K_orig, V_orig)
        return self.Wo(ctx)
