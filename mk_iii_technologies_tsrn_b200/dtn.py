"""``DTNAttention`` drop-in (deep_tropical_net.py:90-165) on the sm_100a kernels.

Same constructor, sub-module names and state-dict keys as the reference
(``q_proj``, ``k_proj`` tropical; ``v_proj``, ``out_proj``, ``score_gate``
classical; ``maslov``; ``attn_dropout``), so a reference checkpoint loads
unchanged.  The tropical Q/K projections run the max-plus GEMM kernels and
the tropical score runs the batched max-plus kernel on strided head views;
the gate blend, mask and Maslov softmax run as one kernel (forward and
backward); the classical linears and products stay in PyTorch.
"""
from __future__ import annotations

import torch
import torch.nn as nn

from . import ops, tropical
from .tropical import LFDualActivation, MaslovTemperature, TropicalLinear, tropical_up_lf


class DTNAttention(nn.Module):
    def __init__(self, d_model: int, num_heads: int, dropout: float = 0.1,
                 init_temp: float = 1.0):
        super().__init__()
        assert d_model % num_heads == 0
        self.d_model = d_model
        self.num_heads = num_heads
        self.d_k = d_model // num_heads
        self._scale = self.d_k ** -0.5
        self.q_proj = TropicalLinear(d_model, d_model)
        self.k_proj = TropicalLinear(d_model, d_model)
        self.v_proj = nn.Linear(d_model, d_model)
        self.out_proj = nn.Linear(d_model, d_model)
        self.score_gate = nn.Linear(d_model, num_heads)
        nn.init.zeros_(self.score_gate.weight)
        nn.init.constant_(self.score_gate.bias, +2.0)
        self.maslov = MaslovTemperature(num_heads, init_temp)
        self.attn_dropout = nn.Dropout(dropout)

    def _split_heads(self, x: torch.Tensor) -> torch.Tensor:
        B, L, D = x.shape
        return x.view(B, L, self.num_heads, self.d_k).transpose(1, 2)

    def forward(self, x: torch.Tensor, mask=None):
        B, L, D = x.shape
        Q = self._split_heads(self.q_proj(x))
        K = self._split_heads(self.k_proj(x))
        V = self._split_heads(self.v_proj(x))
        class_scores = torch.matmul(Q, K.transpose(-2, -1)) * self._scale
        trop_scores = tropical.tropical_score(Q, K, self._scale)
        g = torch.sigmoid(self.score_gate(x))                     # [B, L, H]
        # gate blend, mask and Maslov softmax in one kernel (:152-160)
        attn = ops.maslov_softmax(trop_scores, self.maslov.temperatures,
                                  classical=class_scores, gate=g, mask=mask)
        attn = self.attn_dropout(attn)
        out = torch.matmul(attn, V).transpose(1, 2).contiguous().view(B, L, D)
        return self.out_proj(out), attn


class DTNHybridFFN(nn.Module):
    """Tropical-biased hybrid FFN (deep_tropical_net.py:172-211): tropical branch
    TropicalLinear -> LFDualActivation -> dropout, classical Linear -> GELU,
    g * trop + (1 - g) * classical with g = sigmoid(gate_proj(x)) (bias +2)."""

    def __init__(self, d_model: int, ffn_dim: int, dropout: float = 0.1, lf_pieces: int = 8,
                 lf_mode: str = "blend"):
        super().__init__()
        self.trop_up = TropicalLinear(d_model, ffn_dim)
        self.lf_act = LFDualActivation(ffn_dim, num_pieces=lf_pieces, mode=lf_mode)
        self.trop_drop = nn.Dropout(dropout)
        self.class_up = nn.Linear(d_model, ffn_dim)
        self.gelu = nn.GELU()
        self.gate_proj = nn.Linear(d_model, ffn_dim)
        nn.init.zeros_(self.gate_proj.weight)
        nn.init.constant_(self.gate_proj.bias, +2.0)
        self.down_proj = nn.Linear(ffn_dim, d_model)
        self.dropout = nn.Dropout(dropout)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        trop = self.trop_drop(tropical_up_lf(self.trop_up, self.lf_act, x))
        classical = self.gelu(self.class_up(x))
        g = torch.sigmoid(self.gate_proj(x))
        fused = g * trop + (1.0 - g) * classical
        return self.dropout(self.down_proj(fused))
