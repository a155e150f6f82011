"""Tropical primitives with the reference's names and semantics, on the sm_100a kernels.

Mirrors ``tropformer.py`` (Mediocr3Mik3/MK_III_Technologies_TSRN):

* ``_SMOOTH_MAX_TEMP`` / ``_USE_SMOOTH_MAX`` -- module flags of tropformer.py:84-85.
  With ``_USE_SMOOTH_MAX`` the tropical score keeps the hard max value and
  takes the gradient of ``T*logsumexp(s/T)`` (tropformer.py:95-97).
* ``TropicalLinear`` -- tropformer.py:104-145: same constructor, the
  ``_ste_temp`` class attribute, parameters ``weight`` [out, in] (U(-0.5, 0.5))
  and ``bias`` [out] (zeros); train mode = hard forward + STE backward,
  eval mode = hard forward + argmax backward.
* ``tropical_score`` -- ``_tropical_max(Q.unsqueeze(3) + K.unsqueeze(2), -1) * scale``
  (deep_tropical_net.py:148-150, tropformer.py:378-381) without the
  [B, H, L, L, d] temporary.
* ``MaslovTemperature`` -- tropformer.py:175-217 (per-head softmax temperature).
* ``LFDualActivation`` -- tropformer.py:224-289 (tropical polynomial activation and
  its Legendre-Fenchel dual; primal / dual / blend).
* ``TropicalHybridFFN`` -- tropformer.py:407-456.  In inference the tropical
  up-projection and the activation run as one kernel (``ops.maxplus_lfdual``).
"""
from __future__ import annotations

import math

import torch
import torch.nn as nn

from . import ops
from .ops import MaxPlusLinearFunction, TropicalScoreFunction

_SMOOTH_MAX_TEMP = 50.0   # tropformer.py:84
_USE_SMOOTH_MAX = False   # tropformer.py:85


def _tropical_max(x: torch.Tensor, dim: int = -1) -> torch.Tensor:
    """Hard max value; with ``_USE_SMOOTH_MAX`` the gradient of T*logsumexp(x/T)
    (tropformer.py:87-97)."""
    if not _USE_SMOOTH_MAX:
        return x.max(dim=dim).values
    hard = x.max(dim=dim).values.detach()
    soft = _SMOOTH_MAX_TEMP * torch.logsumexp(x / _SMOOTH_MAX_TEMP, dim=dim)
    return hard + (soft - soft.detach())


def tropical_score(Q: torch.Tensor, K: torch.Tensor, scale: float = 1.0) -> torch.Tensor:
    """``max_f(Q[..., i, f] + K[..., j, f]) * scale`` with the reference's backward rules."""
    tau = _SMOOTH_MAX_TEMP if _USE_SMOOTH_MAX else None
    return TropicalScoreFunction.apply(Q, K, float(scale), tau)


class TropicalLinear(nn.Module):
    """Max-plus linear layer ``y_i = max_j(W_ij + x_j) + b_i`` (tropformer.py:104-145)."""

    _ste_temp = 1.0   # STE temperature (tropformer.py:117)

    def __init__(self, in_features: int, out_features: int, bias: bool = True):
        super().__init__()
        self.in_features = in_features
        self.out_features = out_features
        self.weight = nn.Parameter(torch.empty(out_features, in_features))
        self.bias = nn.Parameter(torch.zeros(out_features)) if bias else None
        nn.init.uniform_(self.weight, -0.5, 0.5)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        leading = x.shape[:-1]
        x_flat = x.reshape(-1, self.in_features)
        mode = "ste" if self.training else "argmax"
        out = MaxPlusLinearFunction.apply(x_flat, self.weight, self.bias, mode,
                                          float(type(self)._ste_temp))
        return out.reshape(*leading, self.out_features)

    def extra_repr(self):
        return f"in={self.in_features}, out={self.out_features}"


class MaslovTemperature(nn.Module):
    """Learnable per-head temperature: ``softmax(scores / tau_h)`` with
    ``tau = exp(log_temps).clamp(0.02, 10)`` (tropformer.py:175-217)."""

    def __init__(self, num_heads: int, init_temp: float = 1.0):
        super().__init__()
        self.log_temps = nn.Parameter(torch.full((num_heads,), math.log(init_temp)))

    @property
    def temperatures(self) -> torch.Tensor:
        return self.log_temps.exp().clamp(min=0.02, max=10.0)

    def forward(self, scores: torch.Tensor) -> torch.Tensor:
        """``scores`` [B, H, Lq, Lk] -> softmax over keys at temperature tau_h
        (one fused kernel, forward and backward)."""
        return ops.maslov_softmax(scores, self.temperatures)

    def extra_repr(self) -> str:
        t = self.temperatures.detach()
        return f"num_heads={len(t)}, tau=[{t.min():.3f}..{t.max():.3f}]"


class LFDualActivation(nn.Module):
    """Elementwise tropical polynomial f(x) = max_k(s_k x + b_k) and its
    Legendre-Fenchel dual f*(y) = max_j(x_j y - f(x_j)); mode "primal", "dual" or
    "blend" (sigmoid(blend_gate) per channel) -- tropformer.py:224-289."""

    def __init__(self, dim: int, num_pieces: int = 8, mode: str = "primal"):
        super().__init__()
        self.mode = mode
        self.num_pieces = num_pieces
        self.slopes = nn.Parameter(torch.linspace(-1.5, 1.5, num_pieces))
        self.biases = nn.Parameter(torch.zeros(num_pieces))
        self.x_grid = nn.Parameter(torch.linspace(-3.0, 3.0, num_pieces))
        if mode == "blend":
            self.blend_gate = nn.Parameter(torch.zeros(dim))

    def f_primal(self, x: torch.Tensor) -> torch.Tensor:
        pieces = x.unsqueeze(-1) * self.slopes + self.biases
        return _tropical_max(pieces, dim=-1)

    def f_dual(self, y: torch.Tensor) -> torch.Tensor:
        f_at_grid = _tropical_max(self.x_grid.unsqueeze(-1) * self.slopes + self.biases, dim=-1)
        dual_pieces = y.unsqueeze(-1) * self.x_grid - f_at_grid
        return _tropical_max(dual_pieces, dim=-1)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if self.mode == "primal":
            return self.f_primal(x)
        if self.mode == "dual":
            return self.f_dual(x)
        g = torch.sigmoid(self.blend_gate)
        return g * self.f_primal(x) + (1.0 - g) * self.f_dual(x)


def tropical_up_lf(trop_up: TropicalLinear, lf_act: LFDualActivation,
                   x: torch.Tensor) -> torch.Tensor:
    """``lf_act(trop_up(x))``: one fused kernel when no gradient is taken (inference),
    the modules' own forward otherwise."""
    needs_graph = torch.is_grad_enabled() and (x.requires_grad or any(
        p.requires_grad for p in (*trop_up.parameters(), *lf_act.parameters())))
    if needs_graph or not x.is_cuda:
        return lf_act(trop_up(x))
    lead = x.shape[:-1]
    gate = torch.sigmoid(lf_act.blend_gate) if lf_act.mode == "blend" else None
    y = ops.maxplus_lfdual(x.reshape(-1, trop_up.in_features), trop_up.weight, trop_up.bias,
                           lf_act.mode, lf_act.slopes, lf_act.biases, lf_act.x_grid, gate)
    return y.reshape(*lead, trop_up.out_features)


class TropicalHybridFFN(nn.Module):
    """Tropical branch (TropicalLinear -> LFDualActivation -> dropout) and classical
    branch (Linear -> GELU) fused by sigmoid(gate_proj(x)); down_proj, dropout,
    LayerNorm with residual -- tropformer.py:407-456."""

    def __init__(self, d_model: int, ffn_dim: int, dropout: float = 0.1,
                 trop_dropout: float = 0.05, lf_pieces: int = 8, lf_mode: str = "blend"):
        super().__init__()
        self.trop_up = TropicalLinear(d_model, ffn_dim)
        self.lf_act = LFDualActivation(ffn_dim, num_pieces=lf_pieces, mode=lf_mode)
        self.trop_drop = nn.Dropout(trop_dropout)
        self.class_up = nn.Linear(d_model, ffn_dim)
        self.gelu = nn.GELU()
        self.gate_proj = nn.Linear(d_model, ffn_dim)
        nn.init.zeros_(self.gate_proj.weight)
        nn.init.constant_(self.gate_proj.bias, -2.0)
        self.down_proj = nn.Linear(ffn_dim, d_model)
        self.dropout = nn.Dropout(dropout)
        self.norm = nn.LayerNorm(d_model)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        trop = self.trop_drop(tropical_up_lf(self.trop_up, self.lf_act, x))
        classical = self.gelu(self.class_up(x))
        g = torch.sigmoid(self.gate_proj(x))
        fused = g * trop + (1.0 - g) * classical
        out = self.dropout(self.down_proj(fused))
        return self.norm(out + x)
