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
"""
from __future__ import annotations

import math

import torch
import torch.nn as nn
import torch.nn.functional as F

from .ops import MaxPlusLinearFunction, TropicalScoreFunction

_SMOOTH_MAX_TEMP = 50.0   # tropformer.py:84
_USE_SMOOTH_MAX = False   # tropformer.py:85


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
        tau = self.temperatures.view(1, -1, 1, 1)
        return F.softmax(scores / tau, dim=-1)

    def extra_repr(self) -> str:
        t = self.temperatures.detach()
        return f"num_heads={len(t)}, tau=[{t.min():.3f}..{t.max():.3f}]"
