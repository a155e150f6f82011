"""Drop-in for the reference's ``cuda/maxplus_binding.py`` (same public names).

``CUDATropicalLinear``, ``MaxPlusForwardBackward`` and ``is_cuda_kernel_available``
keep the reference's constructor arguments, parameter names, initialisation
and call signatures (cuda/maxplus_binding.py:37-153), but:

* the kernels are the sm_100a ones of ``_tropical_b200.so``, called with the
  arguments in the right slots (the reference passed x in W's slot,
  cuda/maxplus_binding.py:58-67 vs cuda/maxplus_gemm.cu:299-301);
* training uses the STE gradient of ``tropformer.TropicalLinear``
  (tropformer.py:133-139) and eval the argmax gradient (tropformer.py:141), which
  is what the reference's CPU fallback computes and what callers of
  TropicalLinear get -- the reference ``.cu`` backward computed softmax(s/tau)
  instead, available here as mode ``"lse"``;
* there is no silent CPU fallback: a CPU input raises.
"""
from __future__ import annotations

import torch
import torch.nn as nn
from torch.autograd import Function

from . import _lib
from .ops import MaxPlusLinearFunction


def is_cuda_kernel_available() -> bool:
    """True when the CUDA library loads and a CUDA device is present
    (cuda/maxplus_binding.py:37-39)."""
    return _lib.is_available() and torch.cuda.is_available()


class MaxPlusForwardBackward(Function):
    """``apply(x, weight, bias, ste_temp[, mode])`` -> y = max_j(W_ij + x_j) + b_i.

    Same positional arguments as the reference (cuda/maxplus_binding.py:42-97);
    backward returns (grad_x, grad_W, grad_bias, None, None).  ``mode`` defaults
    to ``"ste"``; ``"argmax"`` and ``"lse"`` select the other backward semantics."""

    @staticmethod
    def forward(ctx, x, weight, bias, ste_temp, mode: str = "ste"):
        return MaxPlusLinearFunction.forward(ctx, x, weight, bias, mode, ste_temp)

    @staticmethod
    def backward(ctx, grad_y):
        gx, gw, gb, _, _ = MaxPlusLinearFunction.backward(ctx, grad_y)
        return gx, gw, gb, None, None


class CUDATropicalLinear(nn.Module):
    """Max-plus linear layer ``y_i = max_j(W_ij + x_j) + b_i`` on the sm_100a kernels.

    Drop-in replacement for ``tropformer.TropicalLinear`` and the reference's
    ``CUDATropicalLinear`` (cuda/maxplus_binding.py:100-153): weight [out, in]
    initialised U(-0.5, 0.5), bias zeros (or None), any leading dims."""

    def __init__(self, in_features: int, out_features: int, bias: bool = True,
                 ste_temp: float = 1.0):
        super().__init__()
        self.in_features = in_features
        self.out_features = out_features
        self.ste_temp = ste_temp
        self.weight = nn.Parameter(torch.empty(out_features, in_features))
        self.bias = nn.Parameter(torch.zeros(out_features)) if bias else None
        nn.init.uniform_(self.weight, -0.5, 0.5)
        self._use_cuda = True

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        leading = x.shape[:-1]
        x_flat = x.reshape(-1, self.in_features)
        mode = "ste" if self.training else "argmax"
        out = MaxPlusLinearFunction.apply(x_flat, self.weight, self.bias, mode, self.ste_temp)
        return out.reshape(*leading, self.out_features)

    def extra_repr(self):
        return f"in={self.in_features}, out={self.out_features}, cuda=True"
