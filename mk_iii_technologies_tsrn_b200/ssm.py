"""``TropicalSSM`` drop-in (research/tsrn_dml.py:917-980) on the sm_100a scan.

Same constructor, parameters and initialisation (``A``, ``B_proj``, ``C_proj``,
``gate_B``, ``gate_out``, ``mix``), so reference checkpoints load unchanged.
The scan (research/tsrn_dml.py:961-972) changes: the reference evaluates
``h_t = max(A_c + h_{t-1}, u_t)`` (h_{-1} = 0, A_c = clamp(A, max=0)) through
the closed form ``t*A_c + cummax(u - t*A_c)``; here the recurrence itself runs
as one fused kernel (bit-exact with the sequential recurrence; it differs from
the closed form by O(T ulp) rounding).  Gradients follow the same argmax path
(input wins ties, as torch.cummax's last-index rule does).  The three
projections of the input (gate_B, B_proj, gate_out) run as one GEMM on the
stacked weights (in inference an fp32-accurate 3xTF32 tensor-core GEMM,
``ops.linear``).
"""
from __future__ import annotations

import torch
import torch.nn as nn
from torch import Tensor

from . import ops
from .ops import tropical_scan


class TropicalSSM(nn.Module):
    def __init__(self, d_model: int, d_state: int = None):
        super().__init__()
        ds = d_state or d_model
        self.ds = ds
        self.A = nn.Parameter(torch.randn(ds) * 0.01)
        self.B_proj = nn.Linear(d_model, ds, bias=False)
        self.C_proj = nn.Linear(ds, d_model, bias=False)
        nn.init.zeros_(self.C_proj.weight)
        self.gate_B = nn.Linear(d_model, ds)
        self.gate_out = nn.Linear(d_model, d_model)
        nn.init.zeros_(self.gate_B.weight)
        nn.init.constant_(self.gate_B.bias, 2.0)
        nn.init.zeros_(self.gate_out.weight)
        nn.init.constant_(self.gate_out.bias, 2.0)
        self.mix = nn.Parameter(torch.tensor(0.0))

    def forward(self, x: Tensor) -> Tensor:
        # the three projections of x (gate_B, B_proj, gate_out) as one GEMM on
        # the stacked weights; x is read once
        ds, d = self.ds, x.shape[-1]
        w = torch.cat((self.gate_B.weight, self.B_proj.weight, self.gate_out.weight), dim=0)
        b = torch.cat((self.gate_B.bias, self.gate_B.bias.new_zeros(ds), self.gate_out.bias))
        gb, bp, go = ops.linear(x, w, b).split((ds, ds, d), dim=-1)
        u = torch.sigmoid(gb) * bp
        A_c = self.A.clamp(max=0)
        H = tropical_scan(u.contiguous(), None, A_c, 0.0)
        out = torch.sigmoid(go) * ops.linear(H, self.C_proj.weight)
        return torch.sigmoid(self.mix) * out
