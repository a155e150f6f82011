"""The tropical path of a TSRN block (research/tsrn_dml.py:1050-1110) on the B200 kernels.

``TSRNBlock.forward`` (research/tsrn_dml.py:1096-1110) runs pre-LayerNorm
residual branches in this order: tropical attention, sheaf diffusion, the
echo-state reservoir (scale 1), the tropical SSM, the Clifford FFN, and p-adic
memory / attention.  Three of them are the tropical hot path this library
accelerates:

* ``attn``          -- :class:`~.tsrn_attention.TropicalAttention` (fused LSE
  score + ALiBi + causal + top-k + softmax + @V kernel),
* ``reservoir``     -- :class:`~.reservoir.EchoStateReservoir` (the whole
  GRU-gated recurrence in one launch),
* ``tropical_ssm``  -- :class:`~.ssm.TropicalSSM` (max-plus scan kernel).

:class:`TSRNTropicalPath` holds those three branches, with their LayerNorms,
under the block's own attribute names (``ln_attn``/``attn``, ``ln_res``/
``reservoir``, ``ln_ssm``/``tropical_ssm``), so the matching subset of a
``TSRNBlock`` state dict loads unchanged.  It runs the branches in the
block's order without the non-tropical ones between them (sheaf diffusion,
Clifford FFN, p-adic modules).  :func:`swap_into` instead puts this library's
modules into a reference ``TSRNBlock`` in place, with the same weights, so the
reference model itself runs its tropical branches on these kernels.
"""
from __future__ import annotations

from typing import Dict, Optional

import torch
import torch.nn as nn

from . import ops
from .reservoir import EchoStateReservoir
from .ssm import TropicalSSM
from .tsrn_attention import TropicalAttention

BRANCHES = ("attn", "reservoir", "tropical_ssm")


class TSRNTropicalPath(nn.Module):
    def __init__(self, d_model: int, top_k: int, n_heads: int, *, use_reservoir: bool = True,
                 use_tropical_ssm: bool = True, dropout: float = 0.0):
        super().__init__()
        self.ln_attn = nn.LayerNorm(d_model)
        self.attn = TropicalAttention(d_model, top_k=top_k, n_heads=n_heads, dropout=dropout)
        self.use_reservoir = use_reservoir
        if use_reservoir:
            self.ln_res = nn.LayerNorm(d_model)
            self.reservoir = EchoStateReservoir(d_model, d_reservoir=d_model // 2)
        self.use_tropical_ssm = use_tropical_ssm
        if use_tropical_ssm:
            self.ln_ssm = nn.LayerNorm(d_model)
            self.tropical_ssm = TropicalSSM(d_model)

    def forward(self, x: torch.Tensor,
                events: Optional[Dict[str, tuple]] = None) -> torch.Tensor:
        """``events`` (optional): branch name -> (start, end) CUDA events recorded
        around that branch on the current stream, for per-branch timing."""
        def branch(name, ln, mod, h):
            if events is not None and name in events:
                events[name][0].record()
            out = h + mod(ops.layer_norm(h, ln.weight, ln.bias, ln.eps))
            if events is not None and name in events:
                events[name][1].record()
            return out

        x = branch("attn", self.ln_attn, self.attn, x)
        if self.use_reservoir:
            x = branch("reservoir", self.ln_res, self.reservoir, x)
        if self.use_tropical_ssm:
            x = branch("tropical_ssm", self.ln_ssm, self.tropical_ssm, x)
        return x


def _like(new: nn.Module, old: nn.Module) -> nn.Module:
    p = next(old.parameters())
    new = new.to(device=p.device, dtype=p.dtype)
    new.load_state_dict(old.state_dict())
    new.train(old.training)
    return new


def swap_into(block: nn.Module) -> nn.Module:
    """Replace the tropical branches of a reference ``TSRNBlock`` (or any module with
    ``attn`` / ``reservoir`` / ``tropical_ssm`` attributes of the reference classes)
    by this library's modules carrying the same parameters and buffers.  Returns
    the block.  Everything else in the block is left as it is."""
    attn = getattr(block, "attn", None)
    if attn is not None and not isinstance(attn, TropicalAttention):
        d = attn.Wq.in_features
        mod = TropicalAttention(d, top_k=attn.top_k, n_heads=attn.H, dropout=attn.drop.p)
        block.attn = _like(mod, attn)
    res = getattr(block, "reservoir", None)
    if res is not None and not isinstance(res, EchoStateReservoir):
        mod = EchoStateReservoir(res.W_in.in_features, d_reservoir=res.W_in.out_features)
        block.reservoir = _like(mod, res)
    ssm = getattr(block, "tropical_ssm", None)
    if ssm is not None and not isinstance(ssm, TropicalSSM):
        mod = TropicalSSM(ssm.B_proj.in_features, ssm.B_proj.out_features)
        block.tropical_ssm = _like(mod, ssm)
    return block
