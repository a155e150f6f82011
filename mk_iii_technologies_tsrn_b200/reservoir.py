"""Echo-state reservoir drop-ins for TSRN on the B200 recurrence kernels.

``EchoStateReservoir`` replaces the GRU-gated reservoir of
research/tsrn_dml.py:736-843; ``LeakyEchoStateReservoir`` replaces the leaky
``EchoStateReservoir`` of tsrn_gpu.py:435-487 (import it under that name).
Both keep the reference's constructor, parameter and buffer names (so a
reference state dict loads unchanged) and its spectral scaling of the
recurrent matrix.  The recurrence over T steps runs as one launch
(``ops.esn_gru_fwd`` / ``ops.esn_leaky_fwd``) in inference and in training;
for training, :class:`GRUReservoirFunction` / :class:`LeakyReservoirFunction`
add a backward through time: every step's gates are recomputed at once from the
saved states (batched GEMMs), one launch (``ops.esn_gru_bwd`` /
``ops.esn_leaky_bwd``) carries the state gradient backwards through all steps,
and the weight gradients are batched GEMMs over all steps (the gate
recomputation and the weight gradients as fp32-accurate 3xTF32 tensor-core
GEMMs).  CUDA tensors only (no CPU fallback).
"""
from __future__ import annotations

import torch
import torch.nn as nn

from . import ops


def _scaled_sparse_gaussian(n: int, sparsity: float, radius: float) -> torch.Tensor:
    """An n x n N(0,1) matrix keeping each entry with probability 1 - sparsity, scaled
    to spectral radius ``radius`` (the reference draws the entries, then the mask)."""
    W = torch.randn(n, n)
    W = W * (torch.rand(n, n) > sparsity).float()
    with torch.no_grad():
        rho = torch.linalg.eigvals(W).abs().max().real.item()
    return W * (radius / rho) if rho > 0 else W


def _previous_states(H: torch.Tensor, h0=None) -> torch.Tensor:
    """h_{t-1} for every step t of H [B, T, dr] (h_{-1} = 0)."""
    first = torch.zeros_like(H[:, :1]) if h0 is None else h0.unsqueeze(1)
    return torch.cat((first, H[:, :-1]), dim=1)


class GRUReservoirFunction(torch.autograd.Function):
    """H [B, T, dr] of the GRU-gated recurrence (h_{-1} = 0)
    z = sig(h Wzh^T + Uz_t), r = sig(h Wrh^T + Ur_t),
    h~ = tanh((r * h) Ws^T + U_t), h <- (1 - z) h + z h~."""

    @staticmethod
    def forward(ctx, U, Uz, Ur, Wzh, Wrh, Ws):
        H = ops.esn_gru_fwd(U, Uz, Ur, Wzh, Wrh, Ws)
        ctx.save_for_backward(U, Uz, Ur, Wzh, Wrh, Ws, H)
        return H

    @staticmethod
    def backward(ctx, dH):
        U, Uz, Ur, Wzh, Wrh, Ws, H = ctx.saved_tensors
        B, T, dr = H.shape
        Hp = _previous_states(H)
        flat = lambda t: t.reshape(B * T, dr)   # noqa: E731
        # every step's gates at once (fp32-accurate 3xTF32 GEMMs)
        # both gates' recurrent terms from one product with the stacked weights
        hz, hr = ops.matmul_tf32x3(flat(Hp), torch.cat((Wzh, Wrh), 0).t()).split(dr, dim=1)
        z = torch.sigmoid(hz.reshape(B, T, dr) + Uz)
        r = torch.sigmoid(hr.reshape(B, T, dr) + Ur)
        m = r * Hp
        hc = torch.tanh(ops.matmul_tf32x3(flat(m), Ws.t()).view(B, T, dr) + U)
        # per-step factors, all steps at once
        fa = z * (1.0 - hc * hc)              # d h / d a_h  (a_h = m Ws^T + U)
        fz = (hc - Hp) * z * (1.0 - z)        # d h / d a_z
        fr = Hp * r * (1.0 - r)               # d m / d a_r
        keep = 1.0 - z
        # the reverse-time loop over the state gradient: one launch
        dAh, dAz, dAr = ops.esn_gru_bwd(dH, fa, fz, fr, keep, r, Wzh, Wrh, Ws)
        dWs = ops.matmul_tn_tf32x3(flat(dAh), flat(m))
        dWzh = ops.matmul_tn_tf32x3(flat(dAz), flat(Hp))
        dWrh = ops.matmul_tn_tf32x3(flat(dAr), flat(Hp))
        return dAh, dAz, dAr, dWzh, dWrh, dWs


class LeakyReservoirFunction(torch.autograd.Function):
    """H [B, T, dr] of h <- (1 - lk) h + lk tanh(h Ws^T + U_t) (h_{-1} = 0), lk a
    one-element tensor."""

    @staticmethod
    def forward(ctx, U, Ws, lk):
        H = ops.esn_leaky_fwd(U, Ws, lk)
        ctx.save_for_backward(U, Ws, lk, H)
        return H

    @staticmethod
    def backward(ctx, dH):
        U, Ws, lk, H = ctx.saved_tensors
        B, T, dr = H.shape
        Hp = _previous_states(H)
        flat = lambda t: t.reshape(B * T, dr)   # noqa: E731
        s = torch.tanh(ops.matmul_tf32x3(flat(Hp), Ws.t()).view(B, T, dr) + U)
        fa = lk * (1.0 - s * s)
        # the reverse-time loop over the state gradient: one launch
        dA, dHs = ops.esn_leaky_bwd(dH, fa, Ws, lk)
        dWs = ops.matmul_tn_tf32x3(flat(dA), flat(Hp))
        dlk = (dHs * (s - Hp)).sum().reshape(lk.shape)
        return dA, dWs, dlk


def _needs_graph(x: torch.Tensor, module: nn.Module) -> bool:
    return torch.is_grad_enabled() and (x.requires_grad or any(
        p.requires_grad for p in module.parameters()))


class EchoStateReservoir(nn.Module):
    """GRU-gated echo-state reservoir (research/tsrn_dml.py:736-843).  Submodules are
    created in the reference's order, so a seeded construction draws the same
    initial weights."""

    def __init__(self, d_model: int, d_reservoir: int = None, sparsity: float = 0.9):
        super().__init__()
        dr = d_reservoir or d_model
        self.dr = dr
        self.W_in = nn.Linear(d_model, dr, bias=False)
        self.W_res = nn.Parameter(_scaled_sparse_gaussian(dr, sparsity, 0.95))
        self.log_rho = nn.Parameter(torch.tensor(0.0))
        self.readout = nn.Linear(dr, d_model, bias=False)
        nn.init.zeros_(self.readout.weight)
        self.W_z = nn.Linear(2 * dr, dr)
        self.W_r = nn.Linear(2 * dr, dr)
        for gate, bias in ((self.W_z, 0.85), (self.W_r, 2.0)):
            nn.init.zeros_(gate.weight)
            nn.init.constant_(gate.bias, bias)
        self.register_buffer("_cached_v", torch.zeros(dr))

    @torch.no_grad()
    def _radius_estimate(self, iters: int = 3) -> torch.Tensor:
        """Spectral radius of W_res by ``iters`` normalised power iterations started
        from the persistent vector ``_cached_v`` (drawn once if still zero), which is
        advanced in place -- research/tsrn_dml.py:783-806."""
        W = self.W_res.detach()
        if not bool(self._cached_v.any()):
            self._cached_v.copy_(torch.randn(self.dr, device=W.device, dtype=W.dtype))
        v = self._cached_v.clone().unsqueeze(-1)
        for _ in range(iters):
            v = W @ v
            n = v.norm()
            v = torch.where(n > 0, v / n, v)     # no host round trip per iteration
        self._cached_v.copy_(v.squeeze(-1))
        return (W @ v).norm()

    def _scaled_recurrent(self) -> torch.Tensor:
        target = torch.sigmoid(self.log_rho) * 1.5
        return self.W_res * (target / self._radius_estimate().clamp(min=1e-6))

    def recurrence_inputs(self, x: torch.Tensor):
        """(U, Uz, Ur, Wzh, Wrh, Ws) of ``ops.esn_gru_fwd`` for x [B, T, d_model]."""
        dr = self.dr
        Ws = self._scaled_recurrent()
        U = ops.linear(x, self.W_in.weight)
        Wzh, Wzu = self.W_z.weight.split(dr, dim=1)
        Wrh, Wru = self.W_r.weight.split(dr, dim=1)
        # both gates' input terms as one GEMM on the stacked input halves
        Uzr = ops.linear(U, torch.cat((Wzu, Wru), dim=0), torch.cat((self.W_z.bias, self.W_r.bias)))
        Uz, Ur = Uzr.split(dr, dim=-1)
        return U, Uz.contiguous(), Ur.contiguous(), Wzh, Wrh, Ws

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        U, Uz, Ur, Wzh, Wrh, Ws = self.recurrence_inputs(x)
        if _needs_graph(x, self):
            H = GRUReservoirFunction.apply(U, Uz, Ur, Wzh, Wrh, Ws)
        else:
            H = ops.esn_gru_fwd(U, Uz, Ur, Wzh, Wrh, Ws.detach())
        return ops.linear(H, self.readout.weight)


class LeakyEchoStateReservoir(nn.Module):
    """Leaky echo-state reservoir (tsrn_gpu.py:435-487):
    h_t = (1 - lk) h_{t-1} + lk tanh(h_{t-1} W_scaled^T + W_in x_t), lk = sigmoid(leak),
    W_scaled = W_res * sigmoid(log_rho) * 1.5 / (largest |eigenvalue| of W_res)."""

    def __init__(self, d_model: int, d_reservoir: int = None, sparsity: float = 0.9):
        super().__init__()
        dr = d_reservoir or d_model
        self.dr = dr
        self.W_in = nn.Linear(d_model, dr, bias=False)
        self.W_res = nn.Parameter(_scaled_sparse_gaussian(dr, sparsity, 0.95))
        self.log_rho = nn.Parameter(torch.tensor(0.0))
        self.readout = nn.Linear(dr, d_model, bias=False)
        nn.init.zeros_(self.readout.weight)
        self.leak = nn.Parameter(torch.tensor(0.3))

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        radius = torch.linalg.eigvals(self.W_res).abs().max().real.clamp(min=1e-6)
        Ws = self.W_res * (torch.sigmoid(self.log_rho) * 1.5 / radius)
        lk = torch.sigmoid(self.leak)
        U = ops.linear(x, self.W_in.weight)
        if _needs_graph(x, self):
            H = LeakyReservoirFunction.apply(U, Ws, lk.reshape(1))
        else:
            H = ops.esn_leaky_fwd(U, Ws.detach(), lk.detach())
        return ops.linear(H, self.readout.weight)
