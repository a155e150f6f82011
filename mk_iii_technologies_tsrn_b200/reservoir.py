"""Echo-state reservoir drop-ins for TSRN.

``EchoStateReservoir`` replaces the GRU-gated reservoir of
research/tsrn_dml.py:736-843; ``LeakyEchoStateReservoir`` replaces the leaky
``EchoStateReservoir`` of tsrn_gpu.py:435-487 (import it under that name).
Each has the reference's constructor (including its random initialisation
order), parameters and buffers, so a reference state dict loads unchanged.
The spectral scaling and the input projections are the reference's own
expressions; in inference (no autograd graph, CUDA tensors) the T-step
recurrence runs as one launch (``ops.esn_gru_fwd`` / ``ops.esn_leaky_fwd``)
instead of T iterations of small GEMMs.  With autograd the reference loop
runs, so training is unchanged.
"""
from __future__ import annotations

import torch
import torch.nn as nn

from . import ops


class EchoStateReservoir(nn.Module):
    def __init__(self, d_model: int, d_reservoir: int = None, sparsity: float = 0.9):
        super().__init__()
        dr = d_reservoir or d_model
        self.dr = dr
        self.W_in = nn.Linear(d_model, dr, bias=False)
        W_res = torch.randn(dr, dr)
        mask = torch.rand(dr, dr) > sparsity
        W_res = W_res * mask.float()
        with torch.no_grad():
            rho = torch.linalg.eigvals(W_res).abs().max().item()
            if rho > 0:
                W_res = W_res * (0.95 / rho)
        self.W_res = nn.Parameter(W_res)
        self.log_rho = nn.Parameter(torch.tensor(0.0))
        self.readout = nn.Linear(dr, d_model, bias=False)
        nn.init.zeros_(self.readout.weight)
        self.W_z = nn.Linear(2 * dr, dr)
        self.W_r = nn.Linear(2 * dr, dr)
        nn.init.zeros_(self.W_z.weight)
        nn.init.constant_(self.W_z.bias, 0.85)
        nn.init.zeros_(self.W_r.weight)
        nn.init.constant_(self.W_r.bias, 2.0)
        self.register_buffer("_cached_v", torch.zeros(dr))

    def _power_iter_spectral_radius(self, W: torch.Tensor, n_iter: int = 3) -> torch.Tensor:
        W_det = W.detach()
        with torch.no_grad():
            if torch.all(self._cached_v == 0):
                self._cached_v.copy_(torch.randn(W_det.shape[0], device=W_det.device,
                                                 dtype=W_det.dtype))
            v = self._cached_v.clone().unsqueeze(-1)
            for _ in range(n_iter):
                v = W_det @ v
                v_norm = v.norm()
                if v_norm > 0:
                    v = v / v_norm
            self._cached_v.copy_(v.squeeze(-1))
            return (W_det @ v).norm()

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        B, T, d = x.shape
        dr = self.dr
        rho_target = torch.sigmoid(self.log_rho) * 1.5
        rho_current = self._power_iter_spectral_radius(self.W_res)
        scale = rho_target / rho_current.clamp(min=1e-6)
        W_scaled = self.W_res * scale
        U = self.W_in(x)
        W_z_h = self.W_z.weight[:, :dr]
        W_z_u = self.W_z.weight[:, dr:]
        W_r_h = self.W_r.weight[:, :dr]
        W_r_u = self.W_r.weight[:, dr:]
        U_for_z = U @ W_z_u.T + self.W_z.bias
        U_for_r = U @ W_r_u.T + self.W_r.bias
        needs_graph = torch.is_grad_enabled() and any(
            t.requires_grad for t in (x, *self.parameters()))
        if not needs_graph and x.is_cuda:
            H = ops.esn_gru_fwd(U, U_for_z, U_for_r, W_z_h, W_r_h, W_scaled.detach())
            return self.readout(H)
        # the reference loop (autograd through time)
        h = torch.zeros(B, dr, device=x.device, dtype=x.dtype)
        outs = []
        for t in range(T):
            u_t = U[:, t, :]
            z = torch.sigmoid(h @ W_z_h.T + U_for_z[:, t, :])
            r = torch.sigmoid(h @ W_r_h.T + U_for_r[:, t, :])
            h_tilde = torch.tanh((r * h) @ W_scaled.T + u_t)
            h = (1 - z) * h + z * h_tilde
            outs.append(h)
        return self.readout(torch.stack(outs, dim=1))


class LeakyEchoStateReservoir(nn.Module):
    """Leaky echo-state reservoir (tsrn_gpu.py:435-487):
    h_t = (1 - lk) h_{t-1} + lk tanh(h_{t-1} W_scaled^T + W_in x_t), lk = sigmoid(leak)."""

    def __init__(self, d_model: int, d_reservoir: int = None, sparsity: float = 0.9):
        super().__init__()
        dr = d_reservoir or d_model
        self.dr = dr
        self.W_in = nn.Linear(d_model, dr, bias=False)
        W_res = torch.randn(dr, dr)
        mask = torch.rand(dr, dr) > sparsity
        W_res = W_res * mask.float()
        with torch.no_grad():
            rho = torch.linalg.eigvals(W_res).abs().max().real
            if rho > 0:
                W_res = W_res * (0.95 / rho.item())
        self.W_res = nn.Parameter(W_res)
        self.log_rho = nn.Parameter(torch.tensor(0.0))
        self.readout = nn.Linear(dr, d_model, bias=False)
        nn.init.zeros_(self.readout.weight)
        self.leak = nn.Parameter(torch.tensor(0.3))

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        B, T, d = x.shape
        rho = torch.sigmoid(self.log_rho) * 1.5
        eigs = torch.linalg.eigvals(self.W_res).abs()
        W_scaled = self.W_res * (rho / (eigs.max().real.clamp(min=1e-6)))
        lk = torch.sigmoid(self.leak)
        needs_graph = torch.is_grad_enabled() and any(
            t.requires_grad for t in (x, *self.parameters()))
        if not needs_graph and x.is_cuda:
            H = ops.esn_leaky_fwd(self.W_in(x), W_scaled, lk)
            return self.readout(H)
        h = torch.zeros(B, self.dr, device=x.device, dtype=x.dtype)
        outs = []
        for t in range(T):
            u = self.W_in(x[:, t, :])
            h = (1 - lk) * h + lk * torch.tanh(h @ W_scaled.T + u)
            outs.append(h)
        return self.readout(torch.stack(outs, dim=1))
