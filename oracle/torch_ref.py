"""The reference's PyTorch expressions, restated for CPU timing -- test
infrastructure only (the timed CPU baseline of bench.py and its
``--impl reference`` arm).

* ``maxplus_fwd_torch``: tropformer.py:131 (``W.unsqueeze(0) + x.unsqueeze(1)``)
  and :141 (``.max(dim=-1)``), chunked over rows so that the [rows, N, K]
  temporary stays bounded (the full broadcast is 2 TiB at M=N=K=8192; the
  chunking follows the pattern described in TropFormer_Benchmarks.md:600-609).
* ``scan_closed_form_torch``: research/tsrn_dml.py:961-972 with h_{-1} given by
  the leading row (the reference's TropicalSSM evaluation).
"""
from __future__ import annotations

import torch


def maxplus_fwd_torch(x: torch.Tensor, w: torch.Tensor, chunk_elems: int = 1 << 25):
    M, K = x.shape
    N = w.shape[0]
    rows = max(1, chunk_elems // max(1, N * K))
    ys, idx = [], []
    for m0 in range(0, M, rows):
        scores = w.unsqueeze(0) + x[m0:m0 + rows].unsqueeze(1)
        mx = scores.max(dim=-1)
        ys.append(mx.values)
        idx.append(mx.indices)
    return torch.cat(ys), torch.cat(idx)


def scan_closed_form_torch(u: torch.Tensor, A_c: torch.Tensor):
    B, T, C = u.shape
    t_idx = torch.arange(T, dtype=u.dtype).unsqueeze(-1)
    shifted = u - t_idx * A_c
    G = torch.cat([A_c.unsqueeze(0).expand(B, -1).unsqueeze(1), shifted], dim=1)
    cm, _ = G.cummax(dim=1)
    return t_idx.unsqueeze(0) * A_c + cm[:, 1:, :]


class DTNAttentionRef(torch.nn.Module):
    """deep_tropical_net.py:90-165 (DTNAttention) on the reference's own torch
    expressions: TropicalLinear Q/K (tropformer.py:127-145, train-mode STE),
    classical V/out projections, the gated tropical/classical score
    (deep_tropical_net.py:145-155) and MaslovTemperature (tropformer.py:206-212).
    For CPU timing only."""

    def __init__(self, d_model: int, num_heads: int, ste_temp: float = 1.0):
        super().__init__()
        import math
        self.h, self.dk = num_heads, d_model // num_heads
        self.scale = self.dk ** -0.5
        self.ste_temp = ste_temp
        self.q_w = torch.nn.Parameter(torch.empty(d_model, d_model).uniform_(-0.5, 0.5))
        self.q_b = torch.nn.Parameter(torch.zeros(d_model))
        self.k_w = torch.nn.Parameter(torch.empty(d_model, d_model).uniform_(-0.5, 0.5))
        self.k_b = torch.nn.Parameter(torch.zeros(d_model))
        self.v = torch.nn.Linear(d_model, d_model)
        self.o = torch.nn.Linear(d_model, d_model)
        self.gate = torch.nn.Linear(d_model, num_heads)
        self.log_temps = torch.nn.Parameter(torch.full((num_heads,), math.log(1.0)))

    def _trop_linear(self, x, w, b):
        lead = x.shape[:-1]
        xf = x.reshape(-1, x.shape[-1])
        scores = w.unsqueeze(0) + xf.unsqueeze(1)
        hard = scores.detach().max(dim=-1).values
        soft_w = torch.softmax(scores / self.ste_temp, dim=-1)
        soft = (soft_w * scores).sum(dim=-1)
        out = hard + (soft - soft.detach()) + b
        return out.reshape(*lead, w.shape[0])

    def forward(self, x):
        B, L, D = x.shape
        split = lambda t: t.view(B, L, self.h, self.dk).transpose(1, 2)
        Q = split(self._trop_linear(x, self.q_w, self.q_b))
        K = split(self._trop_linear(x, self.k_w, self.k_b))
        V = split(self.v(x))
        cls = torch.matmul(Q, K.transpose(-2, -1)) * self.scale
        trop = (Q.unsqueeze(3) + K.unsqueeze(2)).max(dim=-1).values * self.scale
        g = torch.sigmoid(self.gate(x)).permute(0, 2, 1).unsqueeze(-1)
        scores = g * trop + (1.0 - g) * cls
        tau = self.log_temps.exp().clamp(min=0.02, max=10.0).view(1, -1, 1, 1)
        attn = torch.softmax(scores / tau, dim=-1)
        out = torch.matmul(attn, V).transpose(1, 2).contiguous().view(B, L, D)
        return self.o(out), attn


def tropical_linear_fwd_bwd_torch(x: torch.Tensor, w: torch.Tensor, g: torch.Tensor):
    """Eval-mode TropicalLinear forward and backward (tropformer.py:131,141 and the
    autograd of ``.max(dim=-1).values``): returns (y, argmax, grad_x, grad_w)."""
    x = x.detach().requires_grad_(True)
    w = w.detach().requires_grad_(True)
    mx = (w.unsqueeze(0) + x.unsqueeze(1)).max(dim=-1)
    gx, gw = torch.autograd.grad(mx.values, (x, w), g)
    return mx.values.detach(), mx.indices, gx, gw


def tsrn_attention_torch(Q, K, V, slopes, top_k: int, causal: bool = True, q_chunk: int = 64):
    """TropicalAttention after RoPE on the reference's own torch expressions
    (research/tsrn_dml.py:384-436 _attend_chunk: logsumexp score per query chunk,
    ALiBi, causal mask, top-k threshold, softmax, @V), fp32.  CPU timing only."""
    B, H, T, dh = Q.shape
    Tkv = K.shape[2]
    out = []
    for qi in range(0, T, q_chunk):
        q_end = min(qi + q_chunk, T)
        Qq = Q[:, :, qi:q_end]
        scores = torch.logsumexp(Qq.unsqueeze(3) + K.unsqueeze(2), dim=-1)
        q_pos = torch.arange(qi, q_end)
        k_pos = torch.arange(0, Tkv)
        dist = (q_pos.unsqueeze(1) - k_pos.unsqueeze(0)).abs()
        scores = scores - slopes.view(-1, 1, 1) * dist.unsqueeze(0)
        if causal:
            scores = scores.masked_fill((k_pos.unsqueeze(0) > q_pos.unsqueeze(1))[None, None],
                                        float("-inf"))
        thr = scores.topk(min(top_k, Tkv), dim=-1).values[..., -1:]
        scores = scores.masked_fill(scores < thr, float("-inf"))
        out.append(torch.softmax(scores, dim=-1) @ V)
    return torch.cat(out, dim=2)


def esn_leaky_torch(U, Ws, lk):
    """The leaky reservoir loop of tsrn_gpu.py:479-487 on precomputed inputs U = W_in(x):
    h = (1 - lk) h + lk tanh(h Ws^T + U_t), h_{-1} = 0; returns H [B, T, dr]."""
    B, T, dr = U.shape
    h = torch.zeros(B, dr, dtype=U.dtype)
    outs = []
    Wt = Ws.T
    for t in range(T):
        h = (1 - lk) * h + lk * torch.tanh(h @ Wt + U[:, t, :])
        outs.append(h)
    return torch.stack(outs, dim=1)


def esn_gru_torch(U, Uz, Ur, Wzh, Wrh, Ws):
    """The GRU-gated reservoir loop of research/tsrn_dml.py:832-842 on precomputed
    inputs; returns H [B, T, dr]."""
    B, T, dr = U.shape
    h = torch.zeros(B, dr, dtype=U.dtype)
    outs = []
    for t in range(T):
        z = torch.sigmoid(h @ Wzh.T + Uz[:, t, :])
        r = torch.sigmoid(h @ Wrh.T + Ur[:, t, :])
        h_tilde = torch.tanh((r * h) @ Ws.T + U[:, t, :])
        h = (1 - z) * h + z * h_tilde
        outs.append(h)
    return torch.stack(outs, dim=1)


def _rope_torch(q, k, inv_freq):
    """Rotary embedding of research/tsrn_dml.py:284-319 (half-split rotation)."""
    T = q.shape[2]
    freqs = torch.outer(torch.arange(T, dtype=inv_freq.dtype), inv_freq)
    emb = torch.cat([freqs, freqs], dim=-1)
    cos, sin = emb.cos(), emb.sin()

    def rot(t):
        h = t.shape[-1] // 2
        return torch.cat([-t[..., h:], t[..., :h]], dim=-1)

    return q * cos + rot(q) * sin, k * cos + rot(k) * sin


def tsrn_block_torch(x, sd, heads: int, top_k: int):
    """The tropical branches of TSRNBlock.forward (research/tsrn_dml.py:1096-1106) in
    the block's order -- attention (:472-540 with the _attend_chunk core of
    tsrn_attention_torch), GRU reservoir (:808-843), TropicalSSM (:951-980 with the
    closed-form scan) -- on CPU torch from a state dict ``sd`` with the block's key
    names.  CPU timing only."""
    import torch.nn.functional as F

    def ln(t, p, n=None):
        return F.layer_norm(t, (n or t.shape[-1],), sd[p + ".weight"], sd[p + ".bias"])

    B, T, d = x.shape
    dh = d // heads
    # attention branch
    h = ln(x, "ln_attn")
    def heads_of(w):
        return (h @ sd[w].T).view(B, T, heads, dh).permute(0, 2, 1, 3)
    Q = ln(heads_of("attn.Wq.weight"), "attn.q_norm")
    K = ln(heads_of("attn.Wk.weight"), "attn.k_norm")
    V = heads_of("attn.Wv.weight")
    Q, K = _rope_torch(Q, K, sd["attn.rope.inv_freq"])
    ctx = tsrn_attention_torch(Q, K, V, sd["attn.alibi_slopes"], min(top_k, T))
    x = x + ctx.permute(0, 2, 1, 3).reshape(B, T, d) @ sd["attn.Wo.weight"].T
    # reservoir branch: spectral scale from 3 power iterations started at the
    # module's cached vector (research/tsrn_dml.py:783-806, :812-814)
    h = ln(x, "ln_res")
    Wres = sd["reservoir.W_res"]
    dr = Wres.shape[0]
    v = sd["reservoir._cached_v"].clone().unsqueeze(-1)
    for _ in range(3):
        v = Wres @ v
        nv = v.norm()
        if nv > 0:
            v = v / nv
    rho = torch.sigmoid(sd["reservoir.log_rho"]) * 1.5
    Ws = Wres * (rho / (Wres @ v).norm().clamp(min=1e-6))
    U = h @ sd["reservoir.W_in.weight"].T
    Wz, Wr = sd["reservoir.W_z.weight"], sd["reservoir.W_r.weight"]
    Uz = U @ Wz[:, dr:].T + sd["reservoir.W_z.bias"]
    Ur = U @ Wr[:, dr:].T + sd["reservoir.W_r.bias"]
    Hres = esn_gru_torch(U, Uz, Ur, Wz[:, :dr], Wr[:, :dr], Ws)
    x = x + Hres @ sd["reservoir.readout.weight"].T
    # tropical SSM branch
    h = ln(x, "ln_ssm")
    u = torch.sigmoid(h @ sd["tropical_ssm.gate_B.weight"].T + sd["tropical_ssm.gate_B.bias"]) \
        * (h @ sd["tropical_ssm.B_proj.weight"].T)
    Hs = scan_closed_form_torch(u, sd["tropical_ssm.A"].clamp(max=0))
    out = torch.sigmoid(h @ sd["tropical_ssm.gate_out.weight"].T
                        + sd["tropical_ssm.gate_out.bias"]) * (Hs @ sd["tropical_ssm.C_proj.weight"].T)
    return x + torch.sigmoid(sd["tropical_ssm.mix"]) * out
