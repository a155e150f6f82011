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
