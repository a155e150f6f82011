"""One-launch backward through time of the reservoir recurrences
(``ops.esn_gru_bwd``, ``ops.esn_leaky_bwd``) against the reverse-time loop of
autograd over the reference loops (research/tsrn_dml.py:834-840,
tsrn_gpu.py:480-484), evaluated here step by step in float64.

The kernels differ from that loop only in the fp32 rounding of their dot
products (summation order), so they are compared within 2e-4 of each
output's scale.  Shapes cover the model's reservoir (B = 64, dr = 320), a
width that is not a multiple of 4, weights too large for shared memory (read
from L2), a single step and empty inputs."""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _ops():
    from mk_iii_technologies_tsrn_b200 import ops
    return ops


def _close(got, ref, rtol=2e-4):
    got = got.double().cpu()
    scale = ref.abs().max().item() + 1e-30
    err = (got - ref).abs().max().item() / scale
    assert err < rtol, err


def _gru_loop(dH, fa, fz, fr, keep, r, Wzh, Wrh, Ws):
    B, T, dr = dH.shape
    out = [torch.zeros_like(dH) for _ in range(3)]
    g = torch.zeros(B, dr, dtype=dH.dtype)
    for t in range(T - 1, -1, -1):
        dh = dH[:, t] + g
        dah = dh * fa[:, t]
        dm = dah @ Ws
        dar = dm * fr[:, t]
        daz = dh * fz[:, t]
        g = dh * keep[:, t] + dm * r[:, t] + daz @ Wzh + dar @ Wrh
        out[0][:, t], out[1][:, t], out[2][:, t] = dah, daz, dar
    return out


def _leaky_loop(dH, fa, Ws, lk):
    B, T, dr = dH.shape
    dA, dHs = torch.zeros_like(dH), torch.zeros_like(dH)
    g = torch.zeros(B, dr, dtype=dH.dtype)
    for t in range(T - 1, -1, -1):
        dh = dH[:, t] + g
        da = dh * fa[:, t]
        g = dh * (1.0 - lk) + da @ Ws
        dA[:, t], dHs[:, t] = da, dh
    return dA, dHs


def _factors(rng, shape, n):
    # factor ranges of the real recurrence: gate derivatives in (0, 1/4],
    # keep in (0, 1)
    return [torch.tensor(rng.uniform(0.0, 0.25 if i < 3 else 1.0, shape).astype(np.float32))
            for i in range(n)]


@pytest.mark.parametrize("B,T,dr", [(3, 40, 48), (64, 96, 320), (5, 17, 70), (2, 24, 640),
                                    (1, 1, 8)])
def test_gru_bwd_vs_loop(cuda, B, T, dr):
    rng = np.random.default_rng(B * 7 + T + dr)
    dH = torch.tensor(rng.standard_normal((B, T, dr)).astype(np.float32))
    fa, fz, fr, keep = _factors(rng, (B, T, dr), 4)
    r = torch.tensor(rng.uniform(0.0, 1.0, (B, T, dr)).astype(np.float32))
    W = [torch.tensor((0.9 / np.sqrt(dr) * rng.standard_normal((dr, dr))).astype(np.float32))
         for _ in range(3)]
    got = _ops().esn_gru_bwd(*(t.to(cuda) for t in (dH, fa, fz, fr, keep, r, *W)))
    ref = _gru_loop(*(t.double() for t in (dH, fa, fz, fr, keep, r, *W)))
    for a, b in zip(got, ref):
        _close(a, b)


def test_gru_bwd_strided_weights(cuda):
    # Wzh / Wrh as column slices of the stacked gate weights, as the module passes them
    rng = np.random.default_rng(3)
    B, T, dr = 4, 33, 64
    dH = torch.tensor(rng.standard_normal((B, T, dr)).astype(np.float32))
    fa, fz, fr, keep, r = _factors(rng, (B, T, dr), 5)
    Wz = torch.tensor((0.1 * rng.standard_normal((dr, 2 * dr))).astype(np.float32))
    Wr = torch.tensor((0.1 * rng.standard_normal((dr, 2 * dr))).astype(np.float32))
    Ws = torch.tensor((0.1 * rng.standard_normal((dr, dr))).astype(np.float32))
    dev = [t.to(cuda) for t in (dH, fa, fz, fr, keep, r)]
    Wzd, Wrd = Wz.to(cuda), Wr.to(cuda)
    got = _ops().esn_gru_bwd(*dev, Wzd[:, :dr], Wrd[:, :dr], Ws.to(cuda))
    ref = _gru_loop(*(t.double() for t in (dH, fa, fz, fr, keep, r)), Wz[:, :dr].double(),
                    Wr[:, :dr].double(), Ws.double())
    for a, b in zip(got, ref):
        _close(a, b)


@pytest.mark.parametrize("B,T,dr", [(3, 40, 48), (64, 96, 640), (5, 17, 70), (1, 1, 8)])
def test_leaky_bwd_vs_loop(cuda, B, T, dr):
    rng = np.random.default_rng(B * 11 + T + dr)
    dH = torch.tensor(rng.standard_normal((B, T, dr)).astype(np.float32))
    fa = torch.tensor(rng.uniform(0.0, 0.4, (B, T, dr)).astype(np.float32))
    Ws = torch.tensor((0.9 / np.sqrt(dr) * rng.standard_normal((dr, dr))).astype(np.float32))
    lk = torch.tensor([0.37])
    dA, dHs = _ops().esn_leaky_bwd(dH.to(cuda), fa.to(cuda), Ws.to(cuda), lk.to(cuda))
    rA, rHs = _leaky_loop(dH.double(), fa.double(), Ws.double(), 0.37)
    _close(dA, rA)
    _close(dHs, rHs)


def test_bwd_empty(cuda):
    ops = _ops()
    z = torch.zeros(2, 0, 16, device=cuda)
    W = torch.zeros(16, 16, device=cuda)
    outs = ops.esn_gru_bwd(z, z, z, z, z, z, W, W, W)
    assert all(o.shape == z.shape for o in outs)
    dA, dHs = ops.esn_leaky_bwd(z, z, W, torch.tensor([0.5], device=cuda))
    assert dA.shape == z.shape and dHs.shape == z.shape


def test_bwd_two_calls_in_a_row(cuda):
    # the planner's cached plan and the kernel's state carry nothing between calls
    ops = _ops()
    rng = np.random.default_rng(9)
    B, T, dr = 8, 20, 96
    W = [torch.tensor((0.1 * rng.standard_normal((dr, dr))).astype(np.float32)).to(cuda)
         for _ in range(3)]
    for _ in range(2):
        args = [torch.tensor(rng.standard_normal((B, T, dr)).astype(np.float32))]
        args = [a.to(cuda) for a in args + _factors(rng, (B, T, dr), 5)]
        got = ops.esn_gru_bwd(*args, *W)
        ref = _gru_loop(*(a.double().cpu() for a in args), *(w.double().cpu() for w in W))
        for a, b in zip(got, ref):
            _close(a, b)
