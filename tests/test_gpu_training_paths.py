"""Training paths of the TSRN drop-ins: forward on the fused kernels, backward
by this library's analytic gradients (GRUReservoirFunction,
LeakyReservoirFunction, TopKAttentionFunction) -- against float64 autograd of
the reference's own expressions on the CPU (oracle/torch_ref.py: the loops of
research/tsrn_dml.py:832-842 and tsrn_gpu.py:479-484, the attention core of
research/tsrn_dml.py:384-436) and against the reference modules' outputs
(golden fixtures)."""
import numpy as np
import pytest
import torch

from conftest import load_golden
from oracle.torch_ref import esn_gru_torch, esn_leaky_torch, tsrn_attention_torch

pytestmark = pytest.mark.gpu


def _close(got, ref, rtol=2e-4, atol=2e-5):
    got = got.detach().double().cpu()
    ref = ref.detach().double()
    scale = ref.abs().max().item() + 1e-30
    assert torch.allclose(got, ref, rtol=rtol, atol=atol * max(1.0, scale)), \
        float((got - ref).abs().max() / scale)


def test_gru_reservoir_training_matches_autograd(cuda):
    from mk_iii_technologies_tsrn_b200.reservoir import EchoStateReservoir
    g = load_golden("esn")
    d = g["x"].shape[-1]
    state = {k[2:]: torch.tensor(v) for k, v in g.items() if k.startswith("p_")}
    mod = EchoStateReservoir(d, d).to(cuda).train()
    mod.load_state_dict(state)
    x = torch.tensor(g["x"], device=cuda, requires_grad=True)
    y = mod(x)
    np.testing.assert_allclose(y.detach().cpu().numpy(), g["H"], rtol=0, atol=2e-5)
    gout = torch.randn(y.shape, generator=torch.Generator().manual_seed(1))
    (y * gout.to(cuda)).sum().backward()
    # float64 reference: the module's expressions with autograd through the loop
    ref = {k: v.double().clone().requires_grad_(v.is_floating_point()) for k, v in state.items()
           if k != "_cached_v"}
    v = state["_cached_v"].double().unsqueeze(-1)
    with torch.no_grad():
        W = ref["W_res"].detach()
        for _ in range(3):
            v = W @ v
            v = v / v.norm()
        radius = (W @ v).norm()
    Ws = ref["W_res"] * (torch.sigmoid(ref["log_rho"]) * 1.5 / radius)
    xd = torch.tensor(g["x"]).double().requires_grad_(True)
    U = xd @ ref["W_in.weight"].T
    Wz, Wr = ref["W_z.weight"], ref["W_r.weight"]
    Uz = U @ Wz[:, d:].T + ref["W_z.bias"]
    Ur = U @ Wr[:, d:].T + ref["W_r.bias"]
    H = esn_gru_torch(U, Uz, Ur, Wz[:, :d], Wr[:, :d], Ws)
    yr = H @ ref["readout.weight"].T
    (yr * gout.double()).sum().backward()
    _close(x.grad, xd.grad)
    params = dict(mod.named_parameters())
    for name in ("W_res", "log_rho", "W_in.weight", "W_z.weight", "W_z.bias", "W_r.weight",
                 "W_r.bias", "readout.weight"):
        _close(params[name].grad, ref[name].grad)


def test_leaky_reservoir_function_matches_autograd(cuda):
    # the recurrence's backward (inputs, scaled recurrent matrix, leak) against
    # float64 autograd of the reference loop on the same leaves
    from mk_iii_technologies_tsrn_b200.reservoir import LeakyReservoirFunction
    rng = np.random.default_rng(6)
    B, T, dr = 3, 40, 48
    U = torch.tensor(rng.standard_normal((B, T, dr)).astype(np.float32))
    Ws = torch.tensor((0.9 / np.sqrt(dr) * rng.standard_normal((dr, dr))).astype(np.float32))
    lk = torch.tensor([0.37])
    gout = torch.tensor(rng.standard_normal((B, T, dr)).astype(np.float32))
    u, w, l = (t.to(cuda).requires_grad_(True) for t in (U, Ws, lk))
    H = LeakyReservoirFunction.apply(u, w, l)
    (H * gout.to(cuda)).sum().backward()
    ud, wd, ld = (t.double().requires_grad_(True) for t in (U, Ws, lk))
    Hr = esn_leaky_torch(ud, wd, ld)
    (Hr * gout.double()).sum().backward()
    _close(H, Hr, rtol=1e-5, atol=2e-5)
    _close(u.grad, ud.grad)
    _close(w.grad, wd.grad)
    _close(l.grad, ld.grad)


def test_leaky_reservoir_module_training(cuda):
    # the module in training mode: output equals the reference module's
    # (golden); then a training step.  The spectral scale differentiates
    # through eigvals, as the reference does, which needs distinct eigenvalues:
    # the sparse initial matrix of the fixture has repeated zero eigenvalues
    # (its eigvals backward is singular in the reference module too), so the
    # step uses a dense recurrent matrix.
    from mk_iii_technologies_tsrn_b200.reservoir import LeakyEchoStateReservoir
    g = load_golden("esn_leaky")
    d = g["x"].shape[-1]
    mod = LeakyEchoStateReservoir(d, d).to(cuda).train()
    mod.load_state_dict({k[2:]: torch.tensor(v) for k, v in g.items() if k.startswith("p_")})
    x = torch.tensor(g["x"], device=cuda, requires_grad=True)
    with torch.no_grad():
        y = mod(x)
    np.testing.assert_allclose(y.cpu().numpy(), g["H"], rtol=0, atol=2e-5)
    with torch.no_grad():
        mod.W_res.copy_(torch.randn(d, d, generator=torch.Generator().manual_seed(7)) / d ** 0.5)
    y = mod(x)
    y.square().sum().backward()
    assert torch.isfinite(x.grad).all()
    for n, p in mod.named_parameters():
        assert p.grad is not None, n


def _unambiguous_case(B, H, T, dh, top_k):
    # inputs whose float64 scores have no near-tie at the top-k cut in any row
    for seed in range(50):
        gen = torch.Generator().manual_seed(seed)
        Q, K, V = (torch.randn(B, H, T, dh, generator=gen) for _ in range(3))
        slopes = 2.0 ** (-8.0 * torch.arange(1, H + 1, dtype=torch.float64) / H)
        S = torch.logsumexp(Q.double().unsqueeze(3) + K.double().unsqueeze(2), dim=-1)
        pos = torch.arange(T)
        S = S - slopes.view(-1, 1, 1) * (pos[:, None] - pos[None, :]).abs()
        S = S.masked_fill(pos[None, :] > pos[:, None], float("-inf"))
        srt = S.sort(dim=-1, descending=True).values
        gap = (srt[..., top_k - 1] - srt[..., top_k]).abs()
        if torch.nan_to_num(gap, nan=1.0, posinf=1.0).min() > 1e-3:
            return Q, K, V, slopes.float()
    raise RuntimeError("no unambiguous case")


@pytest.mark.parametrize("drop", [0.0, 1e-12])
def test_attention_core_gradients_match_autograd(cuda, drop):
    # drop > 0 runs the dense dropout path (with p = 1e-12 it keeps every weight)
    from mk_iii_technologies_tsrn_b200.tsrn_attention import TopKAttentionFunction
    B, H, T, dh, k = 2, 3, 40, 16, 5
    Q, K, V, slopes = _unambiguous_case(B, H, T, dh, k)
    q, kk, v = (t.to(cuda).requires_grad_(True) for t in (Q, K, V))
    out = TopKAttentionFunction.apply(q, kk, v, slopes.to(cuda), k, True, 0, drop)
    gout = torch.randn(out.shape, generator=torch.Generator().manual_seed(9))
    (out * gout.to(cuda)).sum().backward()
    qd, kd, vd = (t.double().requires_grad_(True) for t in (Q, K, V))
    ref = tsrn_attention_torch(qd, kd, vd, slopes.double(), k, True)
    (ref * gout.double()).sum().backward()
    _close(out, ref, rtol=1e-4, atol=2e-5)
    _close(q.grad, qd.grad)
    _close(kk.grad, kd.grad)
    _close(v.grad, vd.grad)


def test_attention_module_training_step(cuda):
    # the module in train mode (no dropout): output equals the inference path,
    # gradients reach every parameter
    from mk_iii_technologies_tsrn_b200.tsrn_attention import TropicalAttention
    torch.manual_seed(3)
    m = TropicalAttention(64, top_k=8, n_heads=4).to(cuda)
    x = torch.randn(2, 48, 64, device=cuda, requires_grad=True)
    m.train()
    y_train = m(x)
    y_train.sum().backward()
    assert x.grad is not None and torch.isfinite(x.grad).all()
    for n, p in m.named_parameters():
        assert p.grad is not None and torch.isfinite(p.grad).all(), n
    m.eval()
    with torch.no_grad():
        y_eval = m(x)
    torch.testing.assert_close(y_train.detach(), y_eval, rtol=1e-4, atol=2e-5)


def test_attention_prologue_matches_torch(cuda):
    # the fused QK-norm + RoPE + layout kernel against the same chain in PyTorch
    from mk_iii_technologies_tsrn_b200.tsrn_attention import TropicalAttention
    torch.manual_seed(5)
    for d, H in ((64, 4), (640, 8), (96, 2)):
        m = TropicalAttention(d, top_k=4, n_heads=H).to(cuda).eval()
        with torch.no_grad():
            m.q_norm.weight.uniform_(0.5, 1.5)
            m.k_norm.bias.uniform_(-0.3, 0.3)
            x = torch.randn(3, 37, d, device=cuda)
            got = m.project(x)
            ref = m._project_differentiable(x)
        for a, b in zip(got, ref):
            torch.testing.assert_close(a, b.contiguous(), rtol=2e-6, atol=2e-6)


@pytest.mark.parametrize("d,H,B,T", [(640, 8, 2, 50), (64, 4, 3, 33), (96, 2, 1, 129)])
def test_attention_prologue_backward_matches_autograd(cuda, d, H, B, T):
    # the fused prologue with its fused backward (PrologueFunction) against the
    # module's differentiable PyTorch chain: outputs and every gradient
    from mk_iii_technologies_tsrn_b200.tsrn_attention import TropicalAttention
    torch.manual_seed(7)
    m = TropicalAttention(d, top_k=4, n_heads=H).to(cuda)
    with torch.no_grad():
        for ln in (m.q_norm, m.k_norm):
            ln.weight.uniform_(0.5, 1.5)
            ln.bias.uniform_(-0.3, 0.3)
    x = torch.randn(B, T, d, device=cuda)
    g = [torch.randn(B, H, T, d // H, device=cuda) for _ in range(3)]
    results = []
    for fn in (m._project_train, m._project_differentiable):
        m.zero_grad(set_to_none=True)
        xr = x.clone().requires_grad_(True)
        outs = fn(xr)
        sum((o * gg).sum() for o, gg in zip(outs, g)).backward()
        grads = [xr.grad] + [p.grad for p in (m.Wq.weight, m.Wk.weight, m.Wv.weight,
                                             m.q_norm.weight, m.q_norm.bias,
                                             m.k_norm.weight, m.k_norm.bias)]
        results.append(([o.detach() for o in outs], grads))
    (o1, g1), (o2, g2) = results
    for a, b in zip(o1, o2):
        torch.testing.assert_close(a, b, rtol=1e-5, atol=2e-6)
    for a, b in zip(g1, g2):
        _close(a, b.double().cpu(), rtol=1e-4, atol=1e-5)


def test_attention_prologue_backward_repeats(cuda):
    from mk_iii_technologies_tsrn_b200 import ops
    g = torch.Generator(device=cuda).manual_seed(3)
    B, T, H, dh = 2, 70, 4, 80
    qkv = torch.randn(B * T, 3 * H * dh, device=cuda, generator=g)
    qg, kg = (torch.rand(dh, device=cuda, generator=g) + 0.5 for _ in range(2))
    ang = torch.outer(torch.arange(T, dtype=torch.float32),
                      torch.rand(dh // 2, generator=torch.Generator().manual_seed(1)))
    cos, sin = ang.cos().to(cuda), ang.sin().to(cuda)
    dQ, dK, dV = (torch.randn(B, H, T, dh, device=cuda, generator=g) for _ in range(3))
    a = ops.tsrn_attention_prologue_bwd(qkv, B, T, H, dh, qg, kg, 1e-5, cos, sin, dQ, dK, dV)
    b = ops.tsrn_attention_prologue_bwd(qkv, B, T, H, dh, qg, kg, 1e-5, cos, sin, dQ, dK, dV)
    for x, y in zip(a, b):
        assert torch.equal(x, y)


@pytest.mark.parametrize("rows,D", [(3000, 640), (517, 128), (64, 1024), (1, 384)])
def test_layer_norm_backward_matches_autograd(cuda, rows, D):
    # the pre-norms of the block's branches (research/tsrn_dml.py:1096-1106)
    # with this library's backward, against float64 autograd
    from mk_iii_technologies_tsrn_b200 import ops
    gen = torch.Generator().manual_seed(rows + D)
    x = torch.randn(rows, D, generator=gen) * 3.0 + 1.5
    w = torch.randn(D, generator=gen)
    b = torch.randn(D, generator=gen)
    gy = torch.randn(rows, D, generator=gen)
    xs, ws, bs = (t.to(cuda).requires_grad_(True) for t in (x, w, b))
    y = ops.layer_norm(xs, ws, bs, 1e-5)
    assert "LayerNormFunction" in type(y.grad_fn).__name__
    (y * gy.to(cuda)).sum().backward()
    xd, wd, bd = (t.double().requires_grad_(True) for t in (x, w, b))
    yd = torch.nn.functional.layer_norm(xd, (D,), wd, bd, 1e-5)
    (yd * gy.double()).sum().backward()
    _close(y, yd, rtol=1e-5, atol=1e-6)
    _close(xs.grad, xd.grad, rtol=1e-4, atol=1e-6)
    _close(ws.grad, wd.grad, rtol=1e-4, atol=1e-6)
    _close(bs.grad, bd.grad, rtol=1e-4, atol=1e-6)


def test_layer_norm_backward_repeats_and_edges(cuda):
    from mk_iii_technologies_tsrn_b200 import ops
    gen = torch.Generator(device=cuda).manual_seed(5)
    x = torch.randn(4099, 640, device=cuda, generator=gen)
    dy = torch.randn(4099, 640, device=cuda, generator=gen)
    w = torch.randn(640, device=cuda, generator=gen)
    first = ops.layer_norm_bwd(x, dy, w, 1e-5)
    second = ops.layer_norm_bwd(x, dy, w, 1e-5)
    for a, b in zip(first, second):
        assert torch.equal(a, b)
    # no weight: gamma = 1 (dx equals the weighted form at w = 1)
    ones = torch.ones(640, device=cuda)
    for a, b in zip(ops.layer_norm_bwd(x, dy, None, 1e-5), ops.layer_norm_bwd(x, dy, ones, 1e-5)):
        assert torch.equal(a, b)
    # no rows: zero parameter gradients
    dx, dw, db = ops.layer_norm_bwd(x[:0], dy[:0], w, 1e-5)
    assert dx.shape == (0, 640) and not dw.any() and not db.any()
    # unsupported width: PyTorch's own backward through ops.layer_norm
    xs = torch.randn(10, 100, device=cuda, requires_grad=True)
    y = ops.layer_norm(xs, None, None)
    assert "LayerNormFunction" not in type(y.grad_fn).__name__
    with pytest.raises(ValueError):
        ops.layer_norm_bwd(xs.detach(), xs.detach(), None, 1e-5)
