"""Stream-K schedules of the large fp32 forward (TMA kernel): tiles shared by
CTAs (an even split of chunks, mode 2; or tiles cut into 2 or 4 k-aligned
pieces, mode 3, the argmax kernel's choice in auto mode) are merged exactly, so
values and argmax equal the whole-tile schedule bit for bit (and the oracle on
sampled rows).  Shapes have at least as many 128x128 tiles as SMs; K values
give odd k-tile counts and K tails."""
import numpy as np
import pytest
import torch

import oracle

pytestmark = pytest.mark.gpu


@pytest.fixture
def lib(cuda):
    from mk_iii_technologies_tsrn_b200 import _lib
    lib = _lib.load()
    old_terms = lib.tp_set_argmax_tma_min_terms(0)     # TMA kernel for every eligible shape
    old_sk = lib.tp_set_stream_k(1)
    yield lib
    lib.tp_set_stream_k(old_sk)
    lib.tp_set_argmax_tma_min_terms(old_terms)


def _inputs(M, N, K, kind, seed):
    rng = np.random.default_rng(seed)
    if kind == "int":                      # exact ties everywhere, also across split points
        x = rng.integers(-3, 4, (M, K)).astype(np.float32)
        w = rng.integers(-3, 4, (N, K)).astype(np.float32)
    else:
        x = rng.standard_normal((M, K)).astype(np.float32)
        w = rng.standard_normal((N, K)).astype(np.float32)
        w[rng.random((N, K)) < 0.05] = -np.inf
        if kind == "special":
            x[5, 7] = np.nan
            x[9, :] = -np.inf
            w[3, K - 1] = np.nan
            w[11, :K // 2] = np.inf
            x[100, K // 3] = np.inf
            w[200, K // 3] = -np.inf           # inf + -inf = NaN in one term
    return x, w


def _fwd(lib, mode, x, w, bias=None, argmax=True):
    from mk_iii_technologies_tsrn_b200 import ops
    lib.tp_set_stream_k(mode)
    y, am = ops.maxplus(x, w, bias, argmax=argmax)
    torch.cuda.synchronize()
    return y.cpu().numpy(), (am.cpu().numpy() if am is not None else None)


@pytest.mark.parametrize("M,N,K,kind", [
    (2048, 1280, 300, "normal"),     # 160 tiles, 10 k-tiles (5 chunks)
    (1536, 1664, 1100, "normal"),    # 156 tiles, 35 k-tiles: last chunk one k-tile, K tail
    (2048, 1280, 256, "int"),
    (1280, 2048, 520, "special"),
    (2048, 2560, 300, "normal"),     # 320 tiles: one whole-tile wave, then stream-K over 172
    (2560, 2048, 160, "int"),        # the same with exact ties, 5 k-tiles
    # k-aligned pieces (mode 3): 16 / 32 k-tiles -> 4 pieces of 160 tiles,
    # 12 k-tiles -> 2 pieces of the 172 remaining tiles, K tail in the last piece
    (2048, 1280, 512, "normal"),
    (1280, 2048, 1024, "special"),
    (2560, 2048, 384, "int"),
    (2048, 1280, 1000, "normal"),
])
def test_stream_k_equals_whole_tiles(lib, cuda, M, N, K, kind):
    x, w = _inputs(M, N, K, kind, seed=M + N + K)
    xt, wt = torch.tensor(x, device=cuda), torch.tensor(w, device=cuda)
    y0, a0 = _fwd(lib, 0, xt, wt)
    for mode in (2, 3, 1):
        ym, am = _fwd(lib, mode, xt, wt)
        np.testing.assert_array_equal(ym.view(np.uint32), y0.view(np.uint32), err_msg=str(mode))
        np.testing.assert_array_equal(am, a0, err_msg=str(mode))
    y3, a3 = _fwd(lib, 3, xt, wt)
    rows = [0, 5, 9, 100, M // 2, M - 1]
    ry, ri = oracle.maxplus_fwd(x[rows], w)
    # against the oracle: NaN is NaN whatever its payload (the GPU's is canonical)
    np.testing.assert_array_equal(y3[rows], ry)
    np.testing.assert_array_equal(a3[rows], ri)


def test_stream_k_value_only_bias_scale(lib, cuda):
    from mk_iii_technologies_tsrn_b200 import ops
    M, N, K = 2048, 1280, 700
    x, w = _inputs(M, N, K, "normal", seed=3)
    b = np.random.default_rng(4).standard_normal(N).astype(np.float32)
    xt, wt, bt = (torch.tensor(a, device=cuda) for a in (x, w, b))
    outs = []
    for mode in (0, 2):
        lib.tp_set_stream_k(mode)
        y, _ = ops.maxplus_strided(xt, wt, bt, argmax=False, scale=0.5)
        outs.append(y.cpu().numpy())
    np.testing.assert_array_equal(outs[1].view(np.uint32), outs[0].view(np.uint32))
    ry, _ = oracle.maxplus_fwd(x[:3], w)
    np.testing.assert_array_equal(outs[1][:3], ((ry + b) * np.float32(0.5)).astype(np.float32))


@pytest.mark.parametrize("mode", ["primal", "blend"])
def test_stream_k_lfdual_epilogue(lib, cuda, mode):
    from mk_iii_technologies_tsrn_b200 import ops
    M, N, K = 2048, 1280, 256
    rng = np.random.default_rng(6)
    x, w = _inputs(M, N, K, "normal", seed=5)
    t = lambda a: torch.tensor(a, device=cuda)
    b = rng.standard_normal(N).astype(np.float32)
    s = np.sort(rng.standard_normal(8)).astype(np.float32)
    pb = rng.standard_normal(8).astype(np.float32)
    xg = np.linspace(-3, 3, 8).astype(np.float32)
    gate = torch.sigmoid(t(rng.standard_normal(N).astype(np.float32))) if mode == "blend" else None
    outs = []
    for m in (0, 2):
        lib.tp_set_stream_k(m)
        outs.append(ops.maxplus_lfdual(t(x), t(w), t(b), mode, t(s), t(pb), t(xg), gate)
                    .cpu().numpy())
    np.testing.assert_array_equal(outs[1].view(np.uint32), outs[0].view(np.uint32))


def test_stream_k_shard_shape(lib, cuda):
    # the per-rank shape of the 8-GPU column-sharded 8192^3 GEMM: 512 tiles for
    # 148 SMs (3.46 waves), where the schedule matters most
    M, N, K = 8192, 1024, 8192
    g = torch.Generator(device=cuda).manual_seed(0)
    x = torch.randn(M, K, device=cuda, generator=g)
    w = torch.randn(N, K, device=cuda, generator=g)
    w[torch.rand(N, K, device=cuda, generator=g) < 0.05] = float("-inf")
    from mk_iii_technologies_tsrn_b200 import ops
    res = {}
    for mode in (0, 2, 3):
        lib.tp_set_stream_k(mode)
        y, am = ops.maxplus(x, w)
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(3):
            ops.maxplus(x, w)
        e1.record()
        torch.cuda.synchronize()
        res[mode] = (y, am, e0.elapsed_time(e1) / 3)
    for mode in (2, 3):
        assert torch.equal(res[0][0].view(torch.int32), res[mode][0].view(torch.int32))
        assert torch.equal(res[0][1], res[mode][1])
    print(f"\n8192x1024x8192: whole tiles {res[0][2]:.2f} ms, even split {res[2][2]:.2f} ms, "
          f"k-aligned pieces {res[3][2]:.2f} ms")
    ry, ri = oracle.maxplus_fwd(x[:2].cpu().numpy(), w[:300].cpu().numpy())
    np.testing.assert_array_equal(res[2][0][:2, :300].cpu().numpy(), ry)
    np.testing.assert_array_equal(res[2][1][:2, :300].cpu().numpy(), ri)
