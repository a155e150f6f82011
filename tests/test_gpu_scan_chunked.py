"""Chunk-parallel tropical scan (tp_scan_fwd_chunked / tp_scan_bwd_chunked) vs
the sequential recurrence (oracle.scan: research/tsrn_dml.py:906-916,961-972).

Forward h and win mask: bit-exact, for every chunk length, with tails, h0,
special values (NaN / +-inf inputs, a = +-0, tiny and -inf decays) and exact
ties at zero.  Backward: gu and gh0 bit-exact; ga within the rounding of its
different summation order (per-chunk partials) against the fp64 oracle.
"""
import numpy as np
import pytest
import torch

from oracle import scan as oscan

pytestmark = pytest.mark.gpu


def _ops():
    from mk_iii_technologies_tsrn_b200 import ops
    return ops


def _inputs(B, T, C, seed):
    rng = np.random.default_rng(seed)
    a = -rng.random(C).astype(np.float32)
    b = (0.1 * rng.standard_normal((B, T, C))).astype(np.float32)
    x = rng.standard_normal((B, T, C)).astype(np.float32)
    return a, b, x


def _fwd(ops, b, x, a, h_init, h0=None, chunk=0, mode="chunked"):
    dev = torch.device("cuda:0")
    h, mask = ops.scan_forward(torch.tensor(b, device=dev),
                               torch.tensor(x, device=dev) if x is not None else None,
                               torch.tensor(a, device=dev), h_init,
                               torch.tensor(h0, device=dev) if h0 is not None else None,
                               need_mask=True, mode=mode, chunk=chunk)
    return h.cpu().numpy(), mask.cpu().numpy().view(np.uint32)


SHAPES = [(2, 1024, 64, 32), (1, 300, 96, 64), (3, 257, 40, 32), (2, 200, 33, 32),
          (1, 31, 8, 32), (2, 640, 128, 128), (1, 4096, 12, 0)]


@pytest.mark.parametrize("B,T,C,chunk", SHAPES)
@pytest.mark.parametrize("h_init", [float("-inf"), 0.0])
def test_forward_bit_exact(cuda, B, T, C, chunk, h_init):
    a, b, x = _inputs(B, T, C, seed=B * 1000 + T + C)
    ops = _ops()
    h, mask = _fwd(ops, b, x, a, h_init, chunk=chunk)
    rh, win = oscan.scan_fwd((b + x).astype(np.float32), a, h_init)
    np.testing.assert_array_equal(h, rh)
    np.testing.assert_array_equal(mask, oscan.win_mask_words(win))


def test_forward_h0_no_x_and_slow_decay(cuda):
    # tiny decays: the carry wins across whole chunks, so the exact chain of
    # rounded adds decides the chunk states
    B, T, C = 2, 2048, 64
    rng = np.random.default_rng(3)
    a = -(10.0 ** rng.uniform(-7, 0, C)).astype(np.float32)
    a[:4] = 0.0
    a[4:8] = -0.0
    u = rng.standard_normal((B, T, C)).astype(np.float32)
    h0 = (3 * rng.standard_normal((B, C))).astype(np.float32)
    ops = _ops()
    for chunk in (32, 64, 256):
        h, mask = _fwd(ops, u, None, a, 0.0, h0=h0, chunk=chunk)
        rh, win = oscan.scan_fwd(u, a, 0.0, h0)
        np.testing.assert_array_equal(h, rh)
        np.testing.assert_array_equal(mask, oscan.win_mask_words(win))


def test_forward_special_values(cuda):
    B, T, C = 2, 512, 16
    rng = np.random.default_rng(5)
    u = rng.standard_normal((B, T, C)).astype(np.float32)
    a = -rng.random(C).astype(np.float32)
    u[0, 100, 0] = np.nan
    u[0, 37, 1] = np.inf
    u[1, 200:260, 2] = -np.inf
    u[:, :, 3] = -np.inf                     # a channel with no finite input
    u[1, 300, 4] = np.inf
    a[4] = -np.inf                           # -inf decay after an inf input: NaN
    a[5] = 0.0
    u[:, :, 5] = np.where(rng.random((B, T)) < 0.5, 0.0, -1.0)   # exact zero ties
    u[:, :, 6] = -0.0
    a[6] = -0.0
    u[:, :, 7] = 0.0
    a[7] = 0.0
    a[8] = np.inf                            # -inf + inf is NaN, finite + inf stays +inf
    u[0, :, 8] = -np.inf                     # no finite input before t = 40 in row 0
    u[0, 40:, 8] = rng.standard_normal(T - 40)
    ops = _ops()
    for h_init in (0.0, -0.0, float("-inf")):
        for chunk in (32, 64, 96):
            h, mask = _fwd(ops, u, None, a, h_init, chunk=chunk)
            rh, win = oscan.scan_fwd(u, a, h_init)
            np.testing.assert_array_equal(h.view(np.uint32)[~np.isnan(rh)],
                                          rh.view(np.uint32)[~np.isnan(rh)])
            np.testing.assert_array_equal(np.isnan(h), np.isnan(rh))
            np.testing.assert_array_equal(mask, oscan.win_mask_words(win))


def test_forward_matches_sequential_kernel_at_config3_b2(cuda):
    # config 3's per-GPU share at 8 GPUs: B=2, T=4096, C=1024
    B, T, C = 2, 4096, 1024
    gen = torch.Generator(device=cuda).manual_seed(0)
    a = -torch.rand(C, device=cuda, generator=gen)
    b = 0.1 * torch.randn(B, T, C, device=cuda, generator=gen)
    x = torch.randn(B, T, C, device=cuda, generator=gen)
    ops = _ops()
    assert ops.scan_mode(B, T, C) == "chunked"
    h1, m1 = ops.scan_forward(b, x, a, float("-inf"), need_mask=True, mode="chunked")
    h2, m2 = ops.scan_forward(b, x, a, float("-inf"), need_mask=True, mode="sequential")
    assert torch.equal(h1, h2) and torch.equal(m1, m2)
    rh, win = oscan.scan_fwd((b + x).cpu().numpy(), a.cpu().numpy(), -np.inf)
    np.testing.assert_array_equal(h1.cpu().numpy(), rh)
    g = torch.randn(B, T, C, device=cuda, generator=gen)
    gu1, ga1, gh1 = ops.scan_backward(g, a, float("-inf"), b=b, x=x, h=h1, need_gh0=True,
                                      mode="chunked")
    gu2, ga2, gh2 = ops.scan_backward(g, a, float("-inf"), b=b, x=x, h=h1, need_gh0=True,
                                      mode="sequential")
    assert torch.equal(gu1, gu2) and torch.equal(gh1, gh2)
    _ga_close(ga1.cpu().numpy(), g.cpu().numpy(), win)


def _ga_close(ga, gh, win):
    # the fp64 oracle, and the rounding bound of an fp32 sum of the lost gradients
    _, ga64, _ = oscan.scan_bwd(gh, win, dtype=np.float64)
    _, gabs, _ = oscan.scan_bwd(np.abs(gh), win, dtype=np.float64)   # bounds sum |lost|
    n = gh.shape[0] * gh.shape[1]
    tol = 4 * n * np.finfo(np.float32).eps * gabs + 1e-6
    assert np.all(np.abs(ga - ga64) <= tol), float(np.max(np.abs(ga - ga64) / tol))


@pytest.mark.parametrize("B,T,C,chunk", [(2, 1024, 64, 32), (1, 300, 96, 64), (3, 257, 40, 32),
                                         (2, 200, 33, 32), (1, 45, 8, 32)])
@pytest.mark.parametrize("use_mask", [True, False])
def test_backward_exact(cuda, B, T, C, chunk, use_mask):
    a, b, x = _inputs(B, T, C, seed=B + T + C)
    a[::7] = -1e-4                                     # slow channels: chunks with no winner
    h0 = np.random.default_rng(3).standard_normal((B, C)).astype(np.float32)
    gh = np.random.default_rng(4).standard_normal((B, T, C)).astype(np.float32)
    ops = _ops()
    bt, xt, at = (torch.tensor(v, device=cuda) for v in (b, x, a))
    h0t = torch.tensor(h0, device=cuda)
    h, mask = ops.scan_forward(bt, xt, at, 0.0, h0t, need_mask=True, mode="chunked",
                               chunk=chunk)
    kw = dict(mask=mask) if use_mask else dict(b=bt, x=xt, h=h)
    gu, ga, gh0 = ops.scan_backward(torch.tensor(gh, device=cuda), at, 0.0, h0t,
                                    need_ga=True, need_gh0=True, mode="chunked", chunk=chunk,
                                    **kw)
    _, win = oscan.scan_fwd((b + x).astype(np.float32), a, 0.0, h0)
    rgu, rga, rgh0 = oscan.scan_bwd(gh, win, dtype=np.float32)
    np.testing.assert_array_equal(gu.cpu().numpy(), rgu)
    np.testing.assert_array_equal(gh0.cpu().numpy(), rgh0)
    _ga_close(ga.cpu().numpy(), gh, win)


def test_workspace_and_arguments(cuda):
    import ctypes
    from mk_iii_technologies_tsrn_b200 import _lib
    lib = _lib.load()
    B, T, C = 2, 256, 64
    b = torch.randn(B, T, C, device=cuda)
    a = -torch.rand(C, device=cuda)
    h = torch.empty_like(b)
    need = lib.tp_scan_chunked_workspace_bytes(B, T, C, 32)
    assert need > 0 and lib.tp_scan_chunked_workspace_bytes(B, T, C, 33) == -1
    ws = torch.empty(need, device=cuda, dtype=torch.uint8)
    p = lambda t: ctypes.c_void_p(t.data_ptr())   # noqa: E731
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    # too small a workspace, a chunk length that is not a multiple of 32
    assert lib.tp_scan_fwd_chunked(B, T, C, p(b), None, p(a), 0.0, None, p(h), None, 32, p(ws),
                                   need - 1, stream) == -7
    assert lib.tp_scan_fwd_chunked(B, T, C, p(b), None, p(a), 0.0, None, p(h), None, 48, p(ws),
                                   need, stream) == -1
    assert lib.tp_scan_fwd_chunked(B, T, C, p(b), None, p(a), 0.0, None, p(h), None, 32, p(ws),
                                   need, stream) == 0
    torch.cuda.synchronize()
    rh, _ = oscan.scan_fwd(b.cpu().numpy(), a.cpu().numpy(), 0.0)
    np.testing.assert_array_equal(h.cpu().numpy(), rh)


def test_forward_carry_chains_at_binade_edges(cuda):
    # inputs that never win (the carry decides every chunk), decays that are
    # exact half-ulps (ties), fractions of an ulp, and starts just above and
    # below binade boundaries of both signs: the chunk states come from the
    # one-step chain (inside a binade) or the step-by-step adds (ties,
    # crossings), and must equal the recurrence bit for bit either way
    B, T = 2, 2048
    a = np.array([-2.0 ** -24, -3 * 2.0 ** -24, -2.0 ** -25, -1e-7, -0.49e-7, 0.0, -1.0,
                  -2.0 ** -23, 2.0 ** -24, 3e-8, -7.3e-6, -2.0 ** -20], np.float32)
    C = a.size
    u = np.full((B, T, C), -np.inf, np.float32)
    u[1, 700, 3] = 0.5                       # one late winner
    h0 = np.array([[1.0000001, 2.0 - 2.0 ** -22, 1.5, -1.5, 1e-30, 3.0e38,
                    1.0, 1.0 + 2.0 ** -22, -2.0 + 2.0 ** -22, 0.75, 1024.0, -0.1],
                   [2.0 ** -126, -2.0 ** -126, 4.0, 4.0 - 2.0 ** -21, -1.0, 8.0,
                    0.3, 1.0 - 2.0 ** -24, 5.0, -5.0, 1e-3, 1.0]], np.float32)
    ops = _ops()
    for chunk in (32, 64, 256):
        h, mask = _fwd(ops, u, None, a, 0.0, h0=h0, chunk=chunk)
        rh, win = oscan.scan_fwd(u, a, 0.0, h0)
        np.testing.assert_array_equal(h.view(np.uint32), rh.view(np.uint32))
        np.testing.assert_array_equal(mask, oscan.win_mask_words(win))


def test_forward_scan_over_many_chunks(cuda):
    # the chunks' starting states come from a parallel scan over the chunks of
    # each (b, c) lane, 128 chunks per tile: 313 / 625 / 157 chunks (several
    # tiles, a partial last chunk and warp), slow channels whose carry
    # survives many chunks in a row, C not a multiple of 4 (one channel per
    # thread); bit-exact with the recurrence, also when called again
    B, T, C = 2, 20000, 130
    rng = np.random.default_rng(11)
    a = -rng.random(C).astype(np.float32)
    a[::5] = -(10.0 ** rng.uniform(-7, -3, a[::5].size)).astype(np.float32)
    u = rng.standard_normal((B, T, C)).astype(np.float32)
    h0 = rng.standard_normal((B, C)).astype(np.float32)
    rh, win = oscan.scan_fwd(u, a, 0.0, h0)
    words = oscan.win_mask_words(win)
    ops = _ops()
    for chunk in (64, 32, 64, 128):
        h, mask = _fwd(ops, u, None, a, 0.0, h0=h0, chunk=chunk)
        np.testing.assert_array_equal(h.view(np.uint32), rh.view(np.uint32))
        np.testing.assert_array_equal(mask, words)
    ops.check_device_error()
