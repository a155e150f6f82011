"""Tensor-core (tcgen05, 3xTF32) TSRN attention kernel vs the oracle and vs the
CUDA-core kernel (research/tsrn_dml.py:438-460, 509-524).

Both kernels are run explicitly through ``ops.set_attention_path``.  Scores
agree with the fp64 oracle within ~1e-6; rows whose top_k-th and next scores
are closer than 1e-4 may select differently and are excluded (as in the
CUDA-core kernel's tests).  Exactly tied scores (equal keys, no ALiBi) must
keep every tied key, including rows with more kept keys than the kernel
lists in shared memory.
"""
import numpy as np
import pytest
import torch

import oracle
from test_oracle_golden import _ambiguous_rows

pytestmark = pytest.mark.gpu


def _ops():
    from mk_iii_technologies_tsrn_b200 import ops
    return ops


@pytest.fixture
def path():
    ops = _ops()
    prev = ops.set_attention_path("auto")
    yield ops.set_attention_path
    ops.set_attention_path(prev)


def _case(B, H, T, Tc, dh, seed, scale=1.0):
    rng = np.random.default_rng(seed)
    Tkv = T + Tc
    Q = (rng.standard_normal((B, H, T, dh)) * scale).astype(np.float32)
    K = (rng.standard_normal((B, H, Tkv, dh)) * scale).astype(np.float32)
    V = rng.standard_normal((B, H, Tkv, dh)).astype(np.float32)
    slopes = (2.0 ** (-8.0 / H * (np.arange(H) + 1))).astype(np.float32)
    return Q, K, V, slopes


def _run(cuda, Q, K, V, slopes, top_k, causal, Tc):
    return _ops().tsrn_attention(*(torch.tensor(a, device=cuda) for a in (Q, K, V, slopes)),
                                 top_k=top_k, causal=causal, Tc=Tc).cpu().numpy()


@pytest.mark.parametrize("B,H,T,Tc,dh,top_k,causal", [
    (2, 4, 64, 0, 16, 8, True),
    (1, 2, 200, 0, 40, 16, True),     # T not a multiple of the 128-row tile
    (2, 3, 97, 0, 24, 5, False),      # non-causal; Tkv not a multiple of the 64-key tile
    (1, 2, 120, 40, 32, 8, True),     # cross-window cached keys (Tc > 0)
    (1, 1, 50, 0, 80, 16, True),      # top_k larger than the early rows' key count
    (1, 2, 130, 0, 20, 4, True),      # dh not a multiple of 8 (zero-padded channels)
    (1, 1, 64, 0, 96, 16, False),     # dh at the tensor-core kernel's limit
    (1, 4, 260, 0, 80, 16, True),     # config 5's head size, several tiles per slice
])
def test_tensor_cores_vs_oracle(cuda, path, B, H, T, Tc, dh, top_k, causal):
    Q, K, V, slopes = _case(B, H, T, Tc, dh, seed=B * 1000 + T + dh)
    path("tensor_cores")
    out = _run(cuda, Q, K, V, slopes, top_k, causal, Tc)
    ref, S = oracle.tsrn_attention_fwd(Q, K, V, slopes, top_k, causal, Tc)
    ok = ~_ambiguous_rows(S, top_k)
    assert ok.mean() > 0.9
    np.testing.assert_allclose(out[ok], ref[ok], rtol=1e-4, atol=2e-5)
    # the CUDA-core kernel on the same inputs
    path("cuda_cores")
    out_cc = _run(cuda, Q, K, V, slopes, top_k, causal, Tc)
    np.testing.assert_allclose(out[ok], out_cc[ok], rtol=1e-4, atol=2e-5)


def test_long_cached_keys_beyond_the_cuda_core_limit(cuda, path):
    # Tkv = 6228 keys: more than the CUDA-core kernel holds in shared memory
    B, H, T, Tc, dh, top_k = 1, 1, 128, 6100, 32, 8
    Q, K, V, slopes = _case(B, H, T, Tc, dh, seed=21)
    path("tensor_cores")
    out = _run(cuda, Q, K, V, slopes, top_k, True, Tc)
    ref, S = oracle.tsrn_attention_fwd(Q, K, V, slopes, top_k, True, Tc)
    ok = ~_ambiguous_rows(S, top_k)
    np.testing.assert_allclose(out[ok], ref[ok], rtol=1e-4, atol=2e-5)
    path("cuda_cores")
    with pytest.raises(RuntimeError):
        _run(cuda, Q, K, V, slopes, top_k, True, Tc)
    path("auto")                         # beyond the CUDA-core limit auto takes tensor cores
    np.testing.assert_array_equal(_run(cuda, Q, K, V, slopes, top_k, True, Tc), out)


@pytest.mark.parametrize("causal", [True, False])
@pytest.mark.parametrize("T", [60, 100])
def test_exact_ties_keep_every_tied_key(cuda, path, causal, T):
    # equal keys and no ALiBi: every score of a row ties, so every visible key
    # is kept (in the tensor-core kernel, rows with more than 16 kept keys in
    # either half of the key columns overflow the shared-memory lists and
    # accumulate those V rows in scratch rows; at T = 100 a half's 50 tied
    # candidates also overflow the pass-1 log, so the kernel runs pass 2)
    B, H, dh, top_k = 1, 2, 32, 8
    rng = np.random.default_rng(4)
    Q = rng.standard_normal((B, H, T, dh)).astype(np.float32)
    K = np.repeat(rng.standard_normal((B, H, 1, dh)).astype(np.float32), T, axis=2)
    V = rng.standard_normal((B, H, T, dh)).astype(np.float32)
    slopes = np.zeros(H, np.float32)
    ref, _ = oracle.tsrn_attention_fwd(Q, K, V, slopes, top_k, causal)
    for p in ("tensor_cores", "cuda_cores"):
        path(p)
        out = _run(cuda, Q, K, V, slopes, top_k, causal, 0)
        np.testing.assert_allclose(out, ref, rtol=1e-4, atol=2e-5, err_msg=p)


def test_large_dynamic_range_exact_fallback(cuda, path):
    # scale 8: some exp-feature dots fall below 1e-30 and are recomputed exactly
    Q, K, V, slopes = _case(1, 2, 96, 0, 32, seed=5, scale=8.0)
    path("tensor_cores")
    out = _run(cuda, Q, K, V, slopes, 8, True, 0)
    ref, S = oracle.tsrn_attention_fwd(Q, K, V, slopes, 8)
    ok = ~_ambiguous_rows(S, 8, gap=1e-3)
    np.testing.assert_allclose(out[ok], ref[ok], rtol=1e-4, atol=5e-5)


def test_special_values(cuda, path):
    # a NaN query row gives NaN output in both kernels; +-inf-free rows unaffected
    Q, K, V, slopes = _case(1, 2, 70, 0, 16, seed=8)
    Q[0, 1, 33, 5] = np.nan
    outs = {}
    for p in ("tensor_cores", "cuda_cores"):
        path(p)
        outs[p] = _run(cuda, Q, K, V, slopes, 8, True, 0)
    a, b = outs["tensor_cores"], outs["cuda_cores"]
    np.testing.assert_array_equal(np.isnan(a), np.isnan(b))
    assert np.isnan(a[0, 1, 33]).all()
    fin = ~np.isnan(b)
    ref, S = oracle.tsrn_attention_fwd(Q, K, V, slopes, 8)
    ok = ~_ambiguous_rows(np.nan_to_num(S, nan=0.0), 8)
    sel = ok[..., None] & fin
    np.testing.assert_allclose(a[sel], b[sel], rtol=1e-4, atol=2e-5)


def test_path_selection(cuda, path):
    ops = _ops()
    Q, K, V, slopes = _case(1, 1, 40, 0, 128, seed=1)
    path("tensor_cores")                 # dh = 128: not supported on tensor cores
    with pytest.raises(RuntimeError):
        _run(cuda, Q, K, V, slopes, 4, True, 0)
    path("auto")                         # auto falls back to the CUDA-core kernel
    out = _run(cuda, Q, K, V, slopes, 4, True, 0)
    ref, S = oracle.tsrn_attention_fwd(Q, K, V, slopes, 4)
    ok = ~_ambiguous_rows(S, 4)
    np.testing.assert_allclose(out[ok], ref[ok], rtol=1e-4, atol=2e-5)
    with pytest.raises(ValueError):
        ops.set_attention_path("fast")


@pytest.mark.parametrize("T,expect", [(200, "tensor_cores"), (100, "cuda_cores")])
def test_auto_choice(cuda, path, T, expect):
    # auto takes tensor cores when T fills a 128-query tile, CUDA cores below
    Q, K, V, slopes = _case(1, 2, T, 0, 32, seed=T)
    outs = {}
    for p in ("auto", "tensor_cores", "cuda_cores"):
        path(p)
        outs[p] = _run(cuda, Q, K, V, slopes, 8, True, 0)
    np.testing.assert_array_equal(outs["auto"], outs[expect])
