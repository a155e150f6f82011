"""``chain_exact`` (csrc/chain_exact.cuh) built for the host and compared, bit
for bit, with n step-by-step float32 additions in numpy.

The chunk-parallel scan carries a surviving state through whole chunks with it
(the recurrence h_t = fl(a + h_{t-1}) while no input wins,
research/tsrn_dml.py:906-916), so it must reproduce every rounding: random
decays and starts, addends of exactly half an ulp and other fractions at
binade edges (ties to even), chains that cross zero, growth, zeros,
subnormals, overflow, infinities and NaN."""
import ctypes
import os
import shutil
import subprocess

import numpy as np
import pytest

CSRC = os.path.join(os.path.dirname(__file__), "..", "mk_iii_technologies_tsrn_b200", "csrc")
HARNESS = r"""
#include "chain_exact.cuh"
extern "C" void chain_many(int64_t count, const float* x, const float* a, const int64_t* n,
                           float* out) {
  for (int64_t i = 0; i < count; ++i) out[i] = tp::chain_exact(x[i], a[i], n[i]);
}
"""


@pytest.fixture(scope="module")
def chain(tmp_path_factory):
    cxx = shutil.which("g++") or shutil.which("c++")
    if cxx is None:
        pytest.skip("no C++ compiler")
    d = tmp_path_factory.mktemp("chain")
    src, lib = d / "harness.cpp", d / "libchain.so"
    src.write_text(HARNESS)
    subprocess.run([cxx, "-O2", "-std=c++17", "-shared", "-fPIC", "-ffp-contract=off",
                    "-I", CSRC, str(src), "-o", str(lib)], check=True)
    so = ctypes.CDLL(str(lib))

    def run(x, a, n):
        x, a = np.ascontiguousarray(x, np.float32), np.ascontiguousarray(a, np.float32)
        n = np.ascontiguousarray(n, np.int64)
        out = np.empty_like(x)
        ptr = lambda t: t.ctypes.data_as(ctypes.c_void_p)   # noqa: E731
        so.chain_many(ctypes.c_int64(x.size), ptr(x), ptr(a), ptr(n), ptr(out))
        return out
    return run


def _steps(x, a, n):
    y = x.astype(np.float32).copy()
    a = a.astype(np.float32)
    with np.errstate(all="ignore"):
        for i in range(int(n.max(initial=0))):
            m = n > i
            y[m] = y[m] + a[m]
    return y


def _check(chain, x, a, n):
    got, ref = chain(x, a, n), _steps(x, a, n)
    same = (got.view(np.uint32) == ref.view(np.uint32)) | (np.isnan(got) & np.isnan(ref))
    bad = np.flatnonzero(~same)[:5]
    assert bad.size == 0, [(x[k], a[k], n[k], got[k], ref[k]) for k in bad]


def test_random_decays(chain):
    rng = np.random.default_rng(0)
    N = 30000
    x = (rng.standard_normal(N) * 10.0 ** rng.uniform(-3, 3, N)).astype(np.float32)
    sign = rng.choice([1.0, -1.0], N, p=[0.8, 0.2])
    a = (-(10.0 ** rng.uniform(-9, 0, N)) * sign).astype(np.float32)
    _check(chain, x, a, rng.integers(0, 5000, N))


def test_halfway_and_fractional_addends_at_binade_edges(chain):
    rng = np.random.default_rng(1)
    N = 30000
    e = rng.integers(-30, 30, N)
    start = rng.choice([1.0, 1.0 + 2.0 ** -23, 2.0 - 2.0 ** -23, 1.5, 1.0 + 2.0 ** -22], N)
    x = (2.0 ** e * start * rng.choice([1.0, -1.0], N)).astype(np.float32)
    frac = rng.choice([0.5, 1.5, 2.5, 3.5, 0.25, 0.75, -0.5, -1.5, -2.5, 1.0, 2.0, 7.0, 1e3,
                       1e5, 0.49, 0.51], N)
    a = (2.0 ** (e - 23) * frac * 2.0 ** rng.integers(-3, 4, N)).astype(np.float32)
    _check(chain, x, a, rng.integers(0, 6000, N))


def test_crossing_zero_and_growth(chain):
    rng = np.random.default_rng(2)
    N = 20000
    x = rng.uniform(0, 10, N).astype(np.float32)
    a = -rng.uniform(1e-4, 1e-2, N).astype(np.float32)
    _check(chain, x, a, rng.integers(0, 5000, N))
    _check(chain, -x, -a, rng.integers(0, 5000, N))
    _check(chain, x[:4000], -a[:4000], rng.integers(0, 20000, 4000))


def test_special_values(chain):
    rng = np.random.default_rng(3)
    sp = np.array([0.0, -0.0, 1e-45, -1e-45, 1e-38, -1e-38, 3e38, -3e38, np.inf, -np.inf,
                   np.nan, 1.0, -1.0], np.float32)
    extra = np.array([1e-40, -1e-40, 1e30, -1e-7, 2.0 ** -149], np.float32)
    N = 50000
    x = rng.choice(sp, N)
    a = rng.choice(np.concatenate([sp, extra]), N)
    _check(chain, x, a, rng.integers(0, 300, N))
    # n = 0 and negative n leave x as it is
    _check(chain, sp, np.full(sp.size, 0.5, np.float32), np.zeros(sp.size, np.int64))
    assert np.array_equal(chain(sp, sp, np.full(sp.size, -3)).view(np.uint32)[:10],
                          sp.view(np.uint32)[:10])
