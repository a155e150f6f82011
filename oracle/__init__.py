"""CPU oracle for the tropical hot path -- TEST INFRASTRUCTURE ONLY.

This package restates, in numpy (float32 where the reference computes in
float32, float64 where a tolerance reference is needed), the algorithms of
Mediocr3Mik3/MK_III_Technologies_TSRN that the CUDA library replaces.  Each
function cites the reference file:line it follows.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py`` (its CPU
baseline and ``--impl reference`` arm) may import it, and only as the checker
or as the timed CPU baseline.  The product path (``mk_iii_technologies_tsrn_b200``)
never imports it and has no CPU fallback.

The oracle is pinned against golden vectors produced by running the
reference's own PyTorch code (``tests/golden/gen_golden.py``) and against the
reference's hand-computed known-answer test (``cuda/test_kernel.py:117-136``).
"""
from .maxplus import (  # noqa: F401
    maxplus_fwd,
    maxplus_fwd_bf16,
    maxplus_matmul,
    tropical_power_chain,
    round_bf16,
    tsrn_attention_fwd,
    lfdual_act,
    esn_gru_fwd,
    esn_leaky_fwd,
    maxplus_bwd_argmax,
    maxplus_bwd_smooth,
    maxplus_lse_fwd,
)
from .scan import scan_fwd, scan_bwd, scan_closed_form  # noqa: F401
