"""B200-native (sm_100a) tropical / max-plus hot path of TropFormer and TSRN.

Drop-in replacements for the reference's tropical operator surface
(Mediocr3Mik3/MK_III_Technologies_TSRN): the max-plus linear
(``cuda/maxplus_binding.py``, ``tropformer.TropicalLinear``), the tropical
attention scores (``deep_tropical_net.DTNAttention``, TSRN
``TropicalAttention``) and the ``TropicalSSM`` max-plus scan.  Compute runs in
the in-tree CUDA library ``_tropical_b200.so`` through a C ABI
(``include/tropical_b200.h``); there is no CPU fallback.
"""
from ._lib import is_available as library_available  # noqa: F401

__all__ = ["library_available"]
