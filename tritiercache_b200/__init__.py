"""tritiercache_b200 -- TriTierCache's decode hot path on NVIDIA B200 (sm_100a).

Drop-in for the reference package ``tri_tier``: ``TriTierCache`` (cache.py),
the Hugging Face attention patch (integration/patch_model.py) and the
``_C`` extension surface (fused_attention_decode, quantize_k_block,
quantize_v_block, dequantize_k, dequantize_v, TriTierCacheEngine), all backed
by hand-written CUDA kernels in libtritier_b200.so behind a C ABI
(include/tritier_b200.h).  ``install_as_tri_tier()`` registers this package
under the reference's module names.
"""
from __future__ import annotations

import sys

from . import _C
from ._lib import LIB_PATH
from .cache import TriTierCache
from .constants import CHUNK_SIZE, DEVICE, SINK_SIZE, UPDATE_THRESHOLD

__version__ = "0.1.0"

HAS_CPP_EXT = True  # the compute path is the CUDA library; there is nothing else

__all__ = ["TriTierCache", "DEVICE", "UPDATE_THRESHOLD", "CHUNK_SIZE", "SINK_SIZE", "HAS_CPP_EXT", "_C",
           "__version__", "install_as_tri_tier", "LIB_PATH"]


def install_as_tri_tier() -> None:
    """Makes ``import tri_tier`` / ``tri_tier._C`` / ``tri_tier.integration.patch_model``
    resolve to this package, so code written against the reference runs unchanged."""
    from . import cache, constants
    from .integration import patch_llama, patch_model
    import tritiercache_b200.integration as integ

    pkg = sys.modules[__name__]
    sys.modules.setdefault("tri_tier", pkg)
    sys.modules.setdefault("tri_tier._C", _C)
    sys.modules.setdefault("tri_tier.cache", cache)
    sys.modules.setdefault("tri_tier.constants", constants)
    sys.modules.setdefault("tri_tier.integration", integ)
    sys.modules.setdefault("tri_tier.integration.patch_model", patch_model)
    sys.modules.setdefault("tri_tier.integration.patch_llama", patch_llama)
