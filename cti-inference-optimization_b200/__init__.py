"""B200-native (sm_100a) hot path of the generative ad-ranking CTR model of
shiguangke1/cti-inference-optimization: the Top-2 sparse MoE layer and the
28-feature embedding-bag pooling, as hand-written CUDA behind a C ABI
(``include/cti_b200.h``), with drop-in ``SMoE`` / ``RepEncoder`` modules.

Import it as ``cti_b200`` (the repository root's ``cti_b200.py`` maps that
name to this directory).
"""
from . import build  # noqa: F401  (no CUDA needed)
from ._lib import LIB_PATH, lib  # noqa: F401  (raises if the library is missing)
from . import ops  # noqa: F401
from .embedding import RepEncoder, flatten_slot_batch  # noqa: F401
from .moe import Expert, SMoE, TopKGate  # noqa: F401

__all__ = ["SMoE", "TopKGate", "Expert", "RepEncoder", "ops", "flatten_slot_batch", "lib"]
