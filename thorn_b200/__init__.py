"""thorn_b200: the THORN optimizer step on B200 (sm_100a) kernels.

``from thorn_b200 import THORN`` is a drop-in for ``from thorn import THORN``
(pykeio/THORN v3.1.1).
"""
from . import ops  # noqa: F401  (registers torch.ops.thorn_b200.*)
from .host_stepper import PinnedStepper, pinned_block  # noqa: F401
from .optimizer import THORN, THORNGroup, THORNNonOrthoGroup, THORNOrthoGroup  # noqa: F401

__version__ = "0.1.0"
__all__ = ["THORN", "THORNOrthoGroup", "THORNNonOrthoGroup", "THORNGroup", "PinnedStepper", "pinned_block"]
