"""cufk_b200: B200-native (sm_100a) drop-in for cufk's reconstruction path.

``import cufk_b200 as cufk`` gives the reference's public surface (src/cufk/__init__.py:1-11):
``reconstruct``, ``compile_torsion``, ``BLOCK_SCAN_MAX_POINT_COUNT`` and ``__version__``; and
``reconstruct_long`` for chains longer than ``BLOCK_SCAN_MAX_POINT_COUNT``, which the reference
does not support; ``reconstruct_packed`` for ragged batches (chains of different lengths, packed);
``reconstruct_mse``, the reconstruction fused with a coordinate loss and its gradient;
and ``ops``, the same path as ``torch.library`` operators
(``torch.ops.cufk_b200.*``) that ``torch.compile`` traces through.
"""

from .reconstruct import BLOCK_SCAN_MAX_POINT_COUNT, reconstruct, reconstruct_long, reconstruct_packed
from .losses import reconstruct_mse
from .torsion import compile_torsion
from . import ops  # noqa: E402  (registers the torch.library operators)

__version__ = "0.1.0"

__all__ = [
    "BLOCK_SCAN_MAX_POINT_COUNT",
    "__version__",
    "compile_torsion",
    "ops",
    "reconstruct",
    "reconstruct_long",
    "reconstruct_mse",
    "reconstruct_packed",
]
