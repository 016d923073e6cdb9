"""B200-native Foveal Pattention MLP forward (drop-in for kreasof-ai/foveal-sparse-indexer's hot path).

Public API (same names as the reference package ``foveal_indexer``):

    FovealPattentionMLP, sparsify_model_with_foveal_pattention   (foveal_indexer/foveal_pattention.py)
    FovealIndexer, Route, select_blocks, masked_softmax           (foveal_indexer/core.py)

Compute runs in ``libfovealpatt.so`` (hand-written sm_100a CUDA behind the C ABI of
``include/foveal_pattention.h``); build it with ``build.py``.  The directory name contains hyphens, so
import it with ``importlib.import_module("foveal-sparse-indexer_b200")``; after that first import the
alias ``foveal_sparse_indexer_b200`` is registered in ``sys.modules``.
"""

import sys as _sys

from . import configs, kernels, sharding
from ._lib import LIB_PATH, FovealKernelError, load as load_library
from .core import FovealIndexer, Route, masked_softmax, select_blocks
from .foveal_pattention import FovealPattentionMLP, sparsify_model_with_foveal_pattention

_sys.modules.setdefault("foveal_sparse_indexer_b200", _sys.modules[__name__])

__all__ = [
    "FovealPattentionMLP",
    "sparsify_model_with_foveal_pattention",
    "FovealIndexer",
    "Route",
    "select_blocks",
    "masked_softmax",
    "FovealKernelError",
    "LIB_PATH",
    "load_library",
    "configs",
    "kernels",
    "sharding",
]
