"""B200-native Foveal Pattention MLP forward (drop-in for kreasof-ai/foveal-sparse-indexer's hot path).

Public API (same names as the reference package ``foveal_indexer``):

    FovealPattentionMLP, sparsify_model_with_foveal_pattention   (foveal_indexer/foveal_pattention.py)
    FovealIndexer, Route, select_blocks, masked_softmax           (foveal_indexer/core.py)
    BlockSparseLinear                                             (foveal_indexer/block_matmul.py)
    FovealTokenformerLinear, FovealTokenformerFFN                 (foveal_indexer/tokenformer.py)
    triton_pattention, triton_fused_swiglu, TritonFusedSwiGLUFunction,
    TritonSwiGLUPattentionMLP, convert_llm_mlp_to_pattention      (foveal_indexer/pattention_triton.py)

Compute runs in ``libfovealpatt.so`` (hand-written sm_100a CUDA behind the C ABI of
``include/foveal_pattention.h``); build it with ``build.py``.  The directory name contains hyphens: with
the repository root on ``sys.path``, ``import foveal_sparse_indexer_b200`` loads it (the module of that
name at the root binds to this package), as does ``importlib.import_module("foveal-sparse-indexer_b200")``.
"""

import sys as _sys

from . import block_matmul, configs, kernels, pattention, sharding, tokenformer
from ._lib import LIB_PATH, FovealKernelError, load as load_library
from .block_matmul import BlockSparseLinear
from .core import FovealIndexer, Route, masked_softmax, select_blocks
from .foveal_pattention import FovealPattentionMLP, sparsify_model_with_foveal_pattention
from .pattention import (TritonFusedSwiGLUFunction, TritonSwiGLUPattentionMLP, convert_llm_mlp_to_pattention,
                         triton_fused_swiglu, triton_pattention)
from .tokenformer import FovealTokenformerFFN, FovealTokenformerLinear

_sys.modules.setdefault("foveal_sparse_indexer_b200", _sys.modules[__name__])

__all__ = [
    "FovealPattentionMLP",
    "sparsify_model_with_foveal_pattention",
    "FovealIndexer",
    "Route",
    "select_blocks",
    "masked_softmax",
    "BlockSparseLinear",
    "FovealTokenformerLinear",
    "FovealTokenformerFFN",
    "triton_pattention",
    "triton_fused_swiglu",
    "TritonFusedSwiGLUFunction",
    "TritonSwiGLUPattentionMLP",
    "convert_llm_mlp_to_pattention",
    "FovealKernelError",
    "LIB_PATH",
    "load_library",
    "configs",
    "kernels",
    "pattention",
    "sharding",
]
