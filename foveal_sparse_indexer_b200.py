"""Importable name of the ``foveal-sparse-indexer_b200`` package.

The package directory's name contains hyphens, which a plain ``import`` statement cannot spell.  With
the repository root on ``sys.path``, ``import foveal_sparse_indexer_b200`` loads the package through
this module and binds the name to the package itself (same module object, same attributes).
"""

import importlib as _importlib
import sys as _sys

_pkg = _importlib.import_module("foveal-sparse-indexer_b200")
_sys.modules[__name__] = _pkg
