"""Loader for the native provider (mirrors tonari src/tonari/_extensions.py:63-66).

The op library is built in-tree by ``tonari_b200/_build.py``.  There is no
fallback: if the library is missing, loading raises ``ImportError`` and the
frontend turns it into ``RuntimeError("the CUDA provider is unavailable: ...")``
exactly as the reference frontend does (src/tonari/_torch_frontend.py:141-144).
"""
from __future__ import annotations

from functools import lru_cache
from pathlib import Path

import os

# TONARI_B200_LIB_DIR points the loader at another build of the two libraries
# (used to compare builds side by side); default: the in-tree _lib directory.
_LIB = Path(os.environ.get("TONARI_B200_LIB_DIR", Path(__file__).resolve().parent / "_lib"))
CORE_LIBRARY = _LIB / "libtonari_b200.so"
TORCH_LIBRARY = _LIB / "libtonari_b200_torch.so"


@lru_cache
def load_torch_cuda():
    """Load the custom op library and return the provider module.

    The returned module exposes ``neighbor_list(positions, batch_ptr, cell,
    pbc, cutoff, half_list, include_self, algorithm, sorted) -> [P, S]``, the
    interface of the reference's ``tonari._torch_cuda`` module.
    """
    import torch

    if not TORCH_LIBRARY.exists():
        raise ImportError(
            f"{TORCH_LIBRARY.name} is not built; run `python -m tonari_b200._build`"
        )
    torch.ops.load_library(str(TORCH_LIBRARY))
    from . import _torch_cuda

    return _torch_cuda
