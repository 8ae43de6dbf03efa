"""Public API of the B200 provider: ``neighbor_list``.

Same signature, option validation, messages and output contract as
tonari src/tonari/api.py:52-234 for Torch CUDA tensors.  CPU tensors and
NumPy arrays are rejected with a RuntimeError: this package replaces only the
CUDA provider, and there is no CPU fallback on its path.
"""
from __future__ import annotations

import builtins
from typing import Literal

_VALID_QUANTITIES = frozenset("ijPSdD")
_Algorithm = Literal["auto", "brute_force", "cell_list"]
_VALID_ALGORITHMS = frozenset(("auto", "brute_force", "cell_list"))


def neighbor_list(
    quantities: str,
    positions,
    cell,
    pbc,
    cutoff: float,
    batch_ptr=None,
    *,
    algorithm: _Algorithm = "auto",
    cpu_threads: int | None = None,
    sorted: bool = False,
    half_list: bool = False,
    include_self: bool = False,
):
    """Build an atomistic neighbor list within a strict distance cutoff.

    Finds every atom-image pair (source i, target j, integer cell shift S)
    whose squared distance is strictly below ``cutoff**2``, for a batch of
    structures concatenated along ``batch_ptr``.  Returns a tuple with one
    tensor per character of ``quantities`` (``i j P S d D``), on the input
    device.  ``sorted=True`` returns pairs ordered by source; otherwise the
    order is unspecified (cell order).
    See tonari src/tonari/api.py:66-174 for the full contract.
    """
    if not isinstance(quantities, str):
        raise TypeError("quantities must be a string")
    invalid_quantities = set(quantities) - _VALID_QUANTITIES
    if invalid_quantities:
        invalid = "".join(builtins.sorted(invalid_quantities))
        raise ValueError(f"unsupported quantities: {invalid!r}")
    if not isinstance(algorithm, str):
        raise TypeError("algorithm must be a string")
    if algorithm not in _VALID_ALGORITHMS:
        raise ValueError("algorithm must be 'auto', 'brute_force', or 'cell_list'")
    if cpu_threads is not None:
        if isinstance(cpu_threads, bool) or not isinstance(cpu_threads, int):
            raise TypeError("cpu_threads must be an integer or None")
        if cpu_threads < 1:
            raise ValueError("cpu_threads must be positive")
        if cpu_threads > (1 << 63) - 1:
            raise ValueError("cpu_threads is too large")
    if not all(isinstance(option, bool) for option in (sorted, half_list, include_self)):
        raise TypeError("sorted, half_list, and include_self must be bool")
    import torch

    if isinstance(positions, torch.Tensor):
        from ._frontend import neighbor_list_torch

        return neighbor_list_torch(
            quantities, positions, cell, pbc, cutoff, batch_ptr, algorithm=algorithm,
            cpu_threads=cpu_threads, sorted=sorted, half_list=half_list,
            include_self=include_self,
        )
    import numpy as np

    if isinstance(positions, np.ndarray):
        raise RuntimeError(
            "tonari_b200 is the CUDA provider only; NumPy inputs are served by "
            "tonari's CPU provider"
        )
    raise TypeError("positions must be a PyTorch tensor or NumPy array")
