"""Drop-in for the reference's ``tonari._torch_cuda`` provider module.

``neighbor_list`` has the signature of tonari csrc/torch/bindings_cuda.cpp:59-68
and returns ``[P (E,2) int64, S (E,3) int32]``.  A reference installation can
use it by making ``tonari._extensions.load_torch_cuda`` return this module.
``neighbor_list_fused`` additionally emits i/j/d/D from the same kernel, and
"E", the (2,E) edge_index graph layout (one buffer, no transpose).
"""
from __future__ import annotations

import torch
from torch import Tensor

_INDEX = {"i": 0, "j": 1, "P": 2, "S": 3, "d": 4, "D": 5, "E": 6}


def neighbor_list(
    positions: Tensor,
    batch_ptr: Tensor,
    cell: Tensor,
    pbc: Tensor,
    cutoff: float,
    half_list: bool,
    include_self: bool,
    algorithm: str,
    sorted: bool,
) -> list[Tensor]:
    outputs = torch.ops.tonari_b200.neighbor_list(
        positions, batch_ptr, cell, pbc, float(cutoff), bool(half_list),
        bool(include_self), algorithm, bool(sorted), "PS", 0,
    )
    return [outputs[2], outputs[3]]


def neighbor_list_fused(
    positions: Tensor,
    batch_ptr: Tensor,
    cell: Tensor,
    pbc: Tensor,
    cutoff: float,
    half_list: bool,
    include_self: bool,
    algorithm: str,
    sorted: bool,
    quantities: str,
    index_offset: int = 0,
) -> dict[str, Tensor]:
    """Returns ``{quantity: tensor}`` for each distinct character requested."""
    wanted = "".join(dict.fromkeys(quantities))
    outputs = torch.ops.tonari_b200.neighbor_list(
        positions, batch_ptr, cell, pbc, float(cutoff), bool(half_list),
        bool(include_self), algorithm, bool(sorted), wanted, int(index_offset),
    )
    return {q: outputs[_INDEX[q]] for q in wanted}


def filter_pairs(
    positions: Tensor,
    batch_ptr: Tensor,
    cell: Tensor,
    pairs: Tensor,
    shifts: Tensor,
    cutoff: float,
    quantities: str,
    index_offset: int = 0,
) -> dict[str, Tensor]:
    """The candidate pairs whose exact distance at `positions` is below
    `cutoff`, in candidate order, as ``{quantity: tensor}``."""
    wanted = "".join(dict.fromkeys(quantities))
    outputs = torch.ops.tonari_b200.filter_pairs(
        positions, batch_ptr, cell, pairs, shifts, float(cutoff), wanted, int(index_offset),
    )
    return {q: outputs[_INDEX[q]] for q in wanted}
