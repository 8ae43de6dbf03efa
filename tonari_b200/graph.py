"""Graph adapter: the neighbor list in the (2, E) ``edge_index`` layout.

tonari keeps graph terms out of its core API; its design notes say that a
GNN/PyG adapter should turn the edge-first ``P`` into
``edge_index = P.T.contiguous()`` and map ``D`` to edge vectors at the
adapter boundary (tonari docs/design.md:61, :127; README.md:97).  This
adapter gets that layout straight from the write pass: sources and targets
are written as the two rows of one (2, E) buffer, so there is no transposed
copy.  Inputs, options, validation and errors are those of
:func:`tonari_b200.neighbor_list`.
"""
from __future__ import annotations

import torch
from torch import Tensor

from ._extensions import load_torch_cuda
from ._frontend import (
    _KernelDisplacements,
    _require_torch_tensors,
    normalize_torch_inputs,
    validate_torch_inputs,
)

_VALID_ALGORITHMS = ("auto", "brute_force", "cell_list")


def neighbor_graph(
    positions: Tensor,
    cell: Tensor,
    pbc: Tensor,
    cutoff: float,
    batch_ptr: Tensor | None = None,
    *,
    algorithm: str = "auto",
    sorted: bool = False,
    half_list: bool = False,
    include_self: bool = False,
    edge_vectors: bool = True,
) -> tuple[Tensor, Tensor, Tensor | None]:
    """Returns ``(edge_index, shifts, vectors)``.

    ``edge_index`` is (2, E) int64 (row 0 sources, row 1 targets), ``shifts``
    (E, 3) int32 and ``vectors`` (E, 3) in the input dtype -- the public
    displacement ``pos[j] - pos[i] + S @ cell`` -- or ``None`` when
    ``edge_vectors`` is false.  Gradients flow from ``vectors`` to
    ``positions`` and ``cell`` as for ``neighbor_list``'s ``D``.
    """
    if not isinstance(positions, Tensor):
        raise TypeError("positions must be a PyTorch tensor")
    if algorithm not in _VALID_ALGORITHMS:
        raise ValueError("algorithm must be 'auto', 'brute_force', or 'cell_list'")
    if not all(isinstance(option, bool) for option in (sorted, half_list, include_self)):
        raise TypeError("sorted, half_list, and include_self must be bool")
    _require_torch_tensors(cell=cell, pbc=pbc, batch_ptr=batch_ptr)
    positions, cell, pbc, batch_ptr = normalize_torch_inputs(positions, cell, pbc, batch_ptr)
    cutoff = float(cutoff)
    validate_torch_inputs(positions, cell, pbc, cutoff, batch_ptr)
    if not positions.is_cuda:
        raise RuntimeError(
            "tonari_b200 is the CUDA provider only; CPU tensors are served by "
            "tonari's CPU provider"
        )
    try:
        backend = load_torch_cuda()
    except ImportError as error:
        raise RuntimeError(f"the CUDA provider is unavailable: {error}") from error
    values = backend.neighbor_list_fused(
        positions.detach().contiguous(), batch_ptr.contiguous(), cell.detach().contiguous(),
        pbc.contiguous(), cutoff, half_list, include_self, algorithm, sorted,
        "ESD" if edge_vectors else "ES",
    )
    edge_index, shifts = values["E"], values["S"]
    vectors = values.get("D")
    if edge_vectors and torch.is_grad_enabled() and (positions.requires_grad or cell.requires_grad):
        source, target = edge_index[0], edge_index[1]
        pair_batch = torch.bucketize(source, batch_ptr[1:], right=True)
        vectors = _KernelDisplacements.apply(positions, cell, vectors, source, target, shifts,
                                             pair_batch)
    return edge_index, shifts, vectors
