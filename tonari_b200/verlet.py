"""Verlet-skin reuse of a neighbor list across steps.

tonari lists a Verlet skin and prepared workspaces as future directions
(tonari docs/design.md:127).  ``VerletNeighborList`` builds the list once with
``cutoff + skin`` through the regular provider call and, while no atom has
moved more than 0.49 * skin since that build (and cell, pbc and batch_ptr
are unchanged), answers each step by filtering those candidates on the
device (``tnr_filter_pairs``): the public displacement at the current
positions, evaluated exactly as the search's decisive test, must be strictly
shorter than ``cutoff``.  A pair closer than ``cutoff`` now was closer than
``cutoff + 2 * 0.49 * skin`` at the build, so the candidates contain it.
The allowed motion is further reduced by a rounding allowance of 64 machine
epsilons of the coordinate scale (the reference's own padding rule, tonari
csrc/core/neighbors_cpu.cpp:156-219), so the result is the same pair set as
``neighbor_list`` at ``cutoff``; with ``sorted=True`` the order is
source-major as well.  A skin too small for that allowance rebuilds on every
call.
"""
from __future__ import annotations

from math import isfinite

import torch
from torch import Tensor

from ._extensions import load_torch_cuda
from ._frontend import (
    _KernelDisplacements,
    _require_torch_tensors,
    neighbor_list_torch,
    normalize_torch_inputs,
    validate_torch_inputs,
)

_VALID_QUANTITIES = set("ijPSdD")
_SKIN_FRACTION = 0.49


class VerletNeighborList:
    """Callable ``(positions, cell, pbc, batch_ptr=None) -> tuple`` with the
    options of ``neighbor_list`` fixed at construction."""

    def __init__(self, cutoff: float, skin: float, quantities: str = "PSD", *,
                 algorithm: str = "auto", sorted: bool = False, half_list: bool = False,
                 include_self: bool = False) -> None:
        cutoff, skin = float(cutoff), float(skin)
        if not isfinite(cutoff) or cutoff <= 0:
            raise ValueError("cutoff must be finite and positive")
        if not isfinite(skin) or skin < 0:
            raise ValueError("skin must be finite and non-negative")
        if not isinstance(quantities, str) or set(quantities) - _VALID_QUANTITIES:
            raise ValueError(f"unsupported quantities: {quantities!r}")
        self.cutoff, self.skin, self.quantities = cutoff, skin, quantities
        self.options = {"algorithm": algorithm, "sorted": sorted, "half_list": half_list,
                        "include_self": include_self}
        self.rebuilds = 0
        self._state = None

    def _stale(self, positions: Tensor, cell: Tensor, pbc: Tensor, batch_ptr: Tensor) -> bool:
        state = self._state
        if state is None:
            return True
        reference, ref_cell, ref_pbc, ref_ptr = state["inputs"]
        if (positions.shape != reference.shape or positions.dtype != reference.dtype
                or positions.device != reference.device or cell.shape != ref_cell.shape
                or batch_ptr.shape != ref_ptr.shape):
            return True
        if not (torch.equal(cell, ref_cell) and torch.equal(pbc, ref_pbc)
                and torch.equal(batch_ptr, ref_ptr)):
            return True
        if positions.numel() == 0:
            return False
        moved = (positions.detach().double() - reference.double()).norm(dim=1).max()
        return bool(moved > state["allowed"])

    def __call__(self, positions, cell, pbc, batch_ptr=None):
        _require_torch_tensors(cell=cell, pbc=pbc, batch_ptr=batch_ptr)
        positions, cell, pbc, batch_ptr = normalize_torch_inputs(positions, cell, pbc, batch_ptr)
        validate_torch_inputs(positions, cell, pbc, self.cutoff, batch_ptr)
        if not positions.is_cuda:
            raise RuntimeError(
                "tonari_b200 is the CUDA provider only; CPU tensors are served by "
                "tonari's CPU provider"
            )
        cell_values = cell.detach().contiguous()
        if self._stale(positions, cell_values, pbc, batch_ptr):
            pairs, shifts = neighbor_list_torch(
                "PS", positions.detach(), cell_values, pbc, self.cutoff + self.skin, batch_ptr,
                cpu_threads=None, **self.options)
            eps = torch.finfo(positions.dtype).eps
            largest_shift = float(shifts.abs().max()) if shifts.numel() else 0.0
            scale = 2.0 * float(positions.detach().abs().max()) if positions.numel() else 0.0
            scale += (largest_shift + 1.0) * float(cell_values.abs().sum(dim=(1, 2)).max())
            self._state = {
                "inputs": (positions.detach().clone(), cell_values.clone(), pbc.clone(),
                           batch_ptr.clone()),
                "pairs": pairs, "shifts": shifts,
                "allowed": _SKIN_FRACTION * self.skin - 64.0 * eps * scale,
            }
            self.rebuilds += 1
        backend = load_torch_cuda()
        wants_vectors = "d" in self.quantities or "D" in self.quantities
        differentiable = wants_vectors and torch.is_grad_enabled() and (
            positions.requires_grad or cell.requires_grad)
        requested = set(self.quantities) | ({"P", "S", "D"} if differentiable else set())
        values = backend.filter_pairs(
            positions.detach().contiguous(), batch_ptr.contiguous(), cell_values,
            self._state["pairs"], self._state["shifts"], self.cutoff,
            "".join(q for q in "ijPSdD" if q in requested))
        if differentiable:
            source = values["P"][:, 0].contiguous()
            target = values["P"][:, 1].contiguous()
            pair_batch = torch.bucketize(source, batch_ptr[1:], right=True)
            values["D"] = _KernelDisplacements.apply(positions, cell, values["D"], source, target,
                                                     values["S"], pair_batch)
            if "d" in self.quantities:
                values["d"] = torch.linalg.vector_norm(values["D"], dim=1)
        return tuple(values[q] for q in self.quantities)
