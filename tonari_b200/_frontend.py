"""Torch frontend of the B200 provider.

Normalisation and validation restate tonari src/tonari/_torch_frontend.py:25-75
(same checks, same messages, same order).  The provider call then asks the
kernel for every requested quantity at once (i/j/P/S/d/D fused into the write
pass) instead of assembling i/j/d/D with extra passes
(src/tonari/_torch_frontend.py:78-105).  When autograd needs gradients of d/D
with respect to positions or cell, the kernel's D enters a custom autograd
function whose backward is the analytic gradient of the reference formula, so
the gradient contract is unchanged.
"""
from __future__ import annotations

from math import isfinite

import torch
from torch import Tensor

from ._extensions import load_torch_cuda


def _require_torch_tensors(*, cell: object, pbc: object, batch_ptr: object | None) -> None:
    for name, tensor in (("cell", cell), ("pbc", pbc), ("batch_ptr", batch_ptr)):
        if tensor is not None and not isinstance(tensor, Tensor):
            raise TypeError(
                "positions, cell, pbc, and batch_ptr must all be PyTorch tensors; "
                f"{name} has type {type(tensor).__name__}"
            )


def normalize_torch_inputs(positions, cell, pbc, batch_ptr):
    if positions.ndim != 2 or positions.shape[1] != 3:
        raise ValueError("positions must have shape (N_total, 3)")
    if batch_ptr is None:
        if cell.ndim != 2 or cell.shape != (3, 3):
            raise ValueError("single-structure cell must have shape (3, 3)")
        if pbc.ndim != 1 or pbc.shape != (3,):
            raise ValueError("single-structure pbc must have shape (3,)")
        batch_ptr = torch.tensor([0, len(positions)], dtype=torch.int64, device=positions.device)
        cell = cell.unsqueeze(0)
        pbc = pbc.unsqueeze(0)
    else:
        if cell.ndim != 3:
            raise ValueError("batched cell must have shape (B, 3, 3)")
        if pbc.ndim != 2:
            raise ValueError("batched pbc must have shape (B, 3)")
    return positions, cell, pbc, batch_ptr


def validate_torch_inputs(positions, cell, pbc, cutoff, batch_ptr) -> None:
    if positions.device.type not in ("cpu", "cuda"):
        raise ValueError("positions must be a CPU or CUDA tensor")
    if positions.dtype not in (torch.float32, torch.float64):
        raise ValueError("positions must have dtype float32 or float64")
    if batch_ptr.ndim != 1 or batch_ptr.numel() == 0 or batch_ptr.dtype != torch.int64:
        raise ValueError("batch_ptr must be int64 with shape (B + 1,)")
    if cell.shape != (batch_ptr.numel() - 1, 3, 3):
        raise ValueError("cell must have shape (B, 3, 3)")
    if cell.dtype != positions.dtype:
        raise ValueError("cell and positions must have the same dtype")
    if pbc.shape != (batch_ptr.numel() - 1, 3) or pbc.dtype != torch.bool:
        raise ValueError("pbc must be bool with shape (B, 3)")
    if any(tensor.device != positions.device for tensor in (cell, pbc, batch_ptr)):
        raise ValueError("positions, cell, pbc, and batch_ptr must be on the same device")
    if not isfinite(cutoff) or cutoff <= 0:
        raise ValueError("cutoff must be finite and positive")


class _KernelDisplacements(torch.autograd.Function):
    """D from the kernel in the forward; the analytic gradient of the
    reference formula D = pos[j] - pos[i] + S @ cell[b(i)]
    (src/tonari/_torch_frontend.py:94-104) in the backward:
    dL/dpos[j] += g, dL/dpos[i] -= g, dL/dcell[b] += S^T g."""

    @staticmethod
    def forward(ctx, positions, cell, displacements, source, target, shifts, pair_batch):
        ctx.save_for_backward(source, target, shifts, pair_batch)
        ctx.shapes = (positions.shape, cell.shape)
        return displacements

    @staticmethod
    def backward(ctx, grad):
        source, target, shifts, pair_batch = ctx.saved_tensors
        positions_shape, cell_shape = ctx.shapes
        grad_positions = grad_cell = None
        if ctx.needs_input_grad[0]:
            grad_positions = grad.new_zeros(positions_shape)
            grad_positions.index_add_(0, target, grad)
            grad_positions.index_add_(0, source, -grad)
        if ctx.needs_input_grad[1]:
            grad_cell = grad.new_zeros(cell_shape)
            outer = shifts.to(grad.dtype).unsqueeze(2) * grad.unsqueeze(1)  # (E, 3, 3)
            grad_cell.index_add_(0, pair_batch, outer)
        return grad_positions, grad_cell, None, None, None, None, None


def neighbor_list_torch(quantities, positions, cell, pbc, cutoff, batch_ptr, *, algorithm,
                        cpu_threads, sorted, half_list, include_self, index_offset=0):
    _require_torch_tensors(cell=cell, pbc=pbc, batch_ptr=batch_ptr)
    positions, cell, pbc, batch_ptr = normalize_torch_inputs(positions, cell, pbc, batch_ptr)
    cutoff = float(cutoff)
    validate_torch_inputs(positions, cell, pbc, cutoff, batch_ptr)
    if not positions.is_cuda:
        raise RuntimeError(
            "tonari_b200 is the CUDA provider only; CPU tensors and NumPy arrays "
            "are served by tonari's CPU provider"
        )
    if cpu_threads is not None:
        raise ValueError("cpu_threads only applies to CPU inputs")
    try:
        backend = load_torch_cuda()
    except ImportError as error:
        raise RuntimeError(f"the CUDA provider is unavailable: {error}") from error

    wants_vectors = "d" in quantities or "D" in quantities
    differentiable = wants_vectors and torch.is_grad_enabled() and (
        positions.requires_grad or cell.requires_grad
    )
    requested = set(quantities)
    if differentiable:
        requested |= {"P", "S", "D"}
    values = backend.neighbor_list_fused(
        positions.detach().contiguous(), batch_ptr.contiguous(), cell.detach().contiguous(),
        pbc.contiguous(), cutoff, half_list, include_self, algorithm, sorted,
        "".join(q for q in "ijPSdD" if q in requested), index_offset,
    )
    if differentiable:
        pairs = values["P"]
        if index_offset:
            pairs = pairs - index_offset
        source = pairs[:, 0].contiguous()
        target = pairs[:, 1].contiguous()
        pair_batch = torch.bucketize(source, batch_ptr[1:], right=True)
        displacements = _KernelDisplacements.apply(
            positions, cell, values["D"], source, target, values["S"], pair_batch)
        values["D"] = displacements
        if "d" in quantities:
            values["d"] = torch.linalg.vector_norm(displacements, dim=1)
    return tuple(values[q] for q in quantities)
