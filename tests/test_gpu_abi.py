"""tnr_neighbor_list through the C ABI on the GPU, with no allocator
(allocator == NULL): the library then allocates workspace and outputs with
cudaMallocAsync on the caller's stream, and the caller frees the outputs.
The pair set must equal the reference CPU core's (exact keys) and D must
match the reference frontend formula (``src/tonari/_torch_frontend.py:94-104``).
"""
from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

from oracle import oracle
from tests.support import assert_same_pairs, expected_pairs
from tonari_b200 import _cabi, workloads

pytestmark = pytest.mark.gpu


class _DeviceArray:
    """A borrowed device buffer, exposed to torch via __cuda_array_interface__."""

    def __init__(self, pointer: int, shape: tuple, typestr: str):
        self.__cuda_array_interface__ = {"shape": shape, "typestr": typestr,
                                         "data": (pointer, False), "version": 3, "strides": None}


def _device_free(pointer: int) -> None:
    from cuda.bindings import runtime

    (error,) = runtime.cudaFree(pointer)
    assert error == runtime.cudaError_t.cudaSuccess, error


@pytest.mark.parametrize("sorted_pairs", [False, True])
def test_default_allocator_matches_reference(sorted_pairs):
    w = workloads.config5(n_structures=48, seed=51)
    positions, cell, pbc, batch_ptr = w.torch_inputs("cuda")
    stream = torch.cuda.Stream()
    request = _cabi.Request(
        dtype=0, n_atoms=w.n_atoms, n_structures=len(w.batch_ptr) - 1,
        positions=positions.data_ptr(), batch_ptr=batch_ptr.data_ptr(), cell=cell.data_ptr(),
        pbc=pbc.data_ptr(), cutoff=w.cutoff, half_list=1, include_self=0, algorithm=0,
        quantities=_cabi.quantity_mask("PSD"), index_offset=0, sorted=int(sorted_pairs))
    result = _cabi.Result()
    message = ctypes.create_string_buffer(512)
    torch.cuda.synchronize()
    status = _cabi.library().tnr_neighbor_list(ctypes.byref(request), None,
                                               ctypes.c_void_p(stream.cuda_stream),
                                               ctypes.byref(result), message, len(message))
    stream.synchronize()
    assert status == 0, (status, message.value)
    n = result.n_pairs
    assert n > 0
    try:
        P = torch.as_tensor(_DeviceArray(result.P, (n, 2), "<i8"), device="cuda").cpu().numpy()
        S = torch.as_tensor(_DeviceArray(result.S, (n, 3), "<i4"), device="cuda").cpu().numpy()
        D = torch.as_tensor(_DeviceArray(result.D, (n, 3), "<f4"), device="cuda").cpu().numpy()
    finally:
        for pointer in (result.P, result.S, result.D):
            _device_free(pointer)
    assert_same_pairs(P, S, *expected_pairs(w.positions, w.cell, w.pbc, w.cutoff, w.batch_ptr,
                                            half_list=True))
    if sorted_pairs:
        assert np.all(np.diff(P[:, 0]) >= 0)
    ref_D = oracle.public_displacements(w.positions, w.cell, w.batch_ptr, P, S).astype(np.float64)
    scale = np.maximum(np.linalg.norm(ref_D, axis=1), w.cutoff * 1e-3)
    assert np.all(np.linalg.norm(D.astype(np.float64) - ref_D, axis=1) <= 1e-5 * scale)
