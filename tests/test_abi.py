"""The C-ABI library loads and exports every entry point include/tonari_b200.h
declares; the PyTorch op registers.  No device work (runs without a GPU)."""
from __future__ import annotations

import ctypes
import re
from pathlib import Path

import numpy as np
import torch

from tonari_b200 import _cabi
from tonari_b200._extensions import CORE_LIBRARY, TORCH_LIBRARY

HEADER = Path(__file__).resolve().parent.parent / "include" / "tonari_b200.h"


def declared_functions():
    text = HEADER.read_text()
    return sorted(set(re.findall(r"^\s*(?:int|int64_t|const char\*)\s+(tnr_\w+)\(", text, re.M)))


def test_library_exports_every_declared_function():
    lib = ctypes.CDLL(str(CORE_LIBRARY))
    names = declared_functions()
    assert set(names) == set(_cabi.EXPORTED)
    for name in names:
        assert hasattr(lib, name), name


def test_version_and_struct_layout():
    assert _cabi.library().tnr_version().decode().count(".") == 2
    # Field offsets must follow the C declaration order with natural alignment.
    assert _cabi.Request.positions.offset == 24
    assert _cabi.Request.cutoff.offset == 80
    assert _cabi.Request.index_offset.offset == 104
    assert ctypes.sizeof(_cabi.Request) == 120
    assert _cabi.Result.edge_index.offset == 56
    assert ctypes.sizeof(_cabi.Result) == 64


def test_input_errors_are_reported_without_device_work():
    # With host mirrors supplied the library validates batch_ptr and the
    # periodic geometry before touching the device.
    lib = _cabi.library()
    positions = np.zeros((1, 3))
    batch_ptr = np.array([0, 1], np.int64)
    cell = np.array([[1.0, 0, 0], [2.0, 0, 0], [0, 0, 4.0]])
    pbc = np.array([1, 1, 0], np.uint8)
    request = _cabi.Request(dtype=1, n_atoms=1, n_structures=1, positions=positions.ctypes.data,
                            batch_ptr=batch_ptr.ctypes.data, cell=cell.ctypes.data,
                            pbc=pbc.ctypes.data, batch_ptr_host=batch_ptr.ctypes.data,
                            cell_host=cell.ctypes.data, pbc_host=pbc.ctypes.data, cutoff=0.5,
                            quantities=12)
    result = _cabi.Result()
    message = ctypes.create_string_buffer(256)
    status = lib.tnr_neighbor_list(ctypes.byref(request), None, None, ctypes.byref(result),
                                   message, len(message))
    assert status == 1 and b"linearly independent" in message.value
    bad_ptr = np.array([1, 1], np.int64)
    request.batch_ptr_host = bad_ptr.ctypes.data
    status = lib.tnr_neighbor_list(ctypes.byref(request), None, None, ctypes.byref(result),
                                   message, len(message))
    assert status == 1 and b"start at zero" in message.value
    request.cutoff = float("nan")
    status = lib.tnr_neighbor_list(ctypes.byref(request), None, None, ctypes.byref(result),
                                   message, len(message))
    assert status == 1 and b"cutoff must be finite" in message.value


def test_static_entry_point_checks_outputs_without_device_work():
    # Output pointers and the capacity are checked before any device work, so
    # a missing buffer is an input error rather than a device-side write.
    lib = _cabi.library()
    request = _cabi.Request(dtype=0, n_atoms=1, n_structures=1, cutoff=1.0,
                            quantities=_cabi.quantity_mask("PS"))
    result = _cabi.Result(P=16)
    message = ctypes.create_string_buffer(256)
    status = lib.tnr_neighbor_list_static(ctypes.byref(request), None, 8, ctypes.byref(result),
                                          message, len(message))
    assert status == 1 and b"result->S must be set" in message.value
    result = _cabi.Result(P=16, S=16)
    status = lib.tnr_neighbor_list_static(ctypes.byref(request), None, -1, ctypes.byref(result),
                                          message, len(message))
    assert status == 1 and b"pair_capacity must be nonnegative" in message.value


def test_torch_op_registers():
    torch.ops.load_library(str(TORCH_LIBRARY))
    schema = str(torch.ops.tonari_b200.neighbor_list.default._schema)
    assert "quantities" in schema and "index_offset" in schema
