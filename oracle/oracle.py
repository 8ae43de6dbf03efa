"""TEST INFRASTRUCTURE ONLY: ctypes front-ends for the two CPU checkers.

* ``ref_*``  -- oracle/_ref/libtonari_ref.so, the reference's own CPU search
  core (tonari csrc/core/neighbors_cpu.cpp:976-1030) compiled from its sources
  with oracle/ref_shim.cpp.  Bit-exact pair-set oracle and the timed
  ``"kind": "reference"`` CPU baseline.
* ``port_*`` -- oracle/_port/libnl_oracle.so, the plain-C restatement in
  oracle/nl_oracle.c (brute-force enumeration with the reference's exact
  candidate predicate).  Always buildable; pinned against ``ref_*`` and the
  golden fixtures by tests/test_oracle.py.

Only tests/, ``__graft_entry__.smoke()`` and bench.py's CPU-baseline legs may
import this module.  The product never does.
"""
from __future__ import annotations

import ctypes
import os
from pathlib import Path

import numpy as np

_HERE = Path(__file__).resolve().parent
REF_LIBRARY = _HERE / "_ref" / "libtonari_ref.so"
PORT_LIBRARY = _HERE / "_port" / "libnl_oracle.so"

_ALGORITHMS = {"auto": 0, "brute_force": 1, "cell_list": 2}


class OracleInputError(ValueError):
    """The checker rejected its inputs (reference InputError)."""


class OracleSearchError(RuntimeError):
    """The checker failed during the search (reference SearchError)."""


def _raise(status: int, message: bytes) -> None:
    text = message.value.decode() if hasattr(message, "value") else str(message)
    if status == 1:
        raise OracleInputError(text)
    if status == 2:
        raise OracleSearchError(text)
    raise RuntimeError(text)


_ref_lib = None
_port_lib = None


def ref_available() -> bool:
    return REF_LIBRARY.exists()


def port_available() -> bool:
    return PORT_LIBRARY.exists()


def _load_ref():
    global _ref_lib
    if _ref_lib is None:
        lib = ctypes.CDLL(str(REF_LIBRARY))
        lib.tnr_ref_neighbor_list.restype = ctypes.c_int
        lib.tnr_ref_neighbor_list.argtypes = [
            ctypes.c_int, ctypes.c_void_p, ctypes.c_int64, ctypes.c_void_p, ctypes.c_int64,
            ctypes.c_void_p, ctypes.c_void_p, ctypes.c_double, ctypes.c_int, ctypes.c_int,
            ctypes.c_int, ctypes.c_int64, ctypes.POINTER(ctypes.c_void_p),
            ctypes.POINTER(ctypes.c_int64), ctypes.c_char_p, ctypes.c_size_t,
        ]
        lib.tnr_ref_take.restype = ctypes.c_int
        lib.tnr_ref_take.argtypes = [
            ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_char_p, ctypes.c_size_t,
        ]
        lib.tnr_ref_release.argtypes = [ctypes.c_void_p]
        _ref_lib = lib
    return _ref_lib


def _load_port():
    global _port_lib
    if _port_lib is None:
        lib = ctypes.CDLL(str(PORT_LIBRARY))
        lib.oracle_neighbor_list.restype = ctypes.c_int
        lib.oracle_neighbor_list.argtypes = [
            ctypes.c_int, ctypes.c_void_p, ctypes.c_int64, ctypes.c_void_p, ctypes.c_int64,
            ctypes.c_void_p, ctypes.c_void_p, ctypes.c_double, ctypes.c_int, ctypes.c_int,
            ctypes.POINTER(ctypes.POINTER(ctypes.c_int64)),
            ctypes.POINTER(ctypes.POINTER(ctypes.c_int32)),
            ctypes.POINTER(ctypes.c_int64), ctypes.c_char_p, ctypes.c_size_t,
        ]
        lib.oracle_periodic_metadata.restype = ctypes.c_int
        lib.oracle_periodic_metadata.argtypes = [
            ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64, ctypes.c_double,
            ctypes.c_void_p, ctypes.c_void_p, ctypes.c_char_p, ctypes.c_size_t,
        ]
        lib.oracle_free_pairs.argtypes = [ctypes.c_void_p, ctypes.c_void_p]
        _port_lib = lib
    return _port_lib


def _normalise(positions, cell, pbc, batch_ptr):
    positions = np.ascontiguousarray(positions)
    if positions.dtype not in (np.float32, np.float64):
        raise TypeError("positions must be float32 or float64")
    cell = np.ascontiguousarray(cell, dtype=positions.dtype)
    pbc = np.ascontiguousarray(pbc, dtype=np.uint8)
    if batch_ptr is None:
        batch_ptr = np.array([0, len(positions)], dtype=np.int64)
        cell = cell.reshape(1, 3, 3)
        pbc = pbc.reshape(1, 3)
    batch_ptr = np.ascontiguousarray(batch_ptr, dtype=np.int64)
    return positions, cell, pbc, batch_ptr


def ref_neighbor_list(positions, cell, pbc, cutoff, batch_ptr=None, *, half_list=False,
                      include_self=False, algorithm="auto", threads=None):
    """Reference CPU search.  Returns (pairs (E,2) int64, shifts (E,3) int32)."""
    positions, cell, pbc, batch_ptr = _normalise(positions, cell, pbc, batch_ptr)
    lib = _load_ref()
    threads = threads or os.cpu_count() or 1
    handle = ctypes.c_void_p()
    count = ctypes.c_int64()
    error = ctypes.create_string_buffer(512)
    status = lib.tnr_ref_neighbor_list(
        int(positions.dtype == np.float64), positions.ctypes.data, len(positions),
        batch_ptr.ctypes.data, len(batch_ptr) - 1, cell.ctypes.data, pbc.ctypes.data,
        float(cutoff), int(half_list), int(include_self), _ALGORITHMS[algorithm], int(threads),
        ctypes.byref(handle), ctypes.byref(count), error, len(error))
    if status != 0:
        _raise(status, error)
    pairs = np.empty((count.value, 2), dtype=np.int64)
    shifts = np.empty((count.value, 3), dtype=np.int32)
    status = lib.tnr_ref_take(handle, pairs.ctypes.data, shifts.ctypes.data, error, len(error))
    if status != 0:
        _raise(status, error)
    return pairs, shifts


def port_neighbor_list(positions, cell, pbc, cutoff, batch_ptr=None, *, half_list=False,
                       include_self=False):
    """Plain-C restatement.  Returns (pairs (E,2) int64, shifts (E,3) int32)."""
    positions, cell, pbc, batch_ptr = _normalise(positions, cell, pbc, batch_ptr)
    lib = _load_port()
    pairs_ptr = ctypes.POINTER(ctypes.c_int64)()
    shifts_ptr = ctypes.POINTER(ctypes.c_int32)()
    count = ctypes.c_int64()
    error = ctypes.create_string_buffer(512)
    status = lib.oracle_neighbor_list(
        int(positions.dtype == np.float64), positions.ctypes.data, len(positions),
        batch_ptr.ctypes.data, len(batch_ptr) - 1, cell.ctypes.data, pbc.ctypes.data,
        float(cutoff), int(half_list), int(include_self), ctypes.byref(pairs_ptr),
        ctypes.byref(shifts_ptr), ctypes.byref(count), error, len(error))
    if status != 0:
        _raise(status, error)
    n = count.value
    try:
        if n == 0:
            return np.empty((0, 2), np.int64), np.empty((0, 3), np.int32)
        pairs = np.ctypeslib.as_array(pairs_ptr, shape=(n, 2)).copy()
        shifts = np.ctypeslib.as_array(shifts_ptr, shape=(n, 3)).copy()
        return pairs, shifts
    finally:
        lib.oracle_free_pairs(pairs_ptr, shifts_ptr)


def port_periodic_metadata(cells, pbc, counts, cutoff):
    """Restated geometry: duals (B,3,3) float64 and repeats (B,3) int64."""
    cells = np.ascontiguousarray(cells, dtype=np.float64)
    pbc = np.ascontiguousarray(pbc, dtype=np.uint8)
    counts = np.ascontiguousarray(counts, dtype=np.int64)
    batch = len(counts)
    duals = np.zeros((batch, 3, 3), np.float64)
    repeats = np.zeros((batch, 3), np.int64)
    error = ctypes.create_string_buffer(512)
    status = _load_port().oracle_periodic_metadata(
        cells.ctypes.data, pbc.ctypes.data, counts.ctypes.data, batch, float(cutoff),
        duals.ctypes.data, repeats.ctypes.data, error, len(error))
    if status != 0:
        _raise(status, error)
    return duals, repeats


def public_displacements(positions, cell, batch_ptr, pairs, shifts):
    """The reference frontend formula (src/tonari/_torch_frontend.py:94-104):
    D = pos[j] - pos[i] + S @ cell[batch(i)], evaluated in the input dtype."""
    positions = np.asarray(positions)
    cell = np.asarray(cell).reshape(-1, 3, 3)
    batch_ptr = np.asarray(batch_ptr, dtype=np.int64)
    source = pairs[:, 0]
    target = pairs[:, 1]
    pair_batch = np.searchsorted(batch_ptr[1:], source, side="right")
    translation = np.einsum("ei,eij->ej", shifts.astype(positions.dtype), cell[pair_batch])
    return positions[target] - positions[source] + translation


def canonical_rows(pairs, shifts):
    """(E,5) int64 rows (i, j, Sx, Sy, Sz) in lexicographic order."""
    rows = np.concatenate((np.asarray(pairs, np.int64), np.asarray(shifts, np.int64)), axis=1)
    if len(rows) == 0:
        return rows.reshape(0, 5)
    order = np.lexsort(tuple(rows[:, k] for k in range(4, -1, -1)))
    return rows[order]
