"""ctypes view of the C ABI in include/tonari_b200.h (for tests and tools
that call the library without the PyTorch op)."""
from __future__ import annotations

import ctypes
from functools import lru_cache

from ._extensions import CORE_LIBRARY

QUANTITY_BITS = {"i": 1, "j": 2, "P": 4, "S": 8, "d": 16, "D": 32}
ALGORITHMS = {"auto": 0, "brute_force": 1, "cell_list": 2}
STATUS = {0: "TNR_OK", 1: "TNR_INPUT_ERROR", 2: "TNR_SEARCH_ERROR", 3: "TNR_CUDA_ERROR",
          4: "TNR_ALLOC_ERROR"}


class Request(ctypes.Structure):
    _fields_ = [
        ("dtype", ctypes.c_int32), ("n_atoms", ctypes.c_int64), ("n_structures", ctypes.c_int64),
        ("positions", ctypes.c_void_p), ("batch_ptr", ctypes.c_void_p), ("cell", ctypes.c_void_p),
        ("pbc", ctypes.c_void_p), ("batch_ptr_host", ctypes.c_void_p),
        ("cell_host", ctypes.c_void_p), ("pbc_host", ctypes.c_void_p),
        ("cutoff", ctypes.c_double), ("half_list", ctypes.c_int32),
        ("include_self", ctypes.c_int32), ("algorithm", ctypes.c_int32),
        ("quantities", ctypes.c_uint32), ("index_offset", ctypes.c_int64),
        ("sorted", ctypes.c_int32),
    ]


class Result(ctypes.Structure):
    _fields_ = [("n_pairs", ctypes.c_int64)] + [
        (name, ctypes.c_void_p) for name in ("i", "j", "P", "S", "d", "D", "edge_index")]


EXPORTED = ("tnr_neighbor_list", "tnr_neighbor_list_static", "tnr_version",
            "tnr_last_launch_count", "tnr_last_phase_times", "tnr_last_host_times",
            "tnr_filter_pairs")


@lru_cache
def library():
    lib = ctypes.CDLL(str(CORE_LIBRARY))
    lib.tnr_neighbor_list.restype = ctypes.c_int
    lib.tnr_neighbor_list.argtypes = [ctypes.POINTER(Request), ctypes.c_void_p, ctypes.c_void_p,
                                      ctypes.POINTER(Result), ctypes.c_char_p, ctypes.c_size_t]
    lib.tnr_neighbor_list_static.restype = ctypes.c_int
    lib.tnr_neighbor_list_static.argtypes = [ctypes.POINTER(Request), ctypes.c_void_p,
                                             ctypes.c_int64, ctypes.POINTER(Result),
                                             ctypes.c_char_p, ctypes.c_size_t]
    lib.tnr_version.restype = ctypes.c_char_p
    lib.tnr_last_launch_count.restype = ctypes.c_int64
    return lib


def quantity_mask(quantities: str) -> int:
    mask = 0
    for q in quantities:
        mask |= QUANTITY_BITS[q]
    return mask
