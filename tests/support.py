"""Comparison helpers shared by the tests (restating the reference's
tests/support/assertions.py:10-41 key-set comparison)."""
from __future__ import annotations

import numpy as np
import torch


def to_numpy(x):
    if isinstance(x, torch.Tensor):
        return x.detach().cpu().numpy()
    return np.asarray(x)


def pair_keys(pairs, shifts) -> set[tuple[int, int, int, int, int]]:
    pairs = to_numpy(pairs)
    shifts = to_numpy(shifts)
    assert pairs.ndim == 2 and pairs.shape[1] == 2 and pairs.dtype == np.int64
    assert shifts.shape == (len(pairs), 3) and shifts.dtype == np.int32
    rows = np.concatenate((pairs, shifts.astype(np.int64)), axis=1).tolist()
    keys = {tuple(r) for r in rows}
    assert len(keys) == len(rows), "neighbor list contains duplicate pair identities"
    return keys


def canonical(pairs, shifts) -> np.ndarray:
    rows = np.concatenate((to_numpy(pairs).astype(np.int64), to_numpy(shifts).astype(np.int64)), axis=1)
    if len(rows) == 0:
        return rows.reshape(0, 5)
    order = np.lexsort(tuple(rows[:, k] for k in range(4, -1, -1)))
    return rows[order]


def assert_same_pairs(actual_pairs, actual_shifts, expected_pairs, expected_shifts):
    a = canonical(actual_pairs, actual_shifts)
    e = canonical(expected_pairs, expected_shifts)
    assert len(a) == len(e), f"pair count {len(a)} != expected {len(e)}"
    if not np.array_equal(a, e):
        bad = np.nonzero(np.any(a != e, axis=1))[0][:5]
        raise AssertionError(f"pair sets differ, first rows: actual {a[bad]} expected {e[bad]}")


def assert_sorted_by_source(pairs) -> None:
    source = to_numpy(pairs)[:, 0]
    assert np.all(source[1:] >= source[:-1])


def expected_pairs(positions, cell, pbc, cutoff, batch_ptr=None, *, half_list=False,
                   include_self=False):
    """(pairs, shifts) from the reference's own CPU core (oracle/_ref) when it
    was built, else from the plain-C restatement (oracle/_port)."""
    from oracle import oracle

    args = (to_numpy(positions), to_numpy(cell), to_numpy(pbc), cutoff,
            None if batch_ptr is None else to_numpy(batch_ptr))
    if oracle.ref_available():
        return oracle.ref_neighbor_list(*args, half_list=half_list, include_self=include_self)
    return oracle.port_neighbor_list(*args, half_list=half_list, include_self=include_self)
