"""Parity at the benchmarked sizes: the exact inputs bench.py times.

Each test runs the public ``neighbor_list`` on the full configuration on the
GPU and compares the (i, j, S) set with the reference's own CPU core
(oracle/_ref, ``csrc/core/neighbors_cpu.cpp:976-1030``) bit for bit, and d/D
with the reference frontend formula (``src/tonari/_torch_frontend.py:94-104``)
evaluated on the same pairs: 1e-5 relative for float32, with a floor of
1e-3·cutoff on the norm.  Large pair sets are compared as sorted 64-bit packed
keys, per chunk of structures where the batch has several, to bound host
memory.  The lattice-shifted variant of cfg4 moves atoms by whole lattice
vectors, as ``tests/backends/test_cuda_runtime.py:73-87`` does, so the wraps
are nonzero at L = 215 Å.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import oracle
from tonari_b200 import neighbor_list, workloads

pytestmark = pytest.mark.gpu

F32_TOLERANCE = 1e-5


def packed_keys(pairs: np.ndarray, shifts: np.ndarray, index_bits: int, shift_bits: int,
                shift_bias: int) -> np.ndarray:
    """Sorted uint64 keys (i, j, Sx, Sy, Sz) -> one word; order-free set form."""
    key = pairs[:, 0].astype(np.uint64) << np.uint64(index_bits + 3 * shift_bits)
    key |= pairs[:, 1].astype(np.uint64) << np.uint64(3 * shift_bits)
    for axis in range(3):
        part = (shifts[:, axis].astype(np.int64) + shift_bias).astype(np.uint64)
        key |= part << np.uint64((2 - axis) * shift_bits)
    key.sort()
    return key


def assert_same_set(actual, expected, n_atoms: int) -> None:
    (pa, sa), (pe, se) = actual, expected
    assert len(pa) == len(pe), f"pair count {len(pa)} != reference {len(pe)}"
    if len(pa) == 0:
        return
    reach = int(max(np.abs(sa).max(), np.abs(se).max()))
    shift_bits = max(int(reach * 2 + 1).bit_length(), 1)
    index_bits = max(int(n_atoms - 1).bit_length(), 1)
    assert 2 * index_bits + 3 * shift_bits <= 64, "keys do not fit one word"
    ka = packed_keys(pa, sa, index_bits, shift_bits, reach)
    ke = packed_keys(pe, se, index_bits, shift_bits, reach)
    if not np.array_equal(ka, ke):
        differ = np.setxor1d(ka, ke)[:5]
        raise AssertionError(f"pair sets differ in {differ.size}+ keys, e.g. {differ}")


def check_vectors_chunked(positions, cell, batch_ptr, pairs, shifts, d, D, cutoff,
                          chunk: int = 8_000_000) -> None:
    for begin in range(0, len(pairs), chunk):
        end = min(begin + chunk, len(pairs))
        ref_D = oracle.public_displacements(positions, cell, batch_ptr, pairs[begin:end],
                                            shifts[begin:end]).astype(np.float64)
        norm = np.linalg.norm(ref_D, axis=1)
        floor = np.maximum(norm, cutoff * 1e-3)
        if D is not None:
            error = np.linalg.norm(D[begin:end].astype(np.float64) - ref_D, axis=1)
            assert np.all(error <= F32_TOLERANCE * floor), f"D error {error.max()}"
        if d is not None:
            error = np.abs(d[begin:end].astype(np.float64) - norm)
            assert np.all(error <= F32_TOLERANCE * floor), f"d error {error.max()}"


def reference(w: workloads.Workload, positions=None, **options):
    return oracle.ref_neighbor_list(w.positions if positions is None else positions, w.cell,
                                    w.pbc, w.cutoff, w.batch_ptr, **options)


def require_reference():
    if not oracle.ref_available():
        pytest.skip("oracle/_ref (the reference CPU core) was not built")


@pytest.mark.parametrize("shifted", [False, True], ids=["plain", "lattice_shifted"])
def test_cfg4_full_size(shifted):
    require_reference()
    w = workloads.config4()
    positions = w.positions
    if shifted:
        rng = np.random.default_rng(404)
        moved = rng.random(w.n_atoms) < 0.1
        offsets = rng.integers(-3, 4, (int(moved.sum()), 3)).astype(np.float32)
        positions = positions.copy()
        positions[moved] += offsets @ w.cell[0]
    device_inputs = [torch.from_numpy(x).cuda() for x in (positions, w.cell, w.pbc, w.batch_ptr)]
    i, j, S, d, D = neighbor_list("ijSdD", *device_inputs[:3], w.cutoff, device_inputs[3],
                                  algorithm="cell_list")
    pairs = torch.stack((i, j), dim=1).cpu().numpy()
    shifts = S.cpu().numpy()
    del i, j
    expected = reference(w, positions, algorithm="cell_list")
    assert_same_set((pairs, shifts), expected, w.n_atoms)
    del expected
    check_vectors_chunked(positions, w.cell, w.batch_ptr, pairs, shifts, d.cpu().numpy(),
                          D.cpu().numpy(), w.cutoff)


def structure_chunks(batch_ptr: np.ndarray, n_chunks: int):
    n = len(batch_ptr) - 1
    edges = np.linspace(0, n, n_chunks + 1).astype(int)
    return [(int(a), int(b)) for a, b in zip(edges[:-1], edges[1:]) if b > a]


def compare_batch_by_chunks(w, pairs, shifts, n_chunks, **options):
    """The whole batch ran on the GPU in one call; compare per chunk of
    structures (pairs never cross structures), each chunk against the
    reference run on that chunk alone with its indices rebased."""
    source = pairs[:, 0]
    order = np.argsort(source, kind="stable")
    source_sorted = source[order]
    for begin, end in structure_chunks(w.batch_ptr, n_chunks):
        a0, a1 = int(w.batch_ptr[begin]), int(w.batch_ptr[end])
        lo, hi = np.searchsorted(source_sorted, [a0, a1])
        rows = order[lo:hi]
        part = w.shard(begin, end)
        exp_pairs, exp_shifts = reference(part, **options)
        assert_same_set((pairs[rows] - a0, shifts[rows]), (exp_pairs, exp_shifts),
                        part.n_atoms)


def test_cfg5_full_size():
    require_reference()
    w = workloads.config5()
    positions, cell, pbc, batch_ptr = w.torch_inputs("cuda")
    P, S = neighbor_list("PS", positions, cell, pbc, w.cutoff, batch_ptr, half_list=True)
    pairs, shifts = P.cpu().numpy(), S.cpu().numpy()
    del P, S
    assert len(pairs) == 187_188_112
    compare_batch_by_chunks(w, pairs, shifts, 16, half_list=True)


def test_cfg2_full_size():
    require_reference()
    w = workloads.config2()
    positions, cell, pbc, batch_ptr = w.torch_inputs("cuda")
    P, S, D = neighbor_list("PSD", positions, cell, pbc, w.cutoff, batch_ptr)
    pairs, shifts = P.cpu().numpy(), S.cpu().numpy()
    assert_same_set((pairs, shifts), reference(w), w.n_atoms)
    check_vectors_chunked(w.positions, w.cell, w.batch_ptr, pairs, shifts, None,
                          D.cpu().numpy(), w.cutoff)


def test_cfg3_full_size_sorted():
    require_reference()
    w = workloads.config3()
    positions, cell, pbc, batch_ptr = w.torch_inputs("cuda")
    P, D = neighbor_list("PD", positions, cell, pbc, w.cutoff, batch_ptr, sorted=True)
    pairs = P.cpu().numpy()
    assert np.all(np.diff(pairs[:, 0]) >= 0), "sorted=True must give source-major order"
    shifts = np.zeros((len(pairs), 3), np.int32)  # non-periodic: every shift is zero
    expected = reference(w)
    assert not np.any(expected[1])
    assert_same_set((pairs, shifts), expected, w.n_atoms)
    check_vectors_chunked(w.positions, w.cell, w.batch_ptr, pairs, shifts, None,
                          D.cpu().numpy(), w.cutoff)
