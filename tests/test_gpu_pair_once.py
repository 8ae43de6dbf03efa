"""Unsorted cell-list calls test each unordered pair once and write it in its
canonical orientation (half lists) or in both orientations (full lists).
These cases aim at the edges of that scheme: periodic self images (cells
shorter than the cutoff), include_self with a last write group of an odd
number of sources, and full-list outputs whose alignment forbids the
adjacent-row stores (edge_index with an odd pair count).  Every case is
compared with the reference CPU core (oracle/_ref); d/D at 1e-5 (float32)
and 1e-12 (float64) relative.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

from tests.support import assert_same_pairs, canonical, expected_pairs
from tests.test_gpu_differential import check_vectors
from tonari_b200 import neighbor_graph, neighbor_list

pytestmark = pytest.mark.gpu


def _structure(n_atoms, cell_rows, seed, dtype):
    generator = torch.Generator().manual_seed(seed)
    cell = torch.tensor(cell_rows, dtype=torch.float64)
    positions = torch.rand((n_atoms, 3), generator=generator, dtype=torch.float64) @ cell
    return positions.to(dtype), cell.to(dtype)[None], torch.tensor([[True, True, True]]), \
        torch.tensor([0, n_atoms])


def _check(out, quantities, positions, cell, pbc, cutoff, batch_ptr, half_list, include_self):
    values = dict(zip(quantities, out))
    pairs, shifts = values["P"], values["S"]
    assert_same_pairs(pairs, shifts, *expected_pairs(positions, cell, pbc, cutoff, batch_ptr,
                                                     half_list=half_list,
                                                     include_self=include_self))
    p, s = pairs.cpu().numpy(), shifts.cpu().numpy()
    check_vectors(positions.cpu().numpy(), cell.cpu().numpy(), batch_ptr.cpu().numpy(), p, s,
                  values["d"].cpu().numpy(), values["D"].cpu().numpy(), cutoff)
    assert torch.equal(values["i"], pairs[:, 0]) and torch.equal(values["j"], pairs[:, 1])
    return p, s, values["D"].cpu().numpy()


@pytest.mark.parametrize("dtype", [torch.float32, torch.float64])
@pytest.mark.parametrize("half_list", [False, True])
def test_include_self_with_odd_last_group(dtype, half_list):
    # 1,001 cell-list sources: the last write group holds 9, so the self rows
    # that close each group leave an odd row count.
    positions, cell, pbc, batch_ptr = _structure(
        1001, [[21.0, 0.0, 0.0], [1.5, 20.0, 0.0], [0.7, -1.1, 22.0]], 11, dtype)
    args = [t.cuda() for t in (positions, cell, pbc, batch_ptr)]
    quantities = "ijPSdD"
    out = neighbor_list(quantities, args[0], args[1], args[2], 4.5, args[3],
                        algorithm="cell_list", half_list=half_list, include_self=True)
    p, s, D = _check(out, quantities, positions, cell, pbc, 4.5, batch_ptr, half_list, True)
    if half_list:
        assert np.all(p[:, 0] <= p[:, 1])
    else:
        # Both orientations of every pair, with exactly negated displacements.
        rows = canonical(p, s)
        reverse = canonical(p[:, ::-1].copy(), -s)
        assert np.array_equal(rows, reverse)
        forward = {tuple(k): v for k, v in zip(np.concatenate((p, s), 1).tolist(), D)}
        for key, vector in list(forward.items())[:2000]:
            back = forward[(key[1], key[0], -key[2], -key[3], -key[4])]
            assert np.array_equal(back, -vector)  # signed zeros compare equal


@pytest.mark.parametrize("half_list", [False, True])
@pytest.mark.parametrize("include_self", [False, True])
def test_self_images_of_short_cells(half_list, include_self):
    # A 4 Å cell under a 5 Å cutoff: every atom sees its own periodic images,
    # and 60 atoms x 125 images sends the structure to the cell list.
    positions, cell, pbc, batch_ptr = _structure(
        60, [[4.0, 0.0, 0.0], [0.3, 4.2, 0.0], [-0.2, 0.4, 3.9]], 5, torch.float64)
    args = [t.cuda() for t in (positions, cell, pbc, batch_ptr)]
    quantities = "ijPSdD"
    out = neighbor_list(quantities, args[0], args[1], args[2], 5.0, args[3],
                        half_list=half_list, include_self=include_self)
    p, s, _ = _check(out, quantities, positions, cell, pbc, 5.0, batch_ptr, half_list,
                     include_self)
    self_images = (p[:, 0] == p[:, 1]) & np.any(s != 0, axis=1)
    assert self_images.any()


@pytest.mark.parametrize("dtype", [torch.float32, torch.float64])
def test_edge_index_with_odd_pair_count(dtype):
    # include_self on an odd atom count makes E odd, so the target row of the
    # (2, E) buffer is not 16-byte aligned and the full-list write pass uses
    # its unpaired row layout.
    positions, cell, pbc, batch_ptr = _structure(
        777, [[18.0, 0.0, 0.0], [0.0, 19.0, 0.0], [0.0, 0.0, 20.0]], 3, dtype)
    args = [t.cuda() for t in (positions, cell, pbc, batch_ptr)]
    edge_index, shifts, vectors = neighbor_graph(args[0], args[1], args[2], 4.0, args[3],
                                                 algorithm="cell_list", include_self=True)
    assert edge_index.shape[1] % 2 == 1
    assert_same_pairs(edge_index.T, shifts, *expected_pairs(positions, cell, pbc, 4.0, batch_ptr,
                                                            include_self=True))
    p, s = edge_index.T.cpu().numpy(), shifts.cpu().numpy()
    D = vectors.cpu().numpy()
    check_vectors(positions.numpy(), cell.numpy(), batch_ptr.numpy(), p, s,
                  np.linalg.norm(D.astype(np.float64), axis=1).astype(D.dtype), D, 4.0)
