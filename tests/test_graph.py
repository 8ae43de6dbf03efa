"""The (2, E) edge_index adapter (tonari docs/design.md:61 asks adapters for
edge_index = P.T.contiguous(); here the write pass emits that layout)."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from tests.support import canonical, expected_pairs
from tonari_b200 import neighbor_graph, neighbor_list


def _batch(device, dtype=torch.float64):
    generator = torch.Generator().manual_seed(77)
    cell = torch.tensor([[[6.0, 0.0, 0.0], [0.5, 6.5, 0.0], [0.2, 0.3, 7.0]],
                         [[9.0, 0.0, 0.0], [0.0, 8.0, 0.0], [0.0, 0.0, 8.5]]], dtype=dtype)
    counts = (40, 300)
    positions = torch.cat([torch.rand((c, 3), generator=generator, dtype=dtype) @ cell[k]
                           for k, c in enumerate(counts)])
    pbc = torch.tensor([[True, True, True], [True, False, True]])
    batch_ptr = torch.tensor([0, counts[0], sum(counts)])
    return [t.to(device) for t in (positions, cell, pbc, batch_ptr)]


def test_cpu_tensors_are_rejected():
    positions, cell, pbc, batch_ptr = _batch("cpu")
    with pytest.raises(RuntimeError, match="CUDA provider only"):
        neighbor_graph(positions, cell, pbc, 3.0, batch_ptr)


def test_options_are_validated():
    positions, cell, pbc, batch_ptr = _batch("cpu")
    with pytest.raises(ValueError, match="algorithm must be"):
        neighbor_graph(positions, cell, pbc, 3.0, batch_ptr, algorithm="fast")
    with pytest.raises(ValueError, match="cutoff must be finite and positive"):
        neighbor_graph(positions, cell, pbc, -1.0, batch_ptr)


@pytest.mark.gpu
@pytest.mark.parametrize("dtype", [torch.float32, torch.float64])
@pytest.mark.parametrize("half_list", [False, True])
def test_edge_index_matches_neighbor_list(dtype, half_list):
    positions, cell, pbc, batch_ptr = _batch("cuda", dtype)
    edge_index, shifts, vectors = neighbor_graph(positions, cell, pbc, 3.0, batch_ptr,
                                                 half_list=half_list)
    assert edge_index.shape[0] == 2 and edge_index.is_contiguous() and edge_index.dtype == torch.int64
    pairs, ref_shifts, ref_D = neighbor_list("PSD", positions, cell, pbc, 3.0, batch_ptr,
                                             half_list=half_list)
    rows = canonical(edge_index.T, shifts)
    ref_rows = canonical(pairs, ref_shifts)
    assert np.array_equal(rows, ref_rows)
    oracle_rows = canonical(*expected_pairs(positions, cell, pbc, 3.0, batch_ptr,
                                            half_list=half_list))
    assert np.array_equal(rows, oracle_rows)
    key = lambda p, s: np.lexsort(tuple(np.concatenate((p, s), 1)[:, k] for k in range(4, -1, -1)))
    order = key(edge_index.T.cpu().numpy(), shifts.cpu().numpy().astype(np.int64))
    ref_order = key(pairs.cpu().numpy(), ref_shifts.cpu().numpy().astype(np.int64))
    assert torch.equal(vectors.cpu()[order], ref_D.cpu()[ref_order])
    bare = neighbor_graph(positions, cell, pbc, 3.0, batch_ptr, half_list=half_list,
                          edge_vectors=False)
    assert bare[2] is None and bare[0].shape == edge_index.shape


@pytest.mark.gpu
def test_edge_vector_gradients_match_neighbor_list():
    positions, cell, pbc, batch_ptr = _batch("cuda")
    grads = []
    for use_graph in (True, False):
        p = positions.clone().requires_grad_(True)
        c = cell.clone().requires_grad_(True)
        if use_graph:
            vectors = neighbor_graph(p, c, pbc, 3.0, batch_ptr)[2]
        else:
            (vectors,) = neighbor_list("D", p, c, pbc, 3.0, batch_ptr)
        (vectors.pow(2).sum(1).sqrt()).sum().backward()
        grads.append((p.grad, c.grad))
    torch.testing.assert_close(grads[0][0], grads[1][0], rtol=1e-12, atol=1e-12)
    torch.testing.assert_close(grads[0][1], grads[1][1], rtol=1e-12, atol=1e-12)
