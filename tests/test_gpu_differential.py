"""Randomized differential parity and output-contract tests on the GPU.

Cases follow the reference's randomized tests (tests/backends/
test_pair_identity.py:189-223, tests/backends/test_algorithms.py:11-76,
tests/test_pair_options.py:157-184, 324-394) and the benchmark configurations
at reduced sizes.  d/D tolerances: 1e-5 relative (float32), 1e-12 (float64).
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import oracle
from tests.support import assert_same_pairs, assert_sorted_by_source, canonical
from tests.test_gpu_parity import expected_pairs, run
from tonari_b200 import neighbor_list, workloads

pytestmark = pytest.mark.gpu

TOLERANCE = {torch.float32: 1e-5, torch.float64: 1e-12, np.float32: 1e-5, np.float64: 1e-12}


def check_vectors(positions, cell, batch_ptr, pairs, shifts, d, D, cutoff):
    """d/D against the reference frontend formula evaluated on the same pairs."""
    positions = np.asarray(positions)
    tol = TOLERANCE[positions.dtype.type]
    ref_D = oracle.public_displacements(positions, cell, batch_ptr, pairs, shifts)
    ref_d = np.linalg.norm(ref_D.astype(np.float64), axis=1)
    scale = np.maximum(np.linalg.norm(ref_D.astype(np.float64), axis=1), cutoff * 1e-3)
    assert np.all(np.linalg.norm(D.astype(np.float64) - ref_D, axis=1) <= tol * scale * 4)
    assert np.all(np.abs(d.astype(np.float64) - ref_d) <= tol * np.maximum(ref_d, cutoff * 1e-3) * 4)


@pytest.mark.parametrize("algorithm", ["auto", "brute_force", "cell_list"])
def test_randomized_differential(algorithm):
    generator = torch.Generator().manual_seed(29381)
    patterns = torch.tensor([[False, False, False], [True, False, False], [True, False, True],
                             [True, True, False], [True, True, True]])
    for case in range(30):
        n_atoms = case + 1
        cell = torch.diag(1.8 + 2.5 * torch.rand(3, generator=generator))
        cell += 0.35 * torch.tril(torch.rand((3, 3), generator=generator), diagonal=-1)
        positions = torch.rand((n_atoms, 3), generator=generator) @ cell
        pbc = patterns[case % len(patterns)]
        if case % 4 == 0:
            positions[0] += 3 * cell[0]
            if pbc[2]:
                positions[-1] -= 2 * cell[2]
        cutoff = 0.55 + 0.8 * float(torch.rand((), generator=generator))
        try:
            actual = run(positions, cell, pbc, cutoff, algorithm=algorithm)
        except RuntimeError as error:
            assert algorithm == "cell_list" and "cannot safely" in str(error)
            continue
        assert_same_pairs(*actual, *expected_pairs(positions, cell, pbc, cutoff))


def periodic_batch(dtype=torch.float64):
    generator = torch.Generator().manual_seed(1945)
    counts = (32, 288)
    cell = torch.tensor([[[5.0, 0.0, 0.0], [0.0, 5.5, 0.0], [0.0, 0.0, 6.0]],
                         [[8.0, 0.0, 0.0], [0.0, 7.5, 0.0], [0.0, 0.0, 9.0]]], dtype=dtype)
    positions = torch.cat([(0.1 + 0.8 * torch.rand((c, 3), generator=generator, dtype=dtype))
                           @ cell[k] for k, c in enumerate(counts)])
    pbc = torch.tensor([[True, False, False], [True, False, False]])
    return positions, cell, pbc, torch.tensor([0, counts[0], sum(counts)])


@pytest.mark.parametrize("algorithm", ["auto", "brute_force", "cell_list"])
@pytest.mark.parametrize("half_list", [False, True])
@pytest.mark.parametrize("include_self", [False, True])
def test_periodic_batch_pair_options(algorithm, half_list, include_self):
    # tests/backends/test_algorithms.py:131-158
    positions, cell, pbc, batch_ptr = periodic_batch()
    pairs, shifts = run(positions, cell, pbc, 1.2, batch_ptr, algorithm=algorithm, sorted=True,
                        half_list=half_list, include_self=include_self)
    assert_sorted_by_source(pairs)
    assert_same_pairs(pairs, shifts, *expected_pairs(positions, cell, pbc, 1.2, batch_ptr,
                                                     half_list=half_list,
                                                     include_self=include_self))


@pytest.mark.parametrize("dtype", [torch.float32, torch.float64])
@pytest.mark.parametrize("shift_atoms", [False, True])
def test_forced_cell_list_triclinic(dtype, shift_atoms):
    # tests/backends/test_pair_identity.py:268-289 and test_cuda_runtime.py:136-151
    generator = torch.Generator().manual_seed(1842)
    cell = torch.tensor([[8.0, 0.4, 0.1], [0.2, 7.5, 0.5], [0.3, 0.1, 9.0]], dtype=dtype)
    positions = torch.rand((288, 3), generator=generator, dtype=dtype) @ cell
    if shift_atoms:
        positions[:5] += 3 * cell[0] - 2 * cell[1]
    pbc = torch.ones(3, dtype=torch.bool)
    for algorithm in ("auto", "cell_list"):
        assert_same_pairs(*run(positions, cell, pbc, 1.2, algorithm=algorithm),
                          *expected_pairs(positions, cell, pbc, 1.2))


def test_mixed_finite_and_partial_pbc_batch():
    # tests/backends/test_cuda_runtime.py:154-193
    generator = torch.Generator().manual_seed(5801)
    counts = (256, 257)
    cell = torch.tensor([[[0.0] * 3] * 3, [[2.1, 0.3, 0.2], [0.4, 4.0, 0.1], [0.2, 0.5, 5.0]]],
                        dtype=torch.float64)
    positions = torch.cat((torch.rand((counts[0], 3), generator=generator, dtype=torch.float64) * 8,
                           torch.rand((counts[1], 3), generator=generator, dtype=torch.float64)
                           @ cell[1]))
    positions[-3:] += 4 * cell[1, 0]
    batch_ptr = torch.tensor([0, counts[0], sum(counts)])
    pbc = torch.tensor([[False, False, False], [True, False, False]])
    for algorithm in ("auto", "brute_force", "cell_list"):
        assert_same_pairs(*run(positions, cell, pbc, 0.55, batch_ptr, algorithm=algorithm),
                          *expected_pairs(positions, cell, pbc, 0.55, batch_ptr))


@pytest.mark.parametrize("dtype", [torch.float32, torch.float64])
def test_quantities_order_layout_and_values(dtype):
    # tests/test_quantities.py:10-35, 120-151
    positions, cell, pbc, batch_ptr = periodic_batch(dtype)
    out = run(positions, cell, pbc, 1.2, batch_ptr, quantities="jiPSdDi", sorted=True)
    target, source, pairs, shifts, d, D, source_again = out
    assert pairs.dtype == source.dtype == target.dtype == torch.int64
    assert shifts.dtype == torch.int32 and d.dtype == D.dtype == dtype
    assert torch.equal(source, pairs[:, 0]) and torch.equal(target, pairs[:, 1])
    assert torch.equal(source_again, source)
    p, s = pairs.cpu().numpy(), shifts.cpu().numpy()
    check_vectors(positions.numpy(), cell.numpy(), batch_ptr.numpy(), p, s, d.cpu().numpy(),
                  D.cpu().numpy(), 1.2)
    assert neighbor_list("", *[t.cuda() for t in (positions, cell, pbc)], 1.2, batch_ptr.cuda()) == ()


def test_autograd_through_distances_and_displacements():
    # tests/test_quantities.py:97-117; tests/backends/test_pair_identity.py:226-251
    positions = torch.tensor([[0.1, 0.0, 0.0], [1.8, 0.2, 0.0]], device="cuda",
                             dtype=torch.float64, requires_grad=True)
    cell = torch.tensor([[2.0, 0.0, 0.0], [0.1, 2.5, 0.0], [0.0, 0.0, 3.0]], device="cuda",
                        dtype=torch.float64, requires_grad=True)
    pbc = torch.ones(3, device="cuda", dtype=torch.bool)
    d, D, pairs = neighbor_list("dDP", positions, cell, pbc, 0.8)
    (d.sum() + D.square().sum()).backward()
    assert pairs.grad_fn is None
    assert positions.grad is not None and torch.all(torch.isfinite(positions.grad))
    assert cell.grad is not None and torch.count_nonzero(cell.grad) > 0


@pytest.mark.parametrize("name", ["cfg1", "cfg2", "cfg3"])
def test_benchmark_configs_match_oracle(name):
    w = workloads.CONFIGS[name]()
    if name != "cfg1":
        w = w.shard(0, 128)
    positions, cell, pbc, batch_ptr = w.torch_inputs("cuda")
    out = neighbor_list(w.quantities + "PS", positions, cell, pbc, w.cutoff, batch_ptr,
                        algorithm=w.options.get("algorithm", "auto"),
                        sorted=w.options.get("sorted", False),
                        half_list=w.options.get("half_list", False))
    pairs, shifts = out[-2], out[-1]
    if w.options.get("sorted", False):
        assert_sorted_by_source(pairs)
    assert_same_pairs(pairs, shifts, *expected_pairs(w.positions, w.cell, w.pbc, w.cutoff,
                                                     w.batch_ptr,
                                                     half_list=w.options.get("half_list", False)))
    values = dict(zip(w.quantities, out[:-2]))
    if "d" in values or "D" in values:
        p, s = pairs.cpu().numpy(), shifts.cpu().numpy()
        D = values["D"].cpu().numpy() if "D" in values else oracle.public_displacements(
            w.positions, w.cell, w.batch_ptr, p, s)
        d = values["d"].cpu().numpy() if "d" in values else np.linalg.norm(D, axis=1)
        check_vectors(w.positions, w.cell, w.batch_ptr, p, s, d, D, w.cutoff)


def test_cfg5_shard_half_list_matches_oracle():
    w = workloads.config5(n_structures=96)
    positions, cell, pbc, batch_ptr = w.torch_inputs("cuda")
    pairs, shifts = neighbor_list("PS", positions, cell, pbc, w.cutoff, batch_ptr, half_list=True)
    assert_same_pairs(pairs, shifts, *expected_pairs(w.positions, w.cell, w.pbc, w.cutoff,
                                                     w.batch_ptr, half_list=True))


def test_cfg4_reduced_cell_list_matches_oracle():
    w = workloads.config4(n_atoms=40_000)
    positions, cell, pbc, batch_ptr = w.torch_inputs("cuda")
    i, j, S, d, D = neighbor_list("ijSdD", positions, cell, pbc, w.cutoff, batch_ptr,
                                  algorithm="cell_list")
    pairs = torch.stack((i, j), dim=1)
    assert_same_pairs(pairs, S, *expected_pairs(w.positions, w.cell, w.pbc, w.cutoff, w.batch_ptr))
    check_vectors(w.positions, w.cell, w.batch_ptr, pairs.cpu().numpy(), S.cpu().numpy(),
                  d.cpu().numpy(), D.cpu().numpy(), w.cutoff)


@pytest.mark.parametrize("half_list", [False, True])
def test_sorted_and_unsorted_orders_hold_the_same_pairs(half_list):
    w = workloads.config4(n_atoms=30_000)
    positions, cell, pbc, batch_ptr = w.torch_inputs("cuda")
    unsorted = neighbor_list("PSdD", positions, cell, pbc, w.cutoff, batch_ptr,
                             half_list=half_list)
    ordered = neighbor_list("PSdD", positions, cell, pbc, w.cutoff, batch_ptr, sorted=True,
                            half_list=half_list)
    assert_sorted_by_source(ordered[0])
    assert_same_pairs(unsorted[0], unsorted[1], ordered[0], ordered[1])
    a = canonical(unsorted[0], unsorted[1])
    assert len(a) > 0


@pytest.mark.parametrize("dtype", [torch.float64, torch.float32])
def test_fused_displacement_gradients_match_reference_formula(dtype):
    # The backward of the fused d/D equals autograd through the reference
    # formula (src/tonari/_torch_frontend.py:94-104) on the same pairs.
    positions, cell, pbc, batch_ptr = periodic_batch(dtype)
    pos_a = positions.cuda().requires_grad_()
    cell_a = cell.cuda().requires_grad_()
    d, D, pairs, shifts = neighbor_list("dDPS", pos_a, cell_a, pbc.cuda(), 1.2, batch_ptr.cuda())
    weights = torch.linspace(0.5, 1.5, len(d), device="cuda", dtype=dtype)
    ((weights * d).sum() + (D ** 2).sum()).backward()
    pos_b = positions.cuda().requires_grad_()
    cell_b = cell.cuda().requires_grad_()
    pair_batch = torch.bucketize(pairs[:, 0].contiguous(), batch_ptr.cuda()[1:], right=True)
    D_ref = pos_b[pairs[:, 1]] - pos_b[pairs[:, 0]] + torch.einsum(
        "ei,eij->ej", shifts.to(dtype), cell_b[pair_batch])
    d_ref = torch.linalg.vector_norm(D_ref, dim=1)
    ((weights * d_ref).sum() + (D_ref ** 2).sum()).backward()
    tol = 1e-4 if dtype == torch.float32 else 1e-10
    torch.testing.assert_close(pos_a.grad, pos_b.grad, rtol=tol, atol=tol)
    torch.testing.assert_close(cell_a.grad, cell_b.grad, rtol=tol, atol=tol)


@pytest.mark.parametrize("dtype", [torch.float32, torch.float64])
@pytest.mark.parametrize("half_list", [False, True])
@pytest.mark.parametrize("sorted_output", [False, True])
def test_cell_list_small_cells_own_images(dtype, half_list, sorted_output):
    # Cells shorter than the cutoff: atoms pair with their own periodic
    # images, which half lists keep by the canonical shift rule
    # (tests/backends/test_pair_identity.py:13-81 for the rule).
    generator = torch.Generator().manual_seed(7021)
    cells, blocks, counts = [], [], (40, 3, 65)
    for k, n in enumerate(counts):
        cell = torch.diag(2.6 + 1.2 * torch.rand(3, generator=generator, dtype=dtype))
        cell += 0.4 * torch.tril(torch.rand((3, 3), generator=generator, dtype=dtype), diagonal=-1)
        cells.append(cell)
        blocks.append(torch.rand((n, 3), generator=generator, dtype=dtype) @ cell)
    positions = torch.cat(blocks)
    cell = torch.stack(cells)
    pbc = torch.tensor([[True, True, True], [True, False, True], [True, True, True]])
    batch_ptr = torch.tensor([0, counts[0], counts[0] + counts[1], sum(counts)])
    pairs, shifts, D = run(positions, cell, pbc, 4.0, batch_ptr, quantities="PSD",
                           algorithm="cell_list", half_list=half_list, sorted=sorted_output)
    if sorted_output:
        assert_sorted_by_source(pairs)
    assert_same_pairs(pairs, shifts, *expected_pairs(positions, cell, pbc, 4.0, batch_ptr,
                                                     half_list=half_list))
    P, S = pairs.cpu().numpy(), shifts.cpu().numpy()
    ref_D = oracle.public_displacements(positions.numpy(), cell.numpy(), batch_ptr.numpy(), P, S)
    scale = np.maximum(np.linalg.norm(ref_D.astype(np.float64), axis=1), 4e-3)
    err = np.linalg.norm(D.cpu().numpy().astype(np.float64) - ref_D, axis=1)
    assert np.all(err <= TOLERANCE[dtype] * scale * 4)
