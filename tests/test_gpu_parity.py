"""Parity of the sm_100a path against the CPU oracle.

Known-answer cases restate the reference's own tests (file:line cited per
test); randomized cases compare the exact (i, j, S) key set with the oracle:
the reference's CPU core (oracle/_ref) when it is built, else the plain-C
restatement (oracle/_port), which is itself pinned to the reference by
tests/test_oracle.py.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

from oracle import oracle
from tests.support import assert_same_pairs, assert_sorted_by_source, pair_keys
from tonari_b200 import neighbor_list

pytestmark = pytest.mark.gpu


def expected_pairs(positions, cell, pbc, cutoff, batch_ptr=None, *, half_list=False,
                   include_self=False):
    args = (to_np(positions), to_np(cell), to_np(pbc), cutoff,
            None if batch_ptr is None else to_np(batch_ptr))
    if oracle.ref_available():
        return oracle.ref_neighbor_list(*args, half_list=half_list, include_self=include_self)
    return oracle.port_neighbor_list(*args, half_list=half_list, include_self=include_self)


def to_np(x):
    return x.detach().cpu().numpy() if isinstance(x, torch.Tensor) else np.asarray(x)


def cuda(*tensors):
    return [t.cuda() if isinstance(t, torch.Tensor) else t for t in tensors]


def run(positions, cell, pbc, cutoff, batch_ptr=None, quantities="PS", **options):
    return neighbor_list(quantities, *cuda(positions, cell, pbc), cutoff,
                         None if batch_ptr is None else batch_ptr.cuda(), **options)


# --- known answers ----------------------------------------------------------

def test_strict_cutoff_and_periodic_self_images():
    # tests/backends/test_pair_identity.py:83-117
    positions = torch.tensor([[0.0, 0.0, 0.0], [1.0, 0.0, 0.0]])
    cell = torch.zeros((3, 3))
    pbc = torch.zeros(3, dtype=torch.bool)
    assert pair_keys(*run(positions, cell, pbc, 1.0)) == set()
    positions[1, 0] = torch.nextafter(torch.tensor(1.0), torch.tensor(0.0))
    assert pair_keys(*run(positions, cell, pbc, 1.0)) == {(0, 1, 0, 0, 0), (1, 0, 0, 0, 0)}
    periodic = run(torch.zeros((1, 3)), torch.diag(torch.tensor([0.4, 8.0, 8.0])),
                   torch.tensor([True, False, False]), 1.0)
    assert pair_keys(*periodic) == {(0, 0, -2, 0, 0), (0, 0, -1, 0, 0), (0, 0, 1, 0, 0),
                                    (0, 0, 2, 0, 0)}


def test_periodic_self_images_and_half_list():
    # tests/test_pair_options.py:187-203
    positions = torch.zeros((1, 3), dtype=torch.float64)
    cell = torch.diag(torch.tensor([0.4, 8.0, 8.0], dtype=torch.float64))
    pbc = torch.tensor([True, False, False])
    half = pair_keys(*run(positions, cell, pbc, 1.0, half_list=True))
    assert half == {(0, 0, -2, 0, 0), (0, 0, -1, 0, 0)}
    full_self = pair_keys(*run(positions, cell, pbc, 1.0, include_self=True))
    assert (0, 0, 0, 0, 0) in full_self and len(full_self) == 5


@pytest.mark.parametrize("half_list", [False, True])
def test_coincident_atoms_are_not_self_pairs(half_list):
    # tests/test_pair_options.py:206-226
    positions = torch.tensor([[0.0, 0.0, 0.0], [0.0, 0.0, 0.0], [1.0, 0.0, 0.0]])
    keys = pair_keys(*run(positions, torch.zeros((3, 3)), torch.zeros(3, dtype=torch.bool), 1.0,
                          half_list=half_list, include_self=True))
    expected = {(a, a, 0, 0, 0) for a in range(3)} | {(0, 1, 0, 0, 0)}
    if not half_list:
        expected.add((1, 0, 0, 0, 0))
    assert keys == expected


@pytest.mark.parametrize(("dtype", "cutoff"), [(torch.float32, 1e-30), (torch.float64, 1e-200)])
@pytest.mark.parametrize("half_list", [False, True])
def test_zero_shift_self_ignores_squared_cutoff_underflow(dtype, cutoff, half_list):
    # tests/test_pair_options.py:229-261
    keys = pair_keys(*run(torch.zeros((1, 3), dtype=dtype), torch.zeros((3, 3), dtype=dtype),
                          torch.zeros(3, dtype=torch.bool), cutoff, half_list=half_list,
                          include_self=True))
    assert keys == {(0, 0, 0, 0, 0)}


@pytest.mark.parametrize("n_atoms", [255, 256])
def test_float32_cutoff_rounding(n_atoms):
    # tests/backends/test_cuda_runtime.py:33-53
    cutoff = 353.2019167901003
    positions = torch.zeros((n_atoms, 3), dtype=torch.float32)
    positions[1, 0] = torch.tensor(353.2019, dtype=torch.float32)
    positions[2:, 1] = 1000 * torch.arange(2, n_atoms, dtype=torch.float32)
    keys = pair_keys(*run(positions, torch.zeros((3, 3)), torch.zeros(3, dtype=torch.bool), cutoff))
    assert keys == {(0, 1, 0, 0, 0), (1, 0, 0, 0, 0)}


def test_nondefault_stream_and_empty_batch_member():
    # tests/backends/test_cuda_runtime.py:56-69
    positions = torch.tensor([[0.0, 0.0, 0.0], [0.3, 0.0, 0.0]], device="cuda")
    batch_ptr = torch.tensor([0, 0, 2], device="cuda")
    cell = torch.zeros((2, 3, 3), device="cuda")
    pbc = torch.zeros((2, 3), dtype=torch.bool, device="cuda")
    stream = torch.cuda.Stream()
    with torch.cuda.stream(stream):
        positions = positions + 0.0
        pairs, shifts = neighbor_list("PS", positions, cell, pbc, 0.5, batch_ptr, sorted=True)
    torch.cuda.current_stream().wait_stream(stream)
    assert pair_keys(pairs, shifts) == {(0, 1, 0, 0, 0), (1, 0, 0, 0, 0)}
    assert_sorted_by_source(pairs)


def test_large_common_translation_uses_public_formula():
    # tests/backends/test_cuda_runtime.py:73-98
    cell = torch.tensor([[-0.9499396681785583, 2.3687520027160645, 1.7597240209579468],
                         [-3.4348089694976807, -1.8801195621490479, 1.9097744226455688],
                         [2.5219004154205322, -1.9322474002838135, 4.843184471130371]])
    positions = torch.tensor([-2138.380859375, -11887.5810546875, 10318.5625]).repeat(256, 1)
    positions[52] = torch.tensor([-2135.800048828125, -11886.6826171875, 10317.2880859375])
    positions[40] = torch.tensor([-2141.306396484375, -11885.267578125, 10315.8291015625])
    positions[61] = torch.tensor([-2135.84033203125, -11887.59375, 10317.1181640625])
    pbc = torch.ones(3, dtype=torch.bool)
    cutoff = 1.4481067657470703
    for algorithm in ("auto", "brute_force", "cell_list"):
        keys = pair_keys(*run(positions, cell, pbc, cutoff, algorithm=algorithm))
        assert (52, 23, 0, -1, 0) in keys and (23, 52, 0, 1, 0) in keys
        assert (61, 40, -1, -1, 1) not in keys and (40, 61, 1, 1, -1) not in keys
        assert_same_pairs(*run(positions, cell, pbc, cutoff, algorithm=algorithm),
                          *expected_pairs(positions, cell, pbc, cutoff))


def test_large_unwrapped_representatives_use_original_geometry():
    # tests/backends/test_pair_identity.py:312-337
    cell = torch.tensor([[-0.7647425305009836, -2.672179555955561, 2.8765648407042885],
                         [-1.0423290504477831, -3.665756214439444, -3.2514359787147056],
                         [5.609321251949969, -2.2087783511424566, -0.0013679155882546645]],
                        dtype=torch.float64)
    positions = torch.tensor([[598110346.0828383, -8096602.288435191, 242913231.3592053],
                              [598110345.1706604, -8096602.339372153, 242913230.9525894]],
                             dtype=torch.float64)
    keys = pair_keys(*run(positions, cell, torch.ones(3, dtype=torch.bool), 1.0))
    assert keys == {(0, 1, 0, 0, 0), (1, 0, 0, 0, 0)}


@pytest.mark.parametrize("dtype", [torch.float32, torch.float64])
def test_forced_cell_list_preserves_nextafter_inside_pair(dtype):
    # tests/backends/test_pair_identity.py:292-309
    positions = torch.zeros((256, 3), dtype=dtype)
    positions[1, 0] = torch.nextafter(torch.tensor(1.0, dtype=dtype), torch.tensor(0.0, dtype=dtype))
    positions[2:, 1] = 3 * torch.arange(2, 256, dtype=dtype)
    keys = pair_keys(*run(positions, torch.zeros((3, 3), dtype=dtype),
                          torch.zeros(3, dtype=torch.bool), 1.0, algorithm="cell_list"))
    assert keys == {(0, 1, 0, 0, 0), (1, 0, 0, 0, 0)}


# --- errors -----------------------------------------------------------------

@pytest.mark.parametrize("value", [float("nan"), float("inf")])
@pytest.mark.parametrize("n_atoms", [2, 256])
def test_rejects_nonfinite_positions(value, n_atoms):
    # tests/backends/test_native_errors.py:11-22; test_cuda_runtime.py:240-253
    positions = torch.zeros((n_atoms, 3), dtype=torch.float64)
    positions[:, 1] = 2 * torch.arange(n_atoms, dtype=torch.float64)
    positions[0, 0] = value
    with pytest.raises(RuntimeError, match="positions must"):
        run(positions, torch.zeros((3, 3), dtype=torch.float64), torch.zeros(3, dtype=torch.bool), 0.5)


def test_rejects_wrap_outside_int32():
    # tests/backends/test_native_errors.py:25-40
    positions = torch.tensor([[0.1, 0.0, 0.0], [2**31 + 0.2, 0.0, 0.0]], dtype=torch.float64)
    with pytest.raises(RuntimeError, match="wraps.*int32"):
        run(positions, torch.eye(3, dtype=torch.float64), torch.tensor([True, False, False]), 0.5)


def test_rejects_output_shift_outside_int32():
    # tests/backends/test_native_errors.py:43-58
    positions = torch.tensor([[-(2**31) + 0.1, 0.0, 0.0], [2**31 - 0.8, 0.0, 0.0]],
                             dtype=torch.float64)
    with pytest.raises(RuntimeError, match="cell shift.*int32"):
        run(positions, torch.eye(3, dtype=torch.float64), torch.tensor([True, False, False]), 0.5)


def test_rejects_dependent_rows_and_nonfinite_cell_and_image_count():
    # tests/backends/test_native_errors.py:61-125
    cell = torch.tensor([[1.0, 0.0, 0.0], [2.0, 0.0, 0.0], [0.0, 0.0, 4.0]], dtype=torch.float64)
    with pytest.raises(ValueError, match="linearly independent"):
        run(torch.zeros((1, 3), dtype=torch.float64), cell, torch.tensor([True, True, False]), 0.5)
    cell = torch.eye(3, dtype=torch.float64)
    cell[2, 0] = torch.nan
    with pytest.raises(ValueError, match="cell must contain only finite values"):
        run(torch.zeros((1, 3), dtype=torch.float64), cell, torch.tensor([True, True, False]), 0.5)
    with pytest.raises(ValueError, match="image count.*resource limit"):
        run(torch.zeros((1, 3), dtype=torch.float64), 0.001 * torch.eye(3, dtype=torch.float64),
            torch.ones(3, dtype=torch.bool), 1.0)


@pytest.mark.parametrize(("batch_ptr", "message"),
                         [((1, 1, 2), "start at zero"), ((0, 1, 1), "end at N_total"),
                          ((0, 2, 1, 2), "nondecreasing")])
def test_rejects_invalid_batch_ptr(batch_ptr, message):
    # tests/backends/test_cuda_runtime.py:256-275
    b = len(batch_ptr) - 1
    with pytest.raises(ValueError, match=message):
        run(torch.zeros((2, 3)), torch.zeros((b, 3, 3)), torch.zeros((b, 3), dtype=torch.bool), 1.0,
            torch.tensor(batch_ptr))


@pytest.mark.parametrize(("edit", "message"),
                         [("first", "start at zero"), ("last", "end at N_total"),
                          ("order", "nondecreasing")])
def test_rejects_invalid_batch_ptr_speculative_batch(edit, message):
    # 64 float32 structures take the device geometry, whose kernels are queued
    # before the host has read batch_ptr; the errors and their order are the
    # reference's all the same (tests/backends/test_cuda_runtime.py:256-275).
    b = 64
    batch_ptr = torch.arange(0, 2 * b + 1, 2)
    if edit == "first":
        batch_ptr[0] = 1
    elif edit == "last":
        batch_ptr[-1] = 2 * b - 1
    else:
        batch_ptr[5], batch_ptr[6] = 12, 9
    cell = 10.0 * torch.eye(3).expand(b, 3, 3).contiguous()
    with pytest.raises(ValueError, match=message):
        run(torch.rand((2 * b, 3)), cell, torch.ones((b, 3), dtype=torch.bool), 1.0, batch_ptr)
    # The stream stays usable: a valid call right after.
    batch_ptr = torch.arange(0, 2 * b + 1, 2)
    pairs, _ = run(torch.rand((2 * b, 3)), cell, torch.ones((b, 3), dtype=torch.bool), 1.0, batch_ptr)
    assert pairs.shape[1] == 2


def test_sparse_layout_auto_and_forced():
    # tests/backends/test_algorithms.py:161-174; test_cuda_runtime.py:278-288
    positions = torch.zeros((256, 3))
    positions[:, 0] = torch.arange(256) * 10000.0
    args = (positions, torch.zeros((3, 3)), torch.zeros(3, dtype=torch.bool), 1.0)
    assert pair_keys(*run(*args)) == set()
    with pytest.raises(RuntimeError, match="cell_list cannot safely"):
        run(*args, algorithm="cell_list")


def test_empty_periodic_structure():
    # tests/backends/test_pair_identity.py:254-265
    pairs, shifts = run(torch.empty((0, 3), dtype=torch.float64),
                        1e-12 * torch.eye(3, dtype=torch.float64)[None],
                        torch.ones((1, 3), dtype=torch.bool), 1.0, torch.tensor([0, 0]))
    assert pairs.shape == (0, 2) and shifts.shape == (0, 3)


# --- golden fixtures (made from the reference's own Torch oracle) -----------

from pathlib import Path  # noqa: E402

GOLDEN = sorted((Path(__file__).parent / "golden").glob("*.npz"))


@pytest.mark.parametrize("path", GOLDEN, ids=[p.stem for p in GOLDEN])
@pytest.mark.parametrize("algorithm", ["auto", "brute_force", "cell_list"])
def test_golden_fixtures(path, algorithm):
    g = np.load(path)
    args = [torch.from_numpy(g[k]) for k in ("positions", "cell", "pbc")]
    try:
        pairs, shifts = run(*args, float(g["cutoff"]), torch.from_numpy(g["batch_ptr"]),
                            algorithm=algorithm, half_list=bool(g["half_list"]),
                            include_self=bool(g["include_self"]), sorted=True)
    except RuntimeError as error:
        assert algorithm == "cell_list" and "cannot safely" in str(error)
        return
    from tests.support import canonical

    assert np.array_equal(canonical(pairs, shifts), g["rows"])
    assert_sorted_by_source(pairs)
