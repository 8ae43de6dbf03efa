"""Drop-in through the reference's own frontend.

The reference package (``tonari``, installed unmodified from its sources into
baseline/_ref with its CPU and CUDA providers) is imported, and its provider
loader is rebound the way a maintainer would bind this library:
``tonari._extensions.load_torch_cuda`` (``src/tonari/_extensions.py:63-66``)
returns ``tonari_b200._torch_cuda``.  Then the reference's public
``tonari.neighbor_list`` (``src/tonari/api.py:52-234`` ->
``_torch_frontend.neighbor_list_torch``, ``_torch_frontend.py:108-158``) runs
on CUDA tensors end to end, and its results are compared with

* the same reference API on CPU tensors (the reference's Torch-CPU provider):
  exact (i, j, S) sets, d/D within 1e-5 (float32) / 1e-12 (float64) relative;
* the reference's own CUDA provider on the same CUDA tensors (stock path);
* gradients of d with respect to positions and cell through the reference
  frontend's autograd formula.

Skipped when baseline/_ref holds no reference install.
"""
from __future__ import annotations

import importlib
import sys
from pathlib import Path

import numpy as np
import pytest
import torch

from tests.support import assert_same_pairs, canonical

pytestmark = pytest.mark.gpu

REF_SITE = Path(__file__).resolve().parent.parent / "baseline" / "_ref"
TOLERANCE = {torch.float32: 1e-5, torch.float64: 1e-12}


@pytest.fixture(scope="module")
def reference_tonari():
    if not (REF_SITE / "tonari" / "api.py").exists():
        pytest.skip("the reference package is not installed in baseline/_ref")
    sys.path.insert(0, str(REF_SITE))
    try:
        tonari = importlib.import_module("tonari")
        frontend = importlib.import_module("tonari._torch_frontend")
        extensions = importlib.import_module("tonari._extensions")
    finally:
        sys.path.remove(str(REF_SITE))
    return tonari, frontend, extensions


@pytest.fixture
def with_b200_provider(reference_tonari, monkeypatch):
    """Rebind the reference's CUDA provider loader to this library."""
    from tonari_b200._extensions import load_torch_cuda

    _, frontend, extensions = reference_tonari
    monkeypatch.setattr(extensions, "load_torch_cuda", load_torch_cuda)
    monkeypatch.setattr(frontend, "load_torch_cuda", load_torch_cuda)
    return reference_tonari[0]


def _cases(dtype):
    generator = torch.Generator().manual_seed(2024)
    cases = []
    for k in range(6):
        batch = 1 + k % 3
        counts = torch.randint(1, 90, (batch,), generator=generator)
        cells = []
        positions = []
        for n in counts.tolist():
            cell = torch.diag(3.0 + 6.0 * torch.rand(3, generator=generator, dtype=torch.float64))
            cell += 0.8 * torch.tril(torch.rand((3, 3), generator=generator, dtype=torch.float64), -1)
            frac = torch.rand((n, 3), generator=generator, dtype=torch.float64)
            frac[: n // 5] += torch.randint(-2, 3, (n // 5, 3), generator=generator)  # nonzero wraps
            positions.append(frac @ cell)
            cells.append(cell)
        pbc = torch.rand((batch, 3), generator=generator) < 0.7
        batch_ptr = torch.cat((torch.zeros(1, dtype=torch.int64), counts.cumsum(0)))
        cutoff = 1.5 + 3.0 * float(torch.rand((), generator=generator))
        cases.append((torch.cat(positions).to(dtype), torch.stack(cells).to(dtype), pbc,
                      batch_ptr, cutoff))
    return cases


def _compare(actual, expected, dtype, quantities):
    P, S = actual[quantities.index("P")], actual[quantities.index("S")]
    eP, eS = expected[quantities.index("P")], expected[quantities.index("S")]
    assert_same_pairs(P.cpu(), S.cpu(), eP.cpu(), eS.cpu())
    rows = np.concatenate((P.cpu().numpy(), S.cpu().numpy()), 1)
    erows = np.concatenate((eP.cpu().numpy(), eS.cpu().numpy()), 1)
    order = np.lexsort(tuple(rows[:, k] for k in range(4, -1, -1)))
    eorder = np.lexsort(tuple(erows[:, k] for k in range(4, -1, -1)))
    tol = TOLERANCE[dtype]
    D = actual[quantities.index("D")].cpu().double().numpy()[order]
    eD = expected[quantities.index("D")].cpu().double().numpy()[eorder]
    scale = np.maximum(np.linalg.norm(eD, axis=1), 1e-3)
    assert np.all(np.linalg.norm(D - eD, axis=1) <= 4 * tol * scale)
    d = actual[quantities.index("d")].cpu().double().numpy()[order]
    ed = expected[quantities.index("d")].cpu().double().numpy()[eorder]
    assert np.all(np.abs(d - ed) <= 4 * tol * np.maximum(ed, 1e-3))
    i, j = actual[quantities.index("i")], actual[quantities.index("j")]
    assert torch.equal(i, P[:, 0]) and torch.equal(j, P[:, 1])


@pytest.mark.parametrize("dtype", [torch.float32, torch.float64])
@pytest.mark.parametrize("options", [{}, {"half_list": True}, {"include_self": True, "sorted": True},
                                     {"algorithm": "brute_force", "sorted": True}])
def test_reference_api_with_b200_provider_matches_reference_cpu(with_b200_provider, dtype, options):
    tonari = with_b200_provider
    quantities = "ijPSdD"
    for positions, cell, pbc, batch_ptr, cutoff in _cases(dtype):
        expected = tonari.neighbor_list(quantities, positions, cell, pbc, cutoff, batch_ptr,
                                        **options)
        actual = tonari.neighbor_list(quantities, positions.cuda(), cell.cuda(), pbc.cuda(),
                                      cutoff, batch_ptr.cuda(), **options)
        assert all(t.is_cuda for t in actual)
        if options.get("sorted"):
            P = actual[quantities.index("P")]
            assert torch.all(P[1:, 0] >= P[:-1, 0])
        _compare(actual, expected, dtype, quantities)


def test_reference_api_errors_are_unchanged(with_b200_provider):
    tonari = with_b200_provider
    positions = torch.zeros((2, 3), device="cuda")
    cell = torch.tensor([[1.0, 0, 0], [2.0, 0, 0], [0, 0, 4.0]], device="cuda")
    pbc = torch.tensor([True, True, False], device="cuda")
    with pytest.raises(ValueError, match="linearly independent"):
        tonari.neighbor_list("PS", positions, cell, pbc, 0.5)
    positions = torch.tensor([[float("nan"), 0.0, 0.0]], device="cuda")
    with pytest.raises(RuntimeError, match="finite"):
        tonari.neighbor_list("PS", positions, torch.eye(3, device="cuda"),
                             torch.tensor([True, True, True], device="cuda"), 0.5)


def test_reference_api_gradients_with_b200_provider(with_b200_provider):
    tonari = with_b200_provider
    positions, cell, pbc, batch_ptr, cutoff = _cases(torch.float64)[1]
    grads = []
    for device in ("cpu", "cuda"):
        p = positions.detach().clone().to(device).requires_grad_(True)
        c = cell.detach().clone().to(device).requires_grad_(True)
        (d,) = tonari.neighbor_list("d", p, c, pbc.to(device), cutoff, batch_ptr.to(device))
        d.sum().backward()
        grads.append((p.grad.cpu(), c.grad.cpu()))
    torch.testing.assert_close(grads[1][0], grads[0][0], rtol=1e-10, atol=1e-10)
    torch.testing.assert_close(grads[1][1], grads[0][1], rtol=1e-10, atol=1e-10)


def test_b200_provider_matches_reference_cuda_provider(reference_tonari):
    """The stock reference CUDA provider and this library, same CUDA inputs."""
    tonari, frontend, extensions = reference_tonari
    from tonari_b200._extensions import load_torch_cuda

    try:
        reference_provider = extensions.load_torch_cuda()
    except ImportError as error:
        pytest.skip(f"reference CUDA provider unavailable: {error}")
    for positions, cell, pbc, batch_ptr, cutoff in _cases(torch.float32):
        inputs = (positions.cuda(), batch_ptr.cuda(), cell.cuda(), pbc.cuda(), cutoff,
                  False, False, "auto")
        ref_P, ref_S = reference_provider.neighbor_list(*inputs, False)
        P, S = load_torch_cuda().neighbor_list(*inputs, False)
        assert np.array_equal(canonical(P, S), canonical(ref_P, ref_S))
