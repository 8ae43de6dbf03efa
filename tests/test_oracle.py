"""Pins the CPU checkers: the plain-C restatement (oracle/_port) against the
golden fixtures (made from the reference's own Torch oracle) and against the
reference's CPU core (oracle/_ref) on seeded random inputs."""
from __future__ import annotations

from pathlib import Path

import numpy as np
import pytest

from oracle import oracle
from tonari_b200 import workloads

GOLDEN = sorted((Path(__file__).parent / "golden").glob("*.npz"))


def load(path):
    data = np.load(path)
    return {k: data[k] for k in data.files}


@pytest.mark.parametrize("path", GOLDEN, ids=[p.stem for p in GOLDEN])
def test_port_matches_golden(path):
    g = load(path)
    rows = oracle.canonical_rows(*oracle.port_neighbor_list(
        g["positions"], g["cell"], g["pbc"], float(g["cutoff"]), g["batch_ptr"],
        half_list=bool(g["half_list"]), include_self=bool(g["include_self"])))
    assert np.array_equal(rows, g["rows"])


@pytest.mark.skipif(not oracle.ref_available(), reason="reference core not built here")
@pytest.mark.parametrize("path", GOLDEN, ids=[p.stem for p in GOLDEN])
def test_reference_core_matches_golden(path):
    g = load(path)
    rows = oracle.canonical_rows(*oracle.ref_neighbor_list(
        g["positions"], g["cell"], g["pbc"], float(g["cutoff"]), g["batch_ptr"],
        half_list=bool(g["half_list"]), include_self=bool(g["include_self"]), threads=2))
    assert np.array_equal(rows, g["rows"])


@pytest.mark.skipif(not oracle.ref_available(), reason="reference core not built here")
def test_port_matches_reference_core_randomized():
    rng = np.random.default_rng(11)
    for case in range(40):
        dtype = np.float32 if case % 2 else np.float64
        n = int(rng.integers(1, 40))
        cell = np.diag(1.8 + 2.5 * rng.random(3)) + 0.35 * np.tril(rng.random((3, 3)), -1)
        positions = rng.random((n, 3)) @ cell
        if case % 4 == 0:
            positions[0] += 3 * cell[0]
        pbc = rng.random(3) < 0.6
        cutoff = 0.55 + 1.2 * rng.random()
        for half in (False, True):
            for self_pairs in (False, True):
                args = (positions.astype(dtype), cell.astype(dtype), pbc, cutoff)
                a = oracle.canonical_rows(*oracle.ref_neighbor_list(
                    *args, half_list=half, include_self=self_pairs, threads=2))
                b = oracle.canonical_rows(*oracle.port_neighbor_list(
                    *args, half_list=half, include_self=self_pairs))
                assert np.array_equal(a, b)


def test_config1_pair_count():
    w = workloads.config1()
    pairs, _ = oracle.port_neighbor_list(w.positions, w.cell, w.pbc, w.cutoff, w.batch_ptr)
    assert len(pairs) == 2130


def test_port_error_messages():
    with pytest.raises(oracle.OracleInputError, match="linearly independent"):
        oracle.port_neighbor_list(np.zeros((1, 3)), np.array([[1.0, 0, 0], [2.0, 0, 0], [0, 0, 4]]),
                                  np.array([True, True, False]), 0.5)
    with pytest.raises(oracle.OracleSearchError, match="wraps.*int32"):
        oracle.port_neighbor_list(np.array([[0.1, 0, 0], [2.0**31 + 0.2, 0, 0]]), np.eye(3),
                                  np.array([True, False, False]), 0.5)
