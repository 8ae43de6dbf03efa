"""Seeded synthetic inputs with the shapes of the five benchmark configurations.

The reference's published workloads (Matbench, QMugs) are not available here,
so every benchmark and full-size parity test uses these generators instead.
All randomness comes from ``numpy.random.default_rng(seed)``.

  cfg1  64 atoms U[0,10)^3, cubic 10 A cell, pbc TTT, float64, cutoff 5,
        'ijSd', brute force                           (reference CPU case)
  cfg2  512 triclinic crystals, 4-64 atoms, density 0.08 / A^3, pbc TTT,
        float32, cutoff 6 (multiple images), 'PSD'
  cfg3  2048 self-avoiding random-walk molecules, 10-120 atoms, pbc FFF,
        float32, cutoff 5, 'PD', sorted
  cfg4  1,000,000 atoms at 0.1 / A^3 in a cubic box, pbc TTT, float32,
        cutoff 6, cell list, 'ijSdD'
  cfg5  8192 triclinic structures, 50-5000 atoms (log-uniform), density
        0.05-0.12 / A^3, mixed pbc (p=0.8 per axis), float32, cutoff 5,
        half list, 'PS'
"""
from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np

# Largest float32 below 1: fractional coordinates stay inside [0, 1).
_BELOW_ONE = np.float32(1.0) - np.float32(2.0**-23)


@dataclass
class Workload:
    name: str
    positions: np.ndarray  # (N, 3)
    cell: np.ndarray  # (B, 3, 3)
    pbc: np.ndarray  # (B, 3) bool
    batch_ptr: np.ndarray  # (B + 1,) int64
    cutoff: float
    quantities: str
    options: dict = field(default_factory=dict)

    @property
    def n_atoms(self) -> int:
        return int(len(self.positions))

    @property
    def n_structures(self) -> int:
        return int(len(self.batch_ptr) - 1)

    def torch_inputs(self, device="cuda"):
        import torch

        return (
            torch.from_numpy(self.positions).to(device),
            torch.from_numpy(self.cell).to(device),
            torch.from_numpy(self.pbc).to(device),
            torch.from_numpy(self.batch_ptr).to(device),
        )

    def shard(self, begin: int, end: int) -> "Workload":
        """Structures [begin, end) as a standalone workload (atoms rebased)."""
        a0, a1 = int(self.batch_ptr[begin]), int(self.batch_ptr[end])
        return Workload(
            f"{self.name}[{begin}:{end}]",
            self.positions[a0:a1].copy(),
            self.cell[begin:end].copy(),
            self.pbc[begin:end].copy(),
            (self.batch_ptr[begin:end + 1] - a0).astype(np.int64),
            self.cutoff,
            self.quantities,
            dict(self.options),
        )


def _triclinic(lengths, angles_deg) -> np.ndarray | None:
    a, b, c = lengths
    alpha, beta, gamma = np.radians(angles_deg)
    cx = c * np.cos(beta)
    cy = c * (np.cos(alpha) - np.cos(beta) * np.cos(gamma)) / np.sin(gamma)
    cz2 = c * c - cx * cx - cy * cy
    if cz2 < 0.05 * c * c:
        return None
    return np.array(
        [[a, 0.0, 0.0], [b * np.cos(gamma), b * np.sin(gamma), 0.0], [cx, cy, np.sqrt(cz2)]]
    )


def _random_cell(rng, length_range, angle_range) -> np.ndarray:
    while True:
        cell = _triclinic(rng.uniform(*length_range, 3), rng.uniform(*angle_range, 3))
        if cell is not None:
            return cell


def _crystal_batch(rng, counts, length_range, angle_range, densities, dtype):
    cells, positions = [], []
    for n, density in zip(counts, densities):
        cell = _random_cell(rng, length_range, angle_range)
        volume = abs(np.linalg.det(cell))
        cell = cell * (n / density / volume) ** (1.0 / 3.0)
        fractional = np.minimum(rng.random((n, 3)), _BELOW_ONE)
        cells.append(cell)
        positions.append(fractional @ cell)
    batch_ptr = np.concatenate(([0], np.cumsum(counts))).astype(np.int64)
    return (np.concatenate(positions).astype(dtype), np.stack(cells).astype(dtype), batch_ptr)


def config1(seed: int = 0) -> Workload:
    rng = np.random.default_rng(seed)
    positions = rng.random((64, 3)) * 10.0
    return Workload(
        "cfg1", positions.astype(np.float64), (10.0 * np.eye(3))[None].astype(np.float64),
        np.ones((1, 3), bool), np.array([0, 64], np.int64), 5.0, "ijSd",
        {"algorithm": "brute_force"},
    )


def config2(seed: int = 2, n_structures: int = 512) -> Workload:
    rng = np.random.default_rng(seed)
    counts = rng.integers(4, 65, n_structures)
    positions, cell, batch_ptr = _crystal_batch(
        rng, counts, (3.0, 10.0), (70.0, 110.0), np.full(n_structures, 0.08), np.float32)
    return Workload("cfg2", positions, cell, np.ones((n_structures, 3), bool), batch_ptr, 6.0,
                    "PSD", {})


def _self_avoiding_walk(rng, n: int) -> np.ndarray:
    points = np.zeros((n, 3))
    for k in range(1, n):
        for _attempt in range(64):
            direction = rng.normal(size=3)
            direction /= np.linalg.norm(direction)
            step = rng.uniform(1.0, 1.6)
            candidate = points[k - 1] + step * direction
            if k < 2 or np.min(np.sum((points[: k - 1] - candidate) ** 2, axis=1)) >= 1.0:
                break
        points[k] = candidate
    return points


def config3(seed: int = 3, n_structures: int = 2048) -> Workload:
    rng = np.random.default_rng(seed)
    counts = rng.integers(10, 121, n_structures)
    positions = np.concatenate([_self_avoiding_walk(rng, int(n)) for n in counts])
    batch_ptr = np.concatenate(([0], np.cumsum(counts))).astype(np.int64)
    return Workload(
        "cfg3", positions.astype(np.float32), np.zeros((n_structures, 3, 3), np.float32),
        np.zeros((n_structures, 3), bool), batch_ptr, 5.0, "PD", {"sorted": True},
    )


def config4(seed: int = 4, n_atoms: int = 1_000_000, density: float = 0.1) -> Workload:
    rng = np.random.default_rng(seed)
    length = (n_atoms / density) ** (1.0 / 3.0)
    fractional = np.minimum(rng.random((n_atoms, 3), dtype=np.float32), _BELOW_ONE)
    positions = (fractional * np.float32(length)).astype(np.float32)
    cell = (np.float32(length) * np.eye(3, dtype=np.float32))[None]
    return Workload("cfg4", positions, cell, np.ones((1, 3), bool),
                    np.array([0, n_atoms], np.int64), 6.0, "ijSdD", {"algorithm": "cell_list"})


def config5(seed: int = 5, n_structures: int = 8192) -> Workload:
    rng = np.random.default_rng(seed)
    counts = np.floor(np.exp(rng.uniform(np.log(50), np.log(5000), n_structures))).astype(np.int64)
    densities = rng.uniform(0.05, 0.12, n_structures)
    positions, cell, batch_ptr = _crystal_batch(
        rng, counts, (8.0, 40.0), (60.0, 120.0), densities, np.float32)
    pbc = rng.random((n_structures, 3)) < 0.8
    return Workload("cfg5", positions, cell, pbc, batch_ptr, 5.0, "PS", {"half_list": True})


CONFIGS = {"cfg1": config1, "cfg2": config2, "cfg3": config3, "cfg4": config4, "cfg5": config5}


def algorithmic_bytes(workload: Workload, n_pairs: int) -> int:
    """Inputs read once plus requested outputs written once:
    N*3*s + B*9*s + B*3 + (B+1)*8 + E*sum(bytes(q) for q in set(quantities)),
    with i=8, j=8, P=16, S=12, d=s, D=3s bytes per pair."""
    s = workload.positions.dtype.itemsize
    per_pair = {"i": 8, "j": 8, "P": 16, "S": 12, "d": s, "D": 3 * s}
    read = (workload.n_atoms * 3 * s + workload.n_structures * 9 * s
            + workload.n_structures * 3 + (workload.n_structures + 1) * 8)
    return int(read + n_pairs * sum(per_pair[q] for q in set(workload.quantities)))


def concatenate(parts: list[Workload], name: str) -> Workload:
    """One batch made of several workloads' structures, in order."""
    offsets = np.cumsum([0] + [p.n_atoms for p in parts])
    batch_ptr = np.concatenate([parts[0].batch_ptr[:1]] +
                               [p.batch_ptr[1:] + o for p, o in zip(parts, offsets)])
    return Workload(name, np.concatenate([p.positions for p in parts]),
                    np.concatenate([p.cell for p in parts]), np.concatenate([p.pbc for p in parts]),
                    batch_ptr.astype(np.int64), parts[0].cutoff, parts[0].quantities,
                    dict(parts[0].options))
