"""Generate tests/golden/*.npz from the reference implementation.

Run where the reference checkout is available, naming it with --reference or
the TONARI_REFERENCE_ROOT environment variable:

    python tests/golden/make_golden.py --reference <reference checkout>

For every case the expected pair set comes from the reference's independent
Torch oracle (tests/support/reference.py, ``neighbor_list_reference``), and is
cross-checked against the reference's CPU search core (oracle/_ref) before
it is written.  Each fixture stores the inputs and the canonical
(i, j, Sx, Sy, Sz) rows.  The fixtures are small; tests read them with no
access to the reference.
"""
from __future__ import annotations

import argparse
import os
import importlib.util
import sys
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent.parent
sys.path.insert(0, str(ROOT))


def load_reference_oracle(reference_root: Path):
    path = reference_root / "tests" / "support" / "reference.py"
    spec = importlib.util.spec_from_file_location("tonari_reference_oracle", path)
    module = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(module)
    return module.neighbor_list_reference


def cases():
    """(name, positions, cell (B,3,3), pbc (B,3), cutoff, batch_ptr, half, self)."""
    out = []
    # Strict boundary and nextafter (tests/backends/test_pair_identity.py:83-117).
    out.append(("strict_boundary", torch.tensor([[0.0, 0.0, 0.0], [1.0, 0.0, 0.0]]),
                torch.zeros((1, 3, 3)), torch.zeros((1, 3), dtype=torch.bool), 1.0, [0, 2], 0, 0))
    inside = torch.tensor([[0.0, 0.0, 0.0], [1.0, 0.0, 0.0]])
    inside[1, 0] = torch.nextafter(torch.tensor(1.0), torch.tensor(0.0))
    out.append(("nextafter_inside", inside, torch.zeros((1, 3, 3)),
                torch.zeros((1, 3), dtype=torch.bool), 1.0, [0, 2], 0, 0))
    # Periodic self images (tests/test_reference.py:26-39).
    out.append(("self_images", torch.zeros((1, 3)), torch.diag(torch.tensor([0.4, 8.0, 8.0]))[None],
                torch.tensor([[True, False, False]]), 1.0, [0, 1], 0, 0))
    # Mixed batch never crossing structures (tests/test_reference.py:42-60).
    out.append(("mixed_batch", torch.tensor([[0.0, 0.0, 0.0], [0.4, 0.0, 0.0], [0.0, 0.0, 0.0]]),
                torch.stack((torch.zeros((3, 3)), torch.diag(torch.tensor([0.5, 8.0, 8.0])))),
                torch.tensor([[False, False, False], [True, False, False]]), 0.6, [0, 2, 3], 0, 0))
    # Randomized triclinic cases over pbc patterns and pair options
    # (after tests/backends/test_pair_identity.py:189-223).
    generator = torch.Generator().manual_seed(29381)
    patterns = torch.tensor([[False, False, False], [True, False, False], [True, False, True],
                             [True, True, False], [True, True, True]])
    for case in range(10):
        n = 3 + 4 * case
        dtype = torch.float64 if case % 2 else torch.float32
        cell = torch.diag(1.8 + 2.5 * torch.rand(3, generator=generator))
        cell += 0.35 * torch.tril(torch.rand((3, 3), generator=generator), diagonal=-1)
        positions = torch.rand((n, 3), generator=generator) @ cell
        pbc = patterns[case % len(patterns)]
        if case % 3 == 0:
            positions[0] += 3 * cell[0]
        cutoff = 0.55 + 0.8 * float(torch.rand((), generator=generator))
        out.append((f"random_{case}", positions.to(dtype), cell.to(dtype)[None], pbc[None],
                    cutoff, [0, n], case % 2, (case // 2) % 2))
    return out


def main() -> None:
    parser = argparse.ArgumentParser()
    parser.add_argument("--reference", default=os.environ.get("TONARI_REFERENCE_ROOT"))
    args = parser.parse_args()
    if not args.reference:
        parser.error("name the reference checkout with --reference or TONARI_REFERENCE_ROOT")
    reference = load_reference_oracle(Path(args.reference))
    from oracle import oracle

    for name, positions, cell, pbc, cutoff, ptr, half, self_pairs in cases():
        batch_ptr = torch.tensor(ptr, dtype=torch.int64)
        pairs, shifts = reference(positions, cell, pbc, cutoff, batch_ptr,
                                  half_list=bool(half), include_self=bool(self_pairs))
        rows = oracle.canonical_rows(pairs.numpy(), shifts.numpy())
        if oracle.ref_available():
            check = oracle.canonical_rows(*oracle.ref_neighbor_list(
                positions.numpy(), cell.numpy(), pbc.numpy(), cutoff, batch_ptr.numpy(),
                half_list=bool(half), include_self=bool(self_pairs), threads=1))
            assert np.array_equal(rows, check), f"{name}: reference oracles disagree"
        np.savez_compressed(HERE / f"{name}.npz", positions=positions.numpy(), cell=cell.numpy(),
                            pbc=pbc.numpy(), batch_ptr=batch_ptr.numpy(), cutoff=cutoff,
                            half_list=half, include_self=self_pairs, rows=rows)
        print(f"{name}: {len(rows)} pairs")


if __name__ == "__main__":
    main()
