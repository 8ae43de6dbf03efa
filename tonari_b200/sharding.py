"""Batch sharding across GPUs (one process per GPU, no data-path collective).

Structures are independent and pairs never cross ``batch_ptr`` boundaries
(tonari docs/design.md:60-62), so a batch splits into contiguous runs of
structures, one per rank.  Shards are balanced by an estimate of the pairs
each structure emits; a single structure is never split.  Every rank computes
the same partition from the same host metadata, runs the neighbor list on its
own shard with ``index_offset`` set so that the emitted indices are global,
and keeps its pairs on its own GPU.  Concatenating the shards' outputs in rank
order gives the whole batch's pairs (source-major when ``sorted=True``).
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import numpy as np


def estimate_pairs(batch_ptr, cell, pbc, cutoff: float, half_list: bool = False) -> np.ndarray:
    """Expected work per structure in pairs (float64, shape (B,)).

    Structures with a cell of nonzero volume (periodic or not):
    N * min(N * 27, rho * 4/3 pi rc^3 * s) with rho the
    atom density of the cell and s the mean fraction of an atom's cutoff
    sphere that lies inside the cell along its non-periodic axes: for atoms
    uniform in a slab of perpendicular width w >= rc that fraction is
    1 - 3 rc / (8 w) (the two faces each cut a spherical cap; averaging the
    cap volume over the slab gives pi rc^4 / (2 w)), and it is taken as
    0.625 w / rc below rc.  Structures without a volume (zero or degenerate
    cells): N * (N - 1), the brute-force upper bound.  Halved for
    half lists.  Each atom adds kAtomWork pairs' worth of per-atom work
    (wrapping, binning of its image copies).  Only the relative sizes matter
    for balancing.
    """
    batch_ptr = np.asarray(batch_ptr, dtype=np.int64)
    cell = np.asarray(cell, dtype=np.float64).reshape(-1, 3, 3)
    pbc = np.asarray(pbc, dtype=bool).reshape(-1, 3)
    counts = np.diff(batch_ptr).astype(np.float64)
    volume = np.abs(np.linalg.det(cell))
    sphere = 4.0 / 3.0 * math.pi * cutoff**3
    with np.errstate(divide="ignore", invalid="ignore"):
        density = np.where(volume > 0, counts / volume, np.inf)
        # Perpendicular width along axis a: volume / |b x c|.
        widths = np.stack([volume / np.linalg.norm(np.cross(cell[:, (a + 1) % 3], cell[:, (a + 2) % 3]), axis=1)
                           for a in range(3)], axis=1)
        slab = np.where(widths >= cutoff, 1.0 - 3.0 * cutoff / (8.0 * widths), 0.625 * widths / cutoff)
    slab = np.where(np.isfinite(slab), np.clip(slab, 0.0, 1.0), 1.0)
    inside = np.prod(np.where(pbc, 1.0, slab), axis=1)
    usable = np.isfinite(density)  # atoms fill a cell of nonzero volume (any pbc)
    per_atom = np.where(usable, np.minimum(density * sphere * inside, counts * 27.0), counts - 1.0)
    pairs = counts * np.maximum(per_atom, 0.0) * (0.5 if half_list else 1.0)
    return pairs + kAtomWork * counts


# Per-atom work (prepare, binning of image copies) in pairs' worth, from the
# measured split of a cfg5 call on one B200: about 2 ms of per-atom kernels
# for 8.8M atoms against 5.5 ms of count and write passes for 187M pairs.
kAtomWork = 8.0


@dataclass(frozen=True)
class Shard:
    rank: int
    structure_begin: int
    structure_end: int
    atom_begin: int
    atom_end: int

    @property
    def n_structures(self) -> int:
        return self.structure_end - self.structure_begin


def partition(batch_ptr, weights, n_shards: int) -> list[Shard]:
    """Split structures [0, B) into n_shards contiguous runs of near-equal
    total weight (greedy cut at the weight quantiles).  Shards may be empty."""
    if n_shards < 1:
        raise ValueError("n_shards must be positive")
    batch_ptr = np.asarray(batch_ptr, dtype=np.int64)
    weights = np.asarray(weights, dtype=np.float64)
    b = len(batch_ptr) - 1
    if len(weights) != b:
        raise ValueError("weights must have one entry per structure")
    prefix = np.concatenate(([0.0], np.cumsum(weights)))
    total = prefix[-1]
    cuts = [0]
    for k in range(1, n_shards):
        target = total * k / n_shards
        cut = int(np.searchsorted(prefix, target, side="left"))
        # Pick the closer of the two neighbouring boundaries.
        if 0 < cut <= b and abs(prefix[cut - 1] - target) < abs(prefix[cut] - target):
            cut -= 1
        cuts.append(min(max(cut, cuts[-1]), b))
    cuts.append(b)
    return [Shard(rank, cuts[rank], cuts[rank + 1], int(batch_ptr[cuts[rank]]),
                  int(batch_ptr[cuts[rank + 1]])) for rank in range(n_shards)]


def shard_inputs(shard: Shard, positions, cell, pbc, batch_ptr):
    """The shard's slice of the batch with batch_ptr rebased to zero.  Works
    for NumPy arrays and Torch tensors alike (slices are views)."""
    s0, s1 = shard.structure_begin, shard.structure_end
    sub_ptr = batch_ptr[s0:s1 + 1] - batch_ptr[s0]
    return positions[shard.atom_begin:shard.atom_end], cell[s0:s1], pbc[s0:s1], sub_ptr


def neighbor_list_shard(quantities: str, shard: Shard, positions, cell, pbc, cutoff: float,
                        batch_ptr, *, neighbor_list=None, **options):
    """Run the neighbor list on one shard with globally numbered atom indices.

    ``neighbor_list`` defaults to the B200 provider's fused entry point; tests
    may pass another implementation with the same signature (it must accept
    ``index_offset``)."""
    sub = shard_inputs(shard, positions, cell, pbc, batch_ptr)
    if neighbor_list is None:
        from ._frontend import neighbor_list_torch

        algorithm = options.pop("algorithm", "auto")
        sort = options.pop("sorted", False)
        half_list = options.pop("half_list", False)
        include_self = options.pop("include_self", False)
        if options:
            raise TypeError(f"unexpected neighbor-list options: {sorted(options)}")
        return neighbor_list_torch(
            quantities, sub[0], sub[1], sub[2], cutoff, sub[3],
            algorithm=algorithm, cpu_threads=None, sorted=sort, half_list=half_list,
            include_self=include_self, index_offset=shard.atom_begin)
    return neighbor_list(quantities, sub[0], sub[1], sub[2], cutoff, sub[3],
                         index_offset=shard.atom_begin, **options)


class ShardFailure(RuntimeError):
    """A shard failed on another rank; carries that rank and its message."""


def agree_on_outcome(error: BaseException | None, group=None) -> None:
    """Host-side failure propagation between ranks, called between steps.

    Every rank passes the exception its shard raised (or None).  The outcomes
    are exchanged with ``all_gather_object`` (no device work is in flight), and
    if any rank failed every rank raises: the failing rank re-raises its own
    exception, the others raise ShardFailure naming the lowest failing rank.
    """
    import torch.distributed as dist

    summary = None if error is None else (type(error).__name__, str(error))
    outcomes = [None] * dist.get_world_size(group)
    dist.all_gather_object(outcomes, summary, group=group)
    failed = [(rank, item) for rank, item in enumerate(outcomes) if item is not None]
    if not failed:
        return
    if error is not None:
        raise error
    rank, (kind, message) = failed[0]
    raise ShardFailure(f"shard on rank {rank} failed with {kind}: {message}")
