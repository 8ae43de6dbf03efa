"""Batch sharding: partition properties and a world-size-2 gloo run on CPU.

The per-shard search on CPU is the oracle port, passed in as the shard's
neighbor-list implementation; on GPUs the same host logic drives the
tonari_b200 kernels (bench.py --gpus N)."""
from __future__ import annotations

import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import oracle
from tonari_b200 import sharding, workloads


def oracle_shard(quantities, positions, cell, pbc, cutoff, batch_ptr, *, index_offset, **options):
    pairs, shifts = oracle.port_neighbor_list(positions, cell, pbc, cutoff, batch_ptr,
                                              half_list=options.get("half_list", False))
    return pairs + index_offset, shifts


def test_partition_is_contiguous_complete_and_balanced():
    w = workloads.config5(n_structures=300)
    weights = sharding.estimate_pairs(w.batch_ptr, w.cell, w.pbc, w.cutoff, half_list=True)
    for n in (1, 2, 3, 8):
        shards = sharding.partition(w.batch_ptr, weights, n)
        assert shards[0].structure_begin == 0 and shards[-1].structure_end == w.n_structures
        for a, b in zip(shards, shards[1:]):
            assert a.structure_end == b.structure_begin and a.atom_end == b.atom_begin
        loads = [weights[s.structure_begin:s.structure_end].sum() for s in shards]
        assert max(loads) <= weights.sum() / n + weights.max() + 1e-6


@pytest.mark.skipif(not oracle.ref_available(), reason="reference CPU core not built")
def test_pair_estimate_tracks_exact_counts_for_every_pbc_pattern():
    """The balancing weight predicts each pbc group's pairs within a few percent
    (non-periodic axes lose the spherical caps cut by the cell faces)."""
    w = workloads.config5(n_structures=400)
    w.pbc = np.asarray(w.pbc).copy()
    w.pbc.reshape(-1, 3)[:20] = False  # finite cells with atoms inside, no periodic axis
    pairs, _ = oracle.ref_neighbor_list(w.positions, w.cell, w.pbc, w.cutoff, w.batch_ptr,
                                        half_list=True, algorithm="auto", threads=os.cpu_count() or 1)
    source = np.asarray(pairs)[:, 0]
    structure = np.searchsorted(w.batch_ptr, source, side="right") - 1
    actual = np.bincount(structure, minlength=w.n_structures).astype(float)
    counts = np.diff(w.batch_ptr)
    estimate = sharding.estimate_pairs(w.batch_ptr, w.cell, w.pbc, w.cutoff, half_list=True)
    estimate = estimate - sharding.kAtomWork * counts
    periodic_axes = np.asarray(w.pbc).reshape(-1, 3).sum(axis=1)
    for k in range(4):
        group = periodic_axes == k
        if group.sum() >= 5:
            assert actual[group].sum() == pytest.approx(estimate[group].sum(), rel=0.08), k


def test_partition_handles_more_shards_than_structures():
    batch_ptr = np.array([0, 5, 9], np.int64)
    shards = sharding.partition(batch_ptr, np.array([1.0, 1.0]), 4)
    assert sum(s.n_structures for s in shards) == 2
    assert shards[-1].atom_end == 9


def test_shard_union_equals_full_batch_single_process():
    w = workloads.config2(n_structures=40)
    weights = sharding.estimate_pairs(w.batch_ptr, w.cell, w.pbc, w.cutoff)
    full = oracle.canonical_rows(*oracle.port_neighbor_list(w.positions, w.cell, w.pbc, w.cutoff,
                                                            w.batch_ptr))
    parts = [sharding.neighbor_list_shard("PS", s, w.positions, w.cell, w.pbc, w.cutoff,
                                          w.batch_ptr, neighbor_list=oracle_shard)
             for s in sharding.partition(w.batch_ptr, weights, 3)]
    merged = oracle.canonical_rows(np.concatenate([p for p, _ in parts]),
                                   np.concatenate([s for _, s in parts]))
    assert np.array_equal(merged, full)


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, fail_rank, queue):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        w = workloads.config2(n_structures=30)
        cell = w.cell.copy()
        weights = sharding.estimate_pairs(w.batch_ptr, cell, w.pbc, w.cutoff)
        shards = sharding.partition(w.batch_ptr, weights, world)
        if rank == fail_rank:
            cell[shards[rank].structure_begin, 0, 0] = np.nan  # this rank's shard is invalid
        error, result = None, None
        try:
            result = sharding.neighbor_list_shard("PS", shards[rank], w.positions, cell, w.pbc,
                                                  w.cutoff, w.batch_ptr, neighbor_list=oracle_shard)
        except Exception as caught:  # noqa: BLE001 - forwarded to every rank
            error = caught
        try:
            sharding.agree_on_outcome(error)
        except Exception as raised:  # noqa: BLE001
            queue.put((rank, "error", type(raised).__name__, str(raised)))
            return
        gathered = [None] * world
        dist.all_gather_object(gathered, result)
        if rank == 0:
            merged = oracle.canonical_rows(np.concatenate([g[0] for g in gathered]),
                                           np.concatenate([g[1] for g in gathered]))
            full = oracle.canonical_rows(*oracle.port_neighbor_list(
                w.positions, w.cell, w.pbc, w.cutoff, w.batch_ptr))
            queue.put((rank, "ok", bool(np.array_equal(merged, full)), len(full)))
        else:
            queue.put((rank, "ok", True, 0))
    finally:
        dist.destroy_process_group()


def _run(world, fail_rank):
    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, fail_rank, queue)) for r in range(world)]
    for p in procs:
        p.start()
    results = [queue.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    return sorted(results)


def test_gloo_two_ranks_reproduce_the_full_batch():
    results = _run(2, fail_rank=-1)
    assert all(r[1] == "ok" and r[2] for r in results)
    assert results[0][3] > 0


def test_gloo_shard_failure_reaches_every_rank():
    results = _run(2, fail_rank=1)
    by_rank = {r[0]: r for r in results}
    assert by_rank[1][1] == "error" and by_rank[1][2] == "OracleInputError"
    assert "cell must contain only finite values" in by_rank[1][3]
    assert by_rank[0][1] == "error" and by_rank[0][2] == "ShardFailure"
    assert "rank 1" in by_rank[0][3]


def test_shard_rejects_unknown_options():
    # With the default provider, an option it does not know is an error, not
    # silently dropped.
    w = workloads.config2(n_structures=4)
    shard = sharding.partition(w.batch_ptr, np.ones(4), 1)[0]
    with pytest.raises(TypeError, match="half_lst"):
        sharding.neighbor_list_shard("PS", shard, w.positions, w.cell, w.pbc, w.cutoff,
                                     w.batch_ptr, half_lst=True)
