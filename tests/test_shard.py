"""Sharding of independent worlds across ranks (CPU: gloo, world size 2).

Worlds never interact, so a multi-GPU step is N independent shards with no
per-step exchange; the tests check the host-side logic that makes that true:
contiguous balanced shard ranges, worlds seeded by their global index (a
shard builds exactly its slice of the full batch and its trajectories do not
depend on the world size), and the end-of-run statistics reduction.
"""
import os
import socket

import numpy as np
import pytest
import torch.multiprocessing as mp

import oracle as orc
from puffysics_b200 import shard, synth
from puffysics_b200.configs import CONFIGS


@pytest.mark.parametrize("n,w", [(16384, 1), (16384, 8), (10, 3), (7, 8), (0, 2), (1048576, 8)])
def test_shard_ranges_cover_disjoint_balanced(n, w):
    ranges = [shard.shard_range(n, r, w) for r in range(w)]
    assert ranges[0][0] == 0 and ranges[-1][1] == n
    for (b0, e0), (b1, e1) in zip(ranges, ranges[1:]):
        assert e0 == b1
    sizes = [e - b for b, e in ranges]
    assert max(sizes) - min(sizes) <= 1


@pytest.mark.parametrize("rank,w", [(-1, 2), (2, 2), (0, 0)])
def test_shard_range_rejects_bad_rank(rank, w):
    with pytest.raises(ValueError):
        shard.shard_range(10, rank, w)


@pytest.mark.parametrize("name", ["stack", "chain"])
def test_shard_builds_its_slice_of_the_full_batch(name):
    cfg = CONFIGS[name]
    lib = synth.SceneLib(cfg)
    n, seed = 37, 5
    full = lib.build(n, seed)
    for w in (2, 3):
        parts = [lib.build(e - b, seed, first=b) for b, e in (shard.shard_range(n, r, w) for r in range(w))]
        assert np.array_equal(np.concatenate(parts), full)
        for r in range(w):
            b, e = shard.shard_range(n, r, w)
            assert np.array_equal(lib.actions(e - b, seed, b, 3), lib.actions(n, seed, 0, 3)[b:e])


def test_trajectories_do_not_depend_on_world_size():
    """Stepping two shards separately (CPU oracle, global-index actions) gives
    the same worlds as stepping the whole batch."""
    cfg = CONFIGS["stack"]
    assert orc.build_oracles() == 0
    o = orc.Oracle("stack", "port")
    n, seed = 12, 9
    full = o.build(n, cfg.scene, seed)
    shards = [full[b:e].copy() for b, e in (shard.shard_range(n, r, 2) for r in range(2))]
    for step in range(1, 6):
        o.apply(full, cfg.scene, seed, 0, step)
        o.batch_step(full, cfg.dt, cfg.substeps)
        for r, part in enumerate(shards):
            b, _ = shard.shard_range(n, r, 2)
            o.apply(part, cfg.scene, seed, b, step)
            o.batch_step(part, cfg.dt, cfg.substeps)
    assert np.array_equal(np.concatenate(shards), full)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, n, out_dir):
    import torch.distributed as dist
    cfg = CONFIGS["stack"]
    dist.init_process_group("gloo", init_method="tcp://127.0.0.1:%d" % port, rank=rank, world_size=world)
    try:
        b, e = shard.shard_range(n, rank, world)
        worlds = synth.SceneLib(cfg).build(e - b, 3, first=b)
        tot = shard.reduce_stats(shard.world_stats(worlds, cfg.caps))
        np.save(os.path.join(out_dir, "rank%d.npy" % rank), tot)
    finally:
        dist.destroy_process_group()


def test_stats_reduction_over_gloo_ranks(tmp_path):
    cfg = CONFIGS["stack"]
    n, world = 50, 2
    mp.start_processes(_rank_main, args=(world, _free_port(), n, str(tmp_path)), nprocs=world, join=True,
                       start_method="spawn")
    expect = shard.world_stats(synth.SceneLib(cfg).build(n, 3), cfg.caps)
    for r in range(world):
        assert np.array_equal(np.load(tmp_path / ("rank%d.npy" % r)), expect)
