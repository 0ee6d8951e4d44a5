"""Steps that take more than one kernel launch, against the reference's CPU
b3_batch_step (reference b3_batch.cuh:81-89: one call steps every world,
whatever the batch size).

A step runs one step-kernel launch per chunk of tiles (32 worlds each); a
chunk is as many tiles as the workspace has slots, at most the device's
resident blocks.  So a call with more tiles than slots runs several launches
that reuse the same slots, each starting at a later tile.  Covered here:
caller workspaces of exactly one and two slots over 5-7 tiles (stack and
pile, masked and unmasked, 20 steps); a reserved workspace with more tiles
than one wave of resident blocks; the library's fixed array (no reservation)
with more tiles than it has slots; and the allocation behaviour of the
default entry point.  Bar: the whole AoS world byte for byte, every step.
"""
import numpy as np
import pytest
import torch

import oracle as orc
from puffysics_b200 import engine, synth
from puffysics_b200.configs import CONFIGS

pytestmark = pytest.mark.gpu


def run_pair(cfg, o, n, steps, seed, step_fn, masked=False):
    """Step the same worlds on the GPU (step_fn(dev, active)) and on the
    oracle, with the scene's actions; compare every step."""
    host = o.build(n, cfg.scene, seed)
    dev = torch.from_numpy(host.copy()).cuda()
    kind, idx, nv = cfg.action
    vals = torch.zeros((n, max(nv, 1)), dtype=torch.float32, device="cuda")
    rng = np.random.default_rng(seed)
    for s in range(1, steps + 1):
        mask = (rng.random(n) < 0.6).astype(np.uint8) if masked else None
        act = None if mask is None else torch.from_numpy(mask).cuda()
        o.apply(host, cfg.scene, seed, 0, s, active=mask)
        if nv:
            assert synth.actions_gpu(vals, n, cfg.scene, seed, 0, s) == nv
            assert engine.batch_apply_gpu(dev, kind, idx, vals, active=act, caps=cfg.caps) == 0
        assert o.batch_step(host, cfg.dt, cfg.substeps, active=mask) == 1
        assert step_fn(dev, act) == 0
        torch.cuda.synchronize()
        got = dev.cpu().numpy()
        if not np.array_equal(got, host):
            bad = np.where((got != host).any(1))[0]
            raise AssertionError("%s: %d worlds differ at step %d (first %d)" % (cfg.name, len(bad), s, bad[0]))
    assert engine.fault_flags() == 0


@pytest.mark.parametrize("name,n", [("stack", 160), ("stack", 223), ("pile", 192)])
@pytest.mark.parametrize("slots", [1, 2])
@pytest.mark.parametrize("masked", [False, True])
def test_caller_workspace_of_one_and_two_slots(name, n, slots, masked, oracle_kind, gpu_lib):
    cfg = CONFIGS[name]
    o = orc.Oracle(name, oracle_kind)
    slot = engine.workspace_slot_bytes(cfg.caps)
    assert slot > 0 and slot % 256 == 0
    ws = torch.empty(slots * slot + slot // 2, dtype=torch.uint8, device="cuda")   # a partial slot is unused
    tiles = (n + 31) // 32
    assert tiles > 2 * slots

    def step(dev, act):
        return engine.batch_step_gpu(dev, cfg.dt, cfg.substeps, active=act, caps=cfg.caps,
                                     joint_iters=cfg.joint_iters, workspace=ws)

    run_pair(cfg, o, n, 20, 4242 + n, step, masked)


def test_reserved_workspace_more_tiles_than_one_wave(oracle_kind, gpu_lib):
    """19,000 stack worlds are 594 tiles: more than one wave of resident
    blocks (148 SMs x 4 = 592 on a B200), so the step runs a second launch
    starting at tile 592 with the reserved workspace's slots reused."""
    cfg = CONFIGS["stack"]
    n = 19000
    o = orc.Oracle("stack", oracle_kind)
    stream = torch.cuda.current_stream()
    assert engine.reserve_workspace(cfg.caps, stream) == 0
    try:
        assert engine.reserved_bytes(stream) == engine.workspace_bytes(cfg.caps)
        assert engine.step_launches(cfg.caps, n) >= 2

        def step(dev, act):
            return engine.batch_step_gpu(dev, cfg.dt, cfg.substeps, active=act, stream=stream, caps=cfg.caps,
                                         joint_iters=cfg.joint_iters)

        run_pair(cfg, o, n, 3, 99, step)
    finally:
        assert engine.release_workspaces() == 0
    assert engine.reserved_bytes(stream) == 0


@pytest.mark.parametrize("name,n", [("stack", 8192), ("pile", 2048)])
def test_library_array_more_tiles_than_slots(name, n, oracle_kind, gpu_lib):
    """Without a reservation the step runs on the library's fixed 128 MiB
    array: 8,192 stack worlds (256 tiles) or 2,048 pile worlds (64 tiles)
    need more slots than it has, so one call runs several launches over the
    same slots."""
    cfg = CONFIGS[name]
    slot = engine.workspace_slot_bytes(cfg.caps)
    assert (n + 31) // 32 > (128 << 20) // slot
    o = orc.Oracle(name, oracle_kind)
    stream = torch.cuda.Stream()
    assert engine.reserved_bytes(stream) == 0

    def step(dev, act):
        rc = engine.batch_step_gpu(dev, cfg.dt, cfg.substeps, active=act, stream=stream, caps=cfg.caps,
                                   joint_iters=cfg.joint_iters)
        stream.synchronize()
        return rc

    run_pair(cfg, o, n, 3, 7, step, masked=(name == "pile"))


def test_default_entry_allocates_nothing(oracle_kind, gpu_lib):
    """b3x_batch_step_gpu only enqueues (reference b3_batch.cuh:77-78): the
    first call on a fresh stream leaves the device's free memory unchanged;
    b3x_reserve_workspace is the one call that allocates, and
    b3x_release_workspaces gives the memory back."""
    cfg = CONFIGS["stack"]
    o = orc.Oracle("stack", oracle_kind)
    host = o.build(4096, cfg.scene, 3)
    a = torch.from_numpy(host.copy()).cuda()
    b = torch.from_numpy(host.copy()).cuda()
    warm = torch.cuda.Stream()
    # loads the library's kernels on this device (module memory) first
    assert engine.batch_step_gpu(a, cfg.dt, cfg.substeps, stream=warm, caps=cfg.caps, joint_iters=8) == 0
    torch.cuda.synchronize()
    fresh = torch.cuda.Stream()
    free0, _ = torch.cuda.mem_get_info()
    assert engine.batch_step_gpu(b, cfg.dt, cfg.substeps, stream=fresh, caps=cfg.caps, joint_iters=8) == 0
    torch.cuda.synchronize()
    free1, _ = torch.cuda.mem_get_info()
    assert free1 == free0, (free0, free1)
    # a reservation allocates the workspace, release frees it
    ws = engine.workspace_bytes(cfg.caps)
    assert engine.reserve_workspace(cfg.caps, fresh) == 0
    free2, _ = torch.cuda.mem_get_info()
    assert free0 - free2 >= ws
    assert engine.reserve_workspace(cfg.caps, fresh) == 0     # kept, not grown
    assert torch.cuda.mem_get_info()[0] == free2
    assert engine.batch_step_gpu(b, cfg.dt, cfg.substeps, stream=fresh, caps=cfg.caps, joint_iters=8) == 0
    torch.cuda.synchronize()
    assert engine.release_workspaces() == 0
    assert torch.cuda.mem_get_info()[0] == free0
    # both calls stepped the same worlds the same way as the oracle
    ref = host.copy()
    o.batch_step(ref, cfg.dt, cfg.substeps)
    assert np.array_equal(a.cpu().numpy(), ref)
    o.batch_step(ref, cfg.dt, cfg.substeps)
    assert np.array_equal(b.cpu().numpy(), ref)


def test_streams_sharing_the_library_array_are_ordered(oracle_kind, gpu_lib):
    """Two unreserved streams step different batches with no host
    synchronisation between the calls: their launches on the library's
    array are ordered on the GPU (an event), so both match the oracle."""
    cfg = CONFIGS["stack"]
    o = orc.Oracle("stack", oracle_kind)
    host = o.build(6000, cfg.scene, 17)
    s1, s2 = torch.cuda.Stream(), torch.cuda.Stream()
    a = torch.from_numpy(host.copy()).cuda()
    b = torch.from_numpy(host[::-1].copy()).cuda()
    torch.cuda.synchronize()
    for _ in range(3):
        assert engine.batch_step_gpu(a, cfg.dt, 4, stream=s1, caps=cfg.caps, joint_iters=8) == 0
        assert engine.batch_step_gpu(b, cfg.dt, 4, stream=s2, caps=cfg.caps, joint_iters=8) == 0
    torch.cuda.synchronize()
    ref = host.copy()
    for _ in range(3):
        o.batch_step(ref, cfg.dt, 4)
    assert np.array_equal(a.cpu().numpy(), ref)
    assert np.array_equal(b.cpu().numpy(), ref[::-1])
