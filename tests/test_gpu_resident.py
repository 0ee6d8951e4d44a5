"""Resident world columns (b3x_engine_*): worlds bound from AoS into
structure-of-arrays columns, stepped there, synced back.

Bar: the synced worlds equal the reference's CPU b3_batch_step (reference
b3_batch.cuh:39-48) on the same worlds and actions, byte for byte every step
for the jointless scenes, the revolute chain within the parity tolerances
(atan2f); bind / sync move the selected worlds exactly; a mask leaves worlds
untouched; a reset is a bind of the initial snapshots with the reset mask.
"""
import numpy as np
import pytest
import torch

import oracle as orc
from gpu_util import TOL_1STEP, TOL_60STEP, contact_keys, state_close
from puffysics_b200 import engine, layout, synth
from puffysics_b200.configs import CONFIGS, SCENE_CHAIN

pytestmark = pytest.mark.gpu


def compare(name, got, want, step):
    cfg = CONFIGS[name]
    if cfg.scene != SCENE_CHAIN:
        if not np.array_equal(got, want):
            bad = np.where((got != want).any(1))[0]
            raise AssertionError("%s: %d worlds differ at step %d (first %d)" % (name, len(bad), step, bad[0]))
        return
    assert contact_keys(got, cfg.caps) == contact_keys(want, cfg.caps), "contact sets differ at step %d" % step
    ok, err = state_close(got, want, cfg.caps, TOL_1STEP if step == 1 else TOL_60STEP)
    assert ok, "state error %.3g at step %d" % (err, step)


def rollout(name, n, steps, seed, oracle_kind, masked=False, reset_every=0):
    cfg = CONFIGS[name]
    o = orc.Oracle(name, oracle_kind)
    host = o.build(n, cfg.scene, seed)
    initial = host.copy()
    aos = torch.from_numpy(host.copy()).cuda()
    snap = torch.from_numpy(initial).cuda()
    cols = engine.Columns(cfg.caps, n)
    assert cols.bind(aos) == 0
    kind, idx, nv = cfg.action
    vals = torch.zeros((n, max(nv, 1)), dtype=torch.float32, device="cuda")
    rng = np.random.default_rng(seed)
    for s in range(1, steps + 1):
        mask = (rng.random(n) < 0.6).astype(np.uint8) if masked else None
        act = None if mask is None else torch.from_numpy(mask).cuda()
        if reset_every and s % reset_every == 0:
            reset = (rng.random(n) < 0.2).astype(np.uint8)
            assert o.batch_restore(host, initial, reset) == 1
            assert cols.bind(snap, select=torch.from_numpy(reset).cuda()) == 0
        o.apply(host, cfg.scene, seed, 0, s, active=mask)
        if nv:
            assert synth.actions_gpu(vals, n, cfg.scene, seed, 0, s) == nv
            assert cols.apply(kind, idx, vals, active=act) == 0
        assert o.batch_step(host, cfg.dt, cfg.substeps, active=mask) == 1
        assert cols.step(cfg.dt, cfg.substeps, active=act, joint_iters=cfg.joint_iters,
                         relax_iters=cfg.relax_iters, flags=cfg.flags) == 0
        assert cols.sync_to_aos(aos) == 0
        torch.cuda.synchronize()
        compare(name, aos.cpu().numpy(), host, s)
    assert engine.fault_flags() == 0


@pytest.mark.parametrize("name", ["hover", "stack", "chain", "pile", "bounce", "capsule", "stackil", "default"])
def test_columns_rollout_matches_oracle(name, oracle_kind, gpu_lib):
    n = {"pile": 96, "default": 48, "chain": 128}.get(name, 200)
    rollout(name, n, 30, 4040, oracle_kind)


@pytest.mark.parametrize("name", ["stack", "hover"])
def test_columns_mask_and_resets(name, oracle_kind, gpu_lib):
    """Masked steps leave worlds untouched; every 4th step 20% of the worlds
    are reset by binding the initial snapshots with the reset mask."""
    rollout(name, 163, 16, 77, oracle_kind, masked=True, reset_every=4)


def test_columns_bind_sync_are_exact_and_selective(oracle_kind, gpu_lib):
    """Embedded worlds (stride and offset) round-trip byte for byte; a sync
    with a mask writes only the selected worlds and nothing around them."""
    cfg = CONFIGS["stack"]
    o = orc.Oracle("stack", oracle_kind)
    n = 70
    host = o.build(n, cfg.scene, 5)
    wb = host.shape[1]
    stride, off = wb + 48, 16
    rng = np.random.default_rng(2)
    env = rng.integers(0, 256, size=(n, stride), dtype=np.uint8)
    env[:, off:off + wb] = host
    dev = torch.from_numpy(env.copy()).cuda()
    cols = engine.Columns(cfg.caps, n)
    assert cols.bind(dev, stride=stride, offset=off) == 0
    other = torch.from_numpy(rng.integers(0, 256, size=(n, stride), dtype=np.uint8)).cuda()
    before = other.cpu().numpy()
    mask = (rng.random(n) < 0.5).astype(np.uint8)
    assert cols.sync_to_aos(other, select=torch.from_numpy(mask).cuda(), stride=stride, offset=off) == 0
    torch.cuda.synchronize()
    got = other.cpu().numpy()
    want = before.copy()
    want[mask == 1, off:off + wb] = host[mask == 1]
    assert np.array_equal(got, want)
    # invalid arguments write nothing
    assert cols.bind(dev, stride=wb - 8) == engine.CUDA_ERROR_INVALID_VALUE
    assert engine.lib().b3x_engine_step(None, 4, cfg.dt, 4, None, None, cols.sig, 8, 8, 0) == \
        engine.CUDA_ERROR_INVALID_VALUE
    assert cols.step(float("nan"), 4) == engine.CUDA_ERROR_INVALID_VALUE
    assert cols.step(cfg.dt, 0) == engine.CUDA_ERROR_INVALID_VALUE
    assert cols.step(cfg.dt, 4, flags=8) == engine.CUDA_ERROR_INVALID_VALUE
    assert cols.step(0.0, 4) == 0
    assert cols.sync_to_aos(dev, stride=stride, offset=off) == 0
    torch.cuda.synchronize()
    assert np.array_equal(dev.cpu().numpy(), env)


def test_columns_observe_matches_aos_observe(oracle_kind, gpu_lib):
    cfg = CONFIGS["stack"]
    o = orc.Oracle("stack", oracle_kind)
    host = o.build(100, cfg.scene, 9)
    aos = torch.from_numpy(host.copy()).cuda()
    cols = engine.Columns(cfg.caps, 100)
    assert cols.bind(aos) == 0
    for _ in range(3):
        assert cols.step(cfg.dt, 4, joint_iters=8) == 0
        assert engine.batch_step_gpu(aos, cfg.dt, 4, caps=cfg.caps, joint_iters=8) == 0
    a = torch.zeros((100, 13), dtype=torch.float32, device="cuda")
    b = torch.zeros((100, 13), dtype=torch.float32, device="cuda")
    for body in (0, 4, 8):
        assert cols.observe(body, a) == 0
        assert engine.batch_observe_gpu(aos, body, b, caps=cfg.caps) == 0
        torch.cuda.synchronize()
        assert torch.equal(a, b)


def test_columns_more_tiles_than_workspace_slots(oracle_kind, gpu_lib):
    """8,192 stack worlds (256 tiles) on the library's fixed array run
    several launches over reused slots; the columns equal the AoS path."""
    cfg = CONFIGS["stack"]
    n = 8192
    o = orc.Oracle("stack", oracle_kind)
    host = o.build(n, cfg.scene, 31)
    aos = torch.from_numpy(host.copy()).cuda()
    out = torch.zeros_like(aos)
    stream = torch.cuda.Stream()
    cols = engine.Columns(cfg.caps, n)
    assert cols.bind(aos, stream=stream) == 0
    for _ in range(3):
        assert cols.step(cfg.dt, 4, stream=stream, joint_iters=8) == 0
        o.batch_step(host, cfg.dt, 4)
    assert cols.sync_to_aos(out, stream=stream) == 0
    stream.synchronize()
    assert np.array_equal(out.cpu().numpy(), host)


STATE_ONLY = 4


def defined_words(raw, caps):
    """A copy with the words the reference leaves undefined zeroed: contact
    slots past a world's contact count, point slots past a contact's point
    count (they keep whatever bytes an earlier step left there)."""
    out = raw.copy()
    v = layout.view(out, caps)
    for wi in range(len(out)):
        k = int(v["contact_count"][wi])
        v["contacts"][wi, k:] = np.zeros(1, v["contacts"].dtype)
        for c in range(k):
            pc = int(v["contacts"][wi, c]["point_count"])
            v["contacts"][wi, c]["points"][pc:] = np.zeros(1, v["contacts"]["points"].dtype.base)
    return out


@pytest.mark.parametrize("name", ["stack", "pile", "chain", "capsule"])
def test_state_only_steps_keep_the_trajectory(name, oracle_kind, gpu_lib):
    """Steps with B3X_STEP_STATE_ONLY write back only what later steps read:
    after such steps the bodies, header and warm-start words equal the
    reference's; after a step without the flag every word the reference
    defines does (contact slots past the contact count and point slots past
    the point count hold stale bytes in both and are not compared)."""
    cfg = CONFIGS[name]
    o = orc.Oracle(name, oracle_kind)
    n = 96 if name == "pile" else 160
    host = o.build(n, cfg.scene, 2024)
    aos = torch.from_numpy(host.copy()).cuda()
    cols = engine.Columns(cfg.caps, n)
    assert cols.bind(aos) == 0
    kind, idx, nv = cfg.action
    vals = torch.zeros((n, max(nv, 1)), dtype=torch.float32, device="cuda")
    for s in range(1, 21):
        full = s % 5 == 0
        o.apply(host, cfg.scene, 2024, 0, s)
        if nv:
            assert synth.actions_gpu(vals, n, cfg.scene, 2024, 0, s) == nv
            assert cols.apply(kind, idx, vals) == 0
        assert o.batch_step(host, cfg.dt, cfg.substeps) == 1
        assert cols.step(cfg.dt, cfg.substeps, joint_iters=cfg.joint_iters, relax_iters=cfg.relax_iters,
                         flags=cfg.flags | (0 if full else STATE_ONLY)) == 0
        assert cols.sync_to_aos(aos) == 0
        torch.cuda.synchronize()
        got = aos.cpu().numpy()
        if full:
            compare(name, defined_words(got, cfg.caps), defined_words(host, cfg.caps), s)
            continue
        g, w = layout.view(got, cfg.caps), layout.view(host, cfg.caps)
        assert contact_keys(got, cfg.caps) == contact_keys(host, cfg.caps), "contact sets differ at step %d" % s
        if cfg.scene == SCENE_CHAIN:
            ok, err = state_close(got, host, cfg.caps, TOL_60STEP)
            assert ok, err
            continue
        assert np.array_equal(g["bodies"], w["bodies"]), "bodies differ at step %d" % s
        for f in ("contact_count", "contact_overflow", "contacts_dropped"):
            assert np.array_equal(g[f], w[f])
        for wi in range(n):
            k = int(w["contact_count"][wi])
            gc, wc = g["contacts"][wi, :k], w["contacts"][wi, :k]
            for f in ("friction_impulse", "twist_impulse", "rolling_impulse"):
                assert np.array_equal(gc[f], wc[f]), (s, wi, f)
            for c in range(k):
                pc = int(wc["point_count"][c])
                assert np.array_equal(gc["points"][c, :pc]["normal_impulse"], wc["points"][c, :pc]["normal_impulse"])
    assert engine.fault_flags() == 0
