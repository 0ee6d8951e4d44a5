"""Boundary semantics of the C-ABI on the GPU, mirroring the reference batch
contract (b3_batch.cuh:19-99): validation without mutation, no-op cases,
masks, worlds embedded in caller structs, restore, actions, caller-owned
workspaces and independent streams."""
import numpy as np
import pytest
import torch

import oracle as orc
from gpu_util import Pair
from puffysics_b200 import engine, layout, synth
from puffysics_b200.configs import CONFIGS

pytestmark = pytest.mark.gpu
STACK = CONFIGS["stack"]


@pytest.fixture
def stack_pair(oracle_kind, gpu_lib):
    o = orc.Oracle("stack", oracle_kind)
    return o, o.build(64, STACK.scene, 11)


def step(dev, cfg=STACK, **kw):
    args = dict(caps=cfg.caps, joint_iters=cfg.joint_iters)
    args.update(kw)
    dt = args.pop("dt", cfg.dt)
    subs = args.pop("substeps", cfg.substeps)
    rc = engine.batch_step_gpu(dev, dt, subs, **args)
    torch.cuda.synchronize()
    return rc


def test_invalid_arguments_return_invalid_value_and_write_nothing(stack_pair):
    o, host = stack_pair
    dev = torch.from_numpy(host.copy()).cuda()
    wb = host.shape[1]
    bad = [dict(dt=float("nan")), dict(dt=float("inf")), dict(dt=-1e-3), dict(substeps=0), dict(substeps=-3),
           dict(stride=wb - 8), dict(count=-1), dict(offset=16), dict(joint_iters=0), dict(relax_iters=0),
           dict(caps=(0, 9, 32, 1)), dict(stride=wb + 4, count=1)]
    for kw in bad:
        assert step(dev, **kw) == engine.CUDA_ERROR_INVALID_VALUE, kw
    assert engine.batch_step_gpu(0, STACK.dt, 4, caps=STACK.caps, stride=wb, count=3) == 1   # NULL data
    torch.cuda.synchronize()
    assert np.array_equal(dev.cpu().numpy(), host)


def test_noop_cases(stack_pair):
    o, host = stack_pair
    dev = torch.from_numpy(host.copy()).cuda()
    assert step(dev, dt=0.0) == 0
    assert step(dev, count=0) == 0
    assert engine.batch_step_gpu(0, STACK.dt, 4, caps=STACK.caps, stride=0, count=0) == 0
    assert np.array_equal(dev.cpu().numpy(), host)


def test_active_mask(stack_pair):
    o, host = stack_pair
    rng = np.random.default_rng(3)
    p = Pair(STACK, o, host, 11)
    for s in range(1, 6):
        mask = (rng.random(len(host)) < 0.5).astype(np.uint8)
        before = p.got()
        p.step(s, active=mask)
        got = p.got()
        assert np.array_equal(got, p.host)
        assert np.array_equal(got[mask == 0], before[mask == 0])


def test_worlds_embedded_in_caller_structs(stack_pair):
    """Env = 24-byte prefix + B3World + 40-byte suffix (stride and offset as
    in the reference's embedded-world example); bytes outside the worlds stay."""
    o, host = stack_pair
    n, wb = host.shape
    stride, off = wb + 64, 24
    env = np.random.default_rng(1).integers(0, 256, size=(n, stride), dtype=np.uint8)
    env[:, off:off + wb] = host
    dev = torch.from_numpy(env.copy()).cuda()
    ref = env.copy()
    for s in range(1, 4):
        o.apply(ref, STACK.scene, 11, 0, s, stride=stride, offset=off)
        o.batch_step(ref, STACK.dt, STACK.substeps, stride=stride, offset=off)
        vals = torch.from_numpy(synth.SceneLib(STACK).actions(n, 11, 0, s)).cuda()
        assert engine.batch_apply_gpu(dev, engine.ACTION_LINEAR_IMPULSE, 8, vals, caps=STACK.caps,
                                      stride=stride, offset=off) == 0
        assert step(dev, stride=stride, offset=off) == 0
    assert np.array_equal(dev.cpu().numpy(), ref)


def test_restore_selected_worlds(stack_pair):
    o, host = stack_pair
    n = len(host)
    dev = torch.from_numpy(host.copy()).cuda()
    for _ in range(3):
        assert step(dev) == 0
    stepped = dev.cpu().numpy()
    initial = torch.from_numpy(host.copy()).cuda()
    reset = (np.arange(n) % 3 == 0).astype(np.uint8)
    assert engine.batch_restore_gpu(dev, initial, torch.from_numpy(reset).cuda(), caps=STACK.caps) == 0
    torch.cuda.synchronize()
    got = dev.cpu().numpy()
    assert np.array_equal(got[reset == 1], host[reset == 1])
    assert np.array_equal(got[reset == 0], stepped[reset == 0])
    assert engine.batch_restore_gpu(dev, None, None, caps=STACK.caps) == engine.CUDA_ERROR_INVALID_VALUE
    assert engine.batch_restore_gpu(dev, initial, None, caps=STACK.caps) == 0
    torch.cuda.synchronize()
    assert np.array_equal(dev.cpu().numpy(), host)


@pytest.mark.parametrize("kind,index,nv", [(0, 3, 3), (1, 2, 6), (2, 8, 3)])
def test_body_actions_match_per_world_api(kind, index, nv, stack_pair):
    o, host = stack_pair
    vals = np.random.default_rng(kind).normal(size=(len(host), nv)).astype(np.float32)
    ref = host.copy()
    o.apply_values(ref, kind, index, vals)
    dev = torch.from_numpy(host.copy()).cuda()
    assert engine.batch_apply_gpu(dev, kind, index, torch.from_numpy(vals).cuda(), caps=STACK.caps) == 0
    torch.cuda.synchronize()
    assert np.array_equal(dev.cpu().numpy(), ref)


def test_joint_target_action(oracle_kind, gpu_lib):
    cfg = CONFIGS["chain"]
    o = orc.Oracle("chain", oracle_kind)
    host = o.build(16, cfg.scene, 2)
    vals = np.random.default_rng(0).uniform(-5, 5, size=(16, 9)).astype(np.float32)
    ref = host.copy()
    o.apply_values(ref, 3, 1, vals)
    dev = torch.from_numpy(host.copy()).cuda()
    assert engine.batch_apply_gpu(dev, 3, 1, torch.from_numpy(vals).cuda(), caps=cfg.caps) == 0
    torch.cuda.synchronize()
    assert np.array_equal(dev.cpu().numpy(), ref)


def test_caller_workspace(stack_pair):
    """b3x_batch_step_gpu_ws never allocates: a full-size caller workspace and
    one with only a few slots (fewer persistent CTAs) give identical worlds; a
    workspace smaller than one slot is rejected."""
    o, host = stack_pair
    full = engine.workspace_bytes(STACK.caps)
    assert full > 0
    a = torch.from_numpy(host.copy()).cuda()
    b = torch.from_numpy(host.copy()).cuda()
    c = torch.from_numpy(host.copy()).cuda()
    ws = torch.empty(full, dtype=torch.uint8, device="cuda")
    few = torch.empty(full // 100, dtype=torch.uint8, device="cuda")
    for _ in range(3):
        assert step(a) == 0
        assert step(b, workspace=ws) == 0
        assert step(c, workspace=few) == 0
    assert np.array_equal(a.cpu().numpy(), b.cpu().numpy())
    assert np.array_equal(a.cpu().numpy(), c.cpu().numpy())
    tiny = torch.empty(256, dtype=torch.uint8, device="cuda")
    assert step(a, workspace=tiny) == engine.CUDA_ERROR_INVALID_VALUE


def test_independent_streams(stack_pair):
    o, host = stack_pair
    s1, s2 = torch.cuda.Stream(), torch.cuda.Stream()
    a = torch.from_numpy(host.copy()).cuda()
    b = torch.from_numpy(host[::-1].copy()).cuda()
    torch.cuda.synchronize()
    for _ in range(4):
        assert engine.batch_step_gpu(a, STACK.dt, 4, stream=s1, caps=STACK.caps, joint_iters=8) == 0
        assert engine.batch_step_gpu(b, STACK.dt, 4, stream=s2, caps=STACK.caps, joint_iters=8) == 0
    torch.cuda.synchronize()
    ref = host.copy()
    for _ in range(4):
        o.batch_step(ref, STACK.dt, 4)
    assert np.array_equal(a.cpu().numpy(), ref)
    assert np.array_equal(b.cpu().numpy(), ref[::-1])


def test_corrupt_counts_are_clamped_not_faulting(stack_pair):
    """Counts above the capacities or negative (undefined in the reference)
    must not fault: the engine clamps them to [0, capacity]."""
    o, host = stack_pair
    h = host[:4].copy()
    v = layout.view(h, STACK.caps)
    v["body_count"][0] = 1000
    v["shape_count"][1] = -5
    v["contact_count"][2] = 99
    v["joint_count"][3] = 77
    dev = torch.from_numpy(h).cuda()
    assert step(dev) == 0
    out = layout.view(dev.cpu().numpy(), STACK.caps)
    assert out["contact_count"][1] == 0


@pytest.mark.parametrize("n", [1, 33, 997])
def test_small_world_path_mask_and_embedding(n, oracle_kind, gpu_lib):
    """Hover worlds take the small-world step (whole worlds staged in shared
    memory, one thread per world): embedded worlds with a mask and a ragged
    last tile match the reference; masked-out worlds and the bytes around
    every world are untouched."""
    cfg = CONFIGS["hover"]
    assert engine.step_launches(cfg.caps, n) == 1
    o = orc.Oracle("hover", oracle_kind)
    host = o.build(n, cfg.scene, 21)
    wb = host.shape[1]
    stride, off = wb + 48, 16
    rng = np.random.default_rng(n)
    env = rng.integers(0, 256, size=(n, stride), dtype=np.uint8)
    env[:, off:off + wb] = host
    dev = torch.from_numpy(env.copy()).cuda()
    ref = env.copy()
    for s in range(1, 8):
        mask = (rng.random(n) < 0.7).astype(np.uint8)
        o.batch_step(ref, cfg.dt, cfg.substeps, active=mask, stride=stride, offset=off)
        rc = engine.batch_step_gpu(dev, cfg.dt, cfg.substeps, active=torch.from_numpy(mask).cuda(), caps=cfg.caps,
                                   joint_iters=cfg.joint_iters, stride=stride, offset=off)
        assert rc == 0
    torch.cuda.synchronize()
    assert np.array_equal(dev.cpu().numpy(), ref)
