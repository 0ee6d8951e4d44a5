"""The per-thread device b3_step of include/puffysics.cuh (one thread steps one
world, the form adapters call from their own kernels) against the reference's
CPU b3_batch_step and against the batched engine.

Bar: as for the batched engine.  Jointless scenes are bit-exact, the whole
AoS world byte for byte, every step; the revolute chain (device atan2f) keeps
identical contact sets and body state within abs/rel 1e-4 after one step and
1e-3 after 60.
"""
import numpy as np
import pytest

import oracle as orc
from gpu_util import TOL_1STEP, TOL_60STEP, Pair, contact_keys, state_close
from puffysics_b200 import engine, layout, synth
from puffysics_b200.configs import CONFIGS, SCENE_CHAIN

pytestmark = pytest.mark.gpu


class ThreadPair(Pair):
    """Pair whose device side steps with the per-thread b3_step launcher."""

    def step(self, step, active=None, contiguous=False):
        import torch
        cfg = self.cfg
        kind, idx, nv = cfg.action
        act_dev = None if active is None else torch.from_numpy(active).cuda()
        n = len(self.host)
        self.o.apply(self.host, cfg.scene, self.seed, self.first, step, active=active)
        if nv:
            assert synth.actions_gpu(self.vals, n, cfg.scene, self.seed, self.first, step) == nv
            assert engine.batch_apply_gpu(self.dev, kind, idx, self.vals, active=act_dev, caps=cfg.caps) == 0
        assert self.o.batch_step(self.host, cfg.dt, cfg.substeps, active=active) == 1
        if contiguous:
            assert active is None
            rc = engine.thread_step_worlds_gpu(cfg.name, self.dev, cfg.dt, cfg.substeps)
        else:
            rc = engine.thread_step_gpu(cfg.name, self.dev, cfg.dt, cfg.substeps, active=act_dev)
        assert rc == 0
        torch.cuda.synchronize()


def check(name, got, want, step):
    cfg = CONFIGS[name]
    if cfg.scene != SCENE_CHAIN:
        if not np.array_equal(got, want):
            bad = np.where((got != want).any(1))[0]
            raise AssertionError("%s: %d worlds differ at step %d (first %d)" % (name, len(bad), step, bad[0]))
        return
    assert contact_keys(got, cfg.caps) == contact_keys(want, cfg.caps), "contact sets differ at step %d" % step
    ok, err = state_close(got, want, cfg.caps, TOL_1STEP if step == 1 else TOL_60STEP)
    assert ok, "state error %.3g at step %d" % (err, step)


@pytest.fixture(scope="module")
def built():
    from puffysics_b200 import build
    build.build()


@pytest.mark.parametrize("name", ["hover", "stack", "chain", "pile", "default", "bounce", "stackil", "chainil",
                                  "bouncenr", "bounceilnr", "hoveruf"])
def test_thread_step_matches_reference(name, oracle_kind, built):
    cfg = CONFIGS[name]
    L = engine.thread_lib(name)
    assert L.b3x_thread_signature() == cfg.signature
    assert L.b3x_thread_joint_iters() == cfg.joint_iters and L.b3x_thread_relax_iters() == cfg.relax_iters
    o = orc.Oracle(name, oracle_kind)
    n = {"pile": 96, "default": 64}.get(name, 256)
    seed = 4242
    p = ThreadPair(cfg, o, o.build(n, cfg.scene, seed), seed)
    for step in range(1, 61):
        p.step(step, contiguous=(step % 2 == 0))
        check(name, p.got(), p.host, step)


def test_thread_step_equals_batched_engine(oracle_kind, built):
    """Both device paths give the same bytes (stack, 40 steps)."""
    import torch
    cfg = CONFIGS["stack"]
    o = orc.Oracle("stack", oracle_kind)
    seed = 77
    init = o.build(200, cfg.scene, seed)
    a = ThreadPair(cfg, o, init, seed)
    b = Pair(cfg, o, init, seed)
    for step in range(1, 41):
        a.step(step)
        b.step(step)
    assert np.array_equal(a.got(), b.got())
    torch.cuda.synchronize()


def test_thread_step_mask_and_embedded_worlds(oracle_kind, built):
    """Worlds embedded in a larger per-environment record (stride > world,
    nonzero offset); masked-out worlds and the bytes around each world are
    untouched."""
    import torch
    cfg = CONFIGS["stack"]
    o = orc.Oracle("stack", oracle_kind)
    n, seed = 97, 13
    wb = layout.world_bytes(*cfg.caps)
    off, stride = 64, wb + 64 + 40
    worlds = o.build(n, cfg.scene, seed)
    rng = np.random.default_rng(1)
    env = rng.integers(0, 256, size=(n, stride), dtype=np.uint8)
    env[:, off:off + wb] = worlds
    active = (rng.random(n) < 0.6).astype(np.uint8)
    dev = torch.from_numpy(env.copy()).cuda()
    act = torch.from_numpy(active).cuda()
    host = env.copy()
    for step in range(1, 6):
        rc = engine.thread_step_gpu("stack", dev, cfg.dt, cfg.substeps, active=act, stride=stride, offset=off,
                                    count=n)
        assert rc == 0
        assert o.batch_step(host, cfg.dt, cfg.substeps, active=active, stride=stride, offset=off, count=n) == 1
    torch.cuda.synchronize()
    got = dev.cpu().numpy()
    assert np.array_equal(got, host)
    assert np.array_equal(got[active == 0], env[active == 0])
    assert np.array_equal(got[:, :off], env[:, :off]) and np.array_equal(got[:, off + wb:], env[:, off + wb:])


def test_thread_step_argument_checks(built):
    """Invalid arguments return cudaErrorInvalidValue and write nothing; dt 0
    and empty batches are no-ops (reference b3_batch.cuh:81-89)."""
    import torch
    cfg = CONFIGS["stack"]
    wb = layout.world_bytes(*cfg.caps)
    dev = torch.zeros((4, wb), dtype=torch.uint8, device="cuda")
    ref = dev.clone()
    assert engine.thread_step_gpu("stack", dev, float("nan"), 4) == 1
    assert engine.thread_step_gpu("stack", dev, -1.0, 4) == 1
    assert engine.thread_step_gpu("stack", dev, 1 / 60, 0) == 1
    assert engine.thread_step_gpu("stack", dev, 1 / 60, 4, stride=wb - 8) == 1
    assert engine.thread_step_gpu("stack", dev, 1 / 60, 4, stride=wb, offset=8) == 1
    assert engine.thread_step_gpu("stack", dev, 0.0, 4) == 0
    assert engine.thread_step_gpu("stack", dev, 1 / 60, 4, count=0) == 0
    torch.cuda.synchronize()
    assert torch.equal(dev, ref)


@pytest.mark.parametrize("name", ["hover", "stack", "chain"])
def test_thread_scene_apply_equals_library_apply(name, built):
    """The per-thread library's one-launch scene actions (the per-thread
    bench leg's input) write the same bytes as the library's action
    generator followed by b3x_batch_apply_gpu, and as the reference's apply
    on the CPU; no launch and no change for a scene without actions."""
    import torch
    cfg = CONFIGS[name]
    kind, idx, nv = cfg.action
    n = 97
    o = orc.Oracle(name, "port")
    host = o.build(n, cfg.scene, 9)
    a = torch.from_numpy(host.copy()).cuda()
    b = a.clone()
    vals = torch.zeros((n, max(nv, 1)), dtype=torch.float32, device="cuda")
    for step in (1, 2):
        assert engine.thread_scene_apply_gpu(name, a, cfg.scene, 9, 0, step) == 0
        assert synth.actions_gpu(vals, n, cfg.scene, 9, 0, step) == nv
        assert engine.batch_apply_gpu(b, kind, idx, vals, caps=cfg.caps) == 0
        o.apply(host, cfg.scene, 9, 0, step)
    torch.cuda.synchronize()
    assert np.array_equal(a.cpu().numpy(), b.cpu().numpy())
    assert np.array_equal(a.cpu().numpy(), host)
    pile = CONFIGS["pile"]
    assert pile.action[2] == 0
    w = torch.from_numpy(orc.Oracle("pile", "port").build(33, pile.scene, 9)).cuda()
    before = w.cpu().numpy()
    assert engine.thread_scene_apply_gpu("pile", w, pile.scene, 9, 0, 1) == 0
    torch.cuda.synchronize()
    assert np.array_equal(w.cpu().numpy(), before)
