"""The articulated contact response (B3_ART_CONTACTS=1) on the GPU.

The reference built with B3_ART_CONTACTS=1 resolves the contacts of worlds
with joints through the articulation of their revolute joints (reference
b3_art.cuh, selected in 08_contacts.inl:194-232 and 424-436).  Here it is
built into the header's per-thread device b3_step when an adapter compiles
with the macro (libb3thread_chainart.so: the chain configuration compiled
with -DB3_ART_CONTACTS=1), and b3_batch_step_gpu then runs that step.

Oracle: the reference's CPU b3_batch_step compiled with the same macro
(oracle/_ref/libb3ref_chainart.so).  The chain reaches the ground after
about 50 steps; the comparison starts from a reference state with the chain
on the ground, so every compared step resolves contacts through the
articulation.  Bar: the revolute chain's tolerances (its joint solver calls
atan2f, whose last bit can differ between CUDA and glibc): contact pair sets
and counts equal after every step, body state within abs/rel 1e-4 after one
step and 1e-3 after 40.
"""
import numpy as np
import pytest
import torch

import oracle as orc
from gpu_util import TOL_1STEP, TOL_60STEP, contact_keys, state_close
from puffysics_b200 import engine, layout, synth
from puffysics_b200.configs import CONFIGS

pytestmark = pytest.mark.gpu
SEED = 5


@pytest.fixture(scope="module")
def landed():
    """Chains after 90 reference steps (all of them on the ground)."""
    if not orc.available("chainart", "ref"):
        pytest.skip("reference build with B3_ART_CONTACTS=1 (oracle/_ref) not present")
    cfg = CONFIGS["chainart"]
    o = orc.Oracle("chainart", "ref")
    w = o.build(96, cfg.scene, SEED)
    for s in range(1, 91):
        o.apply(w, cfg.scene, SEED, 0, s)
        assert o.batch_step(w, cfg.dt, cfg.substeps) == 1
    v = layout.view(w, cfg.caps)
    assert (v["contact_count"] > 0).mean() > 0.5
    return o, w


@pytest.mark.parametrize("entry", ["b3_step", "b3_batch_step_gpu"])
def test_articulated_contacts_match_reference(entry, landed, gpu_lib):
    cfg = CONFIGS["chainart"]
    o, start = landed
    host = start.copy()
    dev = torch.from_numpy(start.copy()).cuda()
    L = engine.thread_lib("chainart")
    kind, idx, nv = cfg.action
    vals = torch.zeros((len(host), nv), dtype=torch.float32, device="cuda")
    art_contacts = 0
    for s in range(91, 131):
        o.apply(host, cfg.scene, SEED, 0, s)
        assert synth.actions_gpu(vals, len(host), cfg.scene, SEED, 0, s) == nv
        assert engine.batch_apply_gpu(dev, kind, idx, vals, caps=cfg.caps) == 0
        assert o.batch_step(host, cfg.dt, cfg.substeps) == 1
        if entry == "b3_step":
            rc = engine.thread_step_gpu("chainart", dev, cfg.dt, cfg.substeps)
        else:
            rc = L.b3x_thread_shim_step_gpu(engine.make_batch(dev), cfg.dt, cfg.substeps, None,
                                            engine._stream(None))
        assert rc == 0
        torch.cuda.synchronize()
        got = dev.cpu().numpy()
        assert contact_keys(got, cfg.caps) == contact_keys(host, cfg.caps), "contact sets differ at step %d" % s
        ok, err = state_close(got, host, cfg.caps, TOL_1STEP if s == 91 else TOL_60STEP)
        assert ok, "state error %.3g at step %d" % (err, s)
        art_contacts += int(layout.view(got, cfg.caps)["contact_count"].sum())
    assert art_contacts > 0


def test_articulated_response_changes_the_step(landed, gpu_lib):
    """The articulated build really resolves contacts differently: from the
    same landed state, one step of the default per-thread step (chain
    library) and of the articulated one (chainart) give different bodies."""
    cfg = CONFIGS["chainart"]
    o, start = landed
    a = torch.from_numpy(start.copy()).cuda()
    b = torch.from_numpy(start.copy()).cuda()
    assert engine.thread_step_gpu("chainart", a, cfg.dt, cfg.substeps) == 0
    assert engine.thread_step_gpu("chain", b, cfg.dt, cfg.substeps) == 0
    torch.cuda.synchronize()
    va, vb = layout.view(a.cpu().numpy(), cfg.caps), layout.view(b.cpu().numpy(), cfg.caps)
    assert not np.array_equal(va["bodies"]["lin_vel"], vb["bodies"]["lin_vel"])
