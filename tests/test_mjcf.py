"""MJCF scene ingestion.  The reference's MJCF loader (mjcf.h) is host code
over the public world-building API, which include/puffysics_b200.h restates
with the same names and struct layouts; an adapter keeps its loader and
compiles it against this library's headers.

CPU: the loader built against include/ spawns byte-identical worlds to the
loader built against the reference's own headers (the bind pose and a
keyframe), and reproduces the committed fixture.  GPU: the ingested robot
steps through the batched engine in agreement with the reference's CPU step
(revolute joints: contact sets exact, state within the chain tolerances).
"""
import os
import sys
import tempfile

import numpy as np
import pytest

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(HERE, "golden"))

import gen_mjcf  # noqa: E402
import oracle as orc  # noqa: E402
from gpu_util import TOL_60STEP, contact_keys, state_close  # noqa: E402
from puffysics_b200 import engine, layout  # noqa: E402
from puffysics_b200.configs import CONFIGS  # noqa: E402

needs_ref = pytest.mark.skipif(not os.path.exists(os.path.join(gen_mjcf.REF_DIR, "mjcf.h")),
                               reason="reference checkout (mjcf.h) not present")
FIXTURE = os.path.join(HERE, "golden", "mjcf_walker.npz")


@needs_ref
def test_loader_against_these_headers_spawns_reference_worlds():
    with tempfile.TemporaryDirectory() as d:
        ours = gen_mjcf.spawn([os.path.join(gen_mjcf.ROOT, "include"), gen_mjcf.REF_DIR], ["-", "crouch"], d)
    with tempfile.TemporaryDirectory() as d:
        ref = gen_mjcf.spawn([gen_mjcf.REF_DIR], ["-", "crouch"], d)
    assert np.array_equal(ours, ref)
    assert np.array_equal(ours, np.load(FIXTURE)["worlds"])


def test_fixture_is_a_default_capacity_world():
    w = np.load(FIXTURE)["worlds"]
    caps = CONFIGS["default"].caps
    assert w.shape[1] == layout.world_bytes(*caps)
    v = layout.view(w, caps)
    assert (v["body_count"] == 7).all() and (v["joint_count"] == 5).all() and (v["shape_count"] == 9).all()


@pytest.mark.gpu
def test_ingested_robot_steps_like_the_reference(oracle_kind, gpu_lib):
    import torch
    cfg = CONFIGS["default"]
    base = np.load(FIXTURE)["worlds"]
    worlds = np.repeat(base, 32, axis=0)
    o = orc.Oracle("default", oracle_kind)
    dev = torch.from_numpy(worlds.copy()).cuda()
    host = worlds.copy()
    for step in range(1, 61):
        assert o.batch_step(host, cfg.dt, cfg.substeps) == 1
        assert engine.batch_step_gpu(dev, cfg.dt, cfg.substeps, caps=cfg.caps, joint_iters=cfg.joint_iters) == 0
        if step in (1, 30, 60):
            torch.cuda.synchronize()
            got = dev.cpu().numpy()
            assert contact_keys(got, cfg.caps) == contact_keys(host, cfg.caps), step
            ok, err = state_close(got, host, cfg.caps, TOL_60STEP)
            assert ok, (step, err)
    v = layout.view(host, cfg.caps)
    assert v["contact_count"].max() > 0          # the feet are on the floor
