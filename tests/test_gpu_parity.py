"""Parity of the CUDA engine with the reference's CPU b3_batch_step.

Oracle: the reference's own code (oracle/_ref) when shipped with the tree,
else the restatement (oracle/port, itself pinned bit-exact against the
reference by tests/test_oracle.py), plus the committed golden fixtures.

Bar: jointless scenes (hover, stack, pile, capacity edges) are bit-exact, the
whole AoS world byte for byte, every step.  The revolute chain evaluates
atan2f on the device, whose last bit can differ from glibc's: contact pair
sets and counts must still match exactly after every step, body state within
abs/rel 1e-4 after one step and 1e-3 after 60 steps.
"""
import os

import numpy as np
import pytest

import oracle as orc
from gpu_util import TOL_1STEP, TOL_60STEP, Pair, contact_keys, state_close
from puffysics_b200 import layout
from puffysics_b200.configs import CONFIGS, SCENE_CHAIN

pytestmark = pytest.mark.gpu
GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
EXACT = ["hover", "stack", "pile", "bounce", "capsule"]


def check_step(name, got, want, step):
    cfg = CONFIGS[name]
    if cfg.scene != SCENE_CHAIN:
        if not np.array_equal(got, want):
            bad = np.where((got != want).any(1))[0]
            raise AssertionError("%s: %d worlds differ at step %d (first %d)" % (name, len(bad), step, bad[0]))
        return
    assert contact_keys(got, cfg.caps) == contact_keys(want, cfg.caps), "contact sets differ at step %d" % step
    ok, err = state_close(got, want, cfg.caps, TOL_1STEP if step == 1 else TOL_60STEP)
    assert ok, "state error %.3g at step %d" % (err, step)


@pytest.mark.parametrize("name", ["hover", "stack", "chain", "pile", "bounce", "capsule"])
def test_golden_fixtures(name, gpu_lib):
    cfg = CONFIGS[name]
    g = np.load(os.path.join(GOLDEN, name + ".npz"))
    kind = "ref" if orc.available(name, "ref") else "port"
    p = Pair(cfg, orc.Oracle(name, kind), g["init"], int(g["seed"]))
    for step in range(1, 61):
        p.step(step)
        if step == 1:
            check_step(name, p.got(), g["step1"], 1)
        if step == 60:
            check_step(name, p.got(), g["step60"], 60)


@pytest.mark.parametrize("name", ["hover", "stack", "chain", "pile", "default", "stacksmall", "bounce", "capsule"])
def test_rollout_matches_oracle_every_step(name, oracle_kind, gpu_lib):
    cfg = CONFIGS[name]
    o = orc.Oracle(name, oracle_kind)
    n = {"pile": 96, "default": 64}.get(name, 256)
    seed = 31337
    p = Pair(cfg, o, o.build(n, cfg.scene, seed), seed)
    for step in range(1, 61):
        p.step(step)
        check_step(name, p.got(), p.host, step)
    if name == "stacksmall":
        v = layout.view(p.got(), cfg.caps)
        assert (v["contact_overflow"] == 1).any() and v["contacts_dropped"].sum() > 0


@pytest.mark.parametrize("name", ["stackil", "chainil", "bouncenr", "bounceilnr"])
def test_step_modes_match_oracle(name, oracle_kind, gpu_lib):
    """The reference's B3_INTERLEAVE_CONTACTS / B3_SKIP_RESTITUTION modes
    (b3x_batch_step_gpu_flags) against the reference built with them."""
    cfg = CONFIGS[name]
    o = orc.Oracle(name, oracle_kind)
    seed = 808
    p = Pair(cfg, o, o.build(128, cfg.scene, seed), seed)
    for step in range(1, 41):
        p.step(step)
        check_step(name, p.got(), p.host, step)


@pytest.mark.parametrize("n", [1, 31, 33, 4097])
def test_odd_batch_sizes(n, oracle_kind, gpu_lib):
    cfg = CONFIGS["stack"]
    o = orc.Oracle("stack", oracle_kind)
    p = Pair(cfg, o, o.build(n, cfg.scene, 5), 5)
    for step in range(1, 4):
        p.step(step)
        check_step("stack", p.got(), p.host, step)


def test_long_chain_rollout_statistics(oracle_kind, gpu_lib):
    """240 steps of the chain: report and bound the atan2f-driven drift."""
    cfg = CONFIGS["chain"]
    o = orc.Oracle("chain", oracle_kind)
    p = Pair(cfg, o, o.build(128, cfg.scene, 8), 8)
    for step in range(1, 241):
        p.step(step)
    got, want = p.got(), p.host
    same = np.mean([a == b for a, b in zip(contact_keys(got, cfg.caps), contact_keys(want, cfg.caps))])
    ok, err = state_close(got, want, cfg.caps, 1e-2)
    assert same >= 0.95, same
    assert err < 0.05, err
