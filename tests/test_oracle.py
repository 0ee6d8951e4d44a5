"""CPU tests of the parity oracles (no GPU).

The restatement (oracle/port) is pinned against golden fixtures that the
reference's own code produced (tests/golden/gen_golden.py) and, where the
reference build is present, against the reference directly.
"""
import os

import numpy as np
import pytest

import oracle as orc
from puffysics_b200 import layout
from puffysics_b200.configs import CONFIGS

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
ROLLOUT_CONFIGS = ["hover", "stack", "chain", "pile", "bounce", "capsule"]
have_ref = orc.available("stack", "ref")
needs_ref = pytest.mark.skipif(not have_ref, reason="reference build (oracle/_ref) not present")


def load_golden(name):
    return np.load(os.path.join(GOLDEN, name + ".npz"))


def replay(o, cfg, init, seed, steps, keep=(1, 60)):
    w = init.copy()
    out = {}
    for step in range(1, steps + 1):
        o.apply(w, cfg.scene, seed, 0, step)
        assert o.batch_step(w, cfg.dt, cfg.substeps) == 1
        if step in keep:
            out[step] = w.copy()
    return out


@pytest.fixture(scope="module")
def port_built():
    assert orc.build_oracles() == 0
    return True


@pytest.mark.parametrize("name", ROLLOUT_CONFIGS)
def test_port_reproduces_reference_golden(name, port_built):
    cfg = CONFIGS[name]
    g = load_golden(name)
    o = orc.Oracle(name, "port")
    seed = int(g["seed"])
    built = o.build(len(g["init"]), cfg.scene, seed)
    assert np.array_equal(built, g["init"]), "scene builders differ from the reference's"
    out = replay(o, cfg, g["init"], seed, 60)
    assert np.array_equal(out[1], g["step1"])
    assert np.array_equal(out[60], g["step60"])


@needs_ref
@pytest.mark.parametrize("name", ROLLOUT_CONFIGS)
def test_reference_reproduces_golden(name):
    cfg = CONFIGS[name]
    g = load_golden(name)
    out = replay(orc.Oracle(name, "ref"), cfg, g["init"], int(g["seed"]), 60)
    assert np.array_equal(out[1], g["step1"]) and np.array_equal(out[60], g["step60"])


MODE_CONFIGS = ["stackil", "chainil", "bouncenr", "bounceilnr", "hoveruf"]


@needs_ref
@pytest.mark.parametrize("name", ROLLOUT_CONFIGS + ["default", "stacksmall"] + MODE_CONFIGS)
def test_port_equals_reference_rollout(name, port_built):
    cfg = CONFIGS[name]
    ref, port = orc.Oracle(name, "ref"), orc.Oracle(name, "port")
    n, seed = (16, 99) if name in ("pile", "default") else (48, 99)
    wr, wp = ref.build(n, cfg.scene, seed), port.build(n, cfg.scene, seed)
    assert np.array_equal(wr, wp)
    for step in range(1, 41):
        ref.apply(wr, cfg.scene, seed, 0, step)
        port.apply(wp, cfg.scene, seed, 0, step)
        ref.batch_step(wr, cfg.dt, cfg.substeps)
        port.batch_step(wp, cfg.dt, cfg.substeps)
        assert np.array_equal(wr, wp), "diverged at step %d" % step


def test_overflow_flags_in_oracle(port_built):
    cfg = CONFIGS["stacksmall"]
    o = orc.Oracle("stacksmall", "port")
    w = o.build(8, cfg.scene, 5)
    o.batch_step(w, cfg.dt, cfg.substeps)
    v = layout.view(w, cfg.caps)
    assert (v["contact_count"] == 4).all()
    assert (v["contact_overflow"] == 1).all() and (v["contacts_dropped"] > 0).all()


def test_manifold_known_answers(port_built):
    k = np.load(os.path.join(GOLDEN, "kats.npz"))
    o = orc.Oracle("hovertask", "port")
    for i, w in enumerate(k["worlds"]):
        cnt, normal, pa, pb, sep, feat = o.collide(w, 0, 1)
        assert cnt == k["count"][i], i
        if cnt:
            assert np.array_equal(normal, k["normal"][i]), i
            assert np.array_equal(pa, k["pa"][i][:cnt]) and np.array_equal(pb, k["pb"][i][:cnt]), i
            assert np.array_equal(sep, k["sep"][i][:cnt]) and np.array_equal(feat, k["feature"][i][:cnt]), i


def test_known_answers_cover_every_pair_type():
    k = np.load(os.path.join(GOLDEN, "kats.npz"))
    v = layout.view(k["worlds"], tuple(k["caps"]))
    types = set()
    for i in range(len(v)):
        if k["count"][i]:
            types.add(tuple(sorted(v["shapes"]["type"][i][:2])))
    assert types == {(a, b) for a in range(3) for b in range(a, 3)}
    feats = set(k["feature"][k["count"] > 0].ravel().tolist())
    assert {1, 2, 3, 4, 5} <= feats and any(16 <= f < 24 for f in feats)


@pytest.mark.parametrize("kind", ["port"] + (["ref"] if have_ref else []))
def test_batch_validation_without_mutation(kind, port_built):
    cfg = CONFIGS["stack"]
    o = orc.Oracle("stack", kind)
    w = o.build(4, cfg.scene, 1)
    before = w.copy()
    wb = o.world_bytes
    assert o.batch_step(w, float("nan"), 4) == 0
    assert o.batch_step(w, -1.0, 4) == 0
    assert o.batch_step(w, 1 / 60, 0) == 0
    assert o.batch_step(w, 1 / 60, 4, stride=wb - 8) == 0
    assert o.batch_step(w, 1 / 60, 4, count=-1) == 0
    assert np.array_equal(w, before)
    assert o.batch_step(w, 0.0, 4) == 1 and np.array_equal(w, before)
    mask = np.array([1, 0, 1, 0], np.uint8)
    assert o.batch_step(w, 1 / 60, 4, active=mask) == 1
    assert np.array_equal(w[1], before[1]) and np.array_equal(w[3], before[3])
    assert not np.array_equal(w[0], before[0])


@needs_ref
@pytest.mark.parametrize("mode,plain", [("stackil", "stack"), ("bouncenr", "bounce"), ("hoveruf", "hover")])
def test_step_modes_change_the_trajectory(mode, plain):
    """The mode builds really run another step: their worlds leave the
    default mode's after a few steps."""
    cfg = CONFIGS[mode]
    a, b = orc.Oracle(mode, "ref"), orc.Oracle(plain, "ref")
    w = a.build(16, cfg.scene, 5)
    wa, wb = w.copy(), w.copy()
    for step in range(1, 6):
        a.apply(wa, cfg.scene, 5, 0, step)
        b.apply(wb, cfg.scene, 5, 0, step)
        a.batch_step(wa, cfg.dt, cfg.substeps)
        b.batch_step(wb, cfg.dt, cfg.substeps)
    assert not np.array_equal(wa, wb)


@needs_ref
def test_articulated_contact_build_changes_the_trajectory():
    """The B3_ART_CONTACTS=1 reference build (the oracle of the articulated
    contact response) leaves the default chain's trajectory once the chain
    touches the ground, and not before."""
    cfg = CONFIGS["chainart"]
    a, b = orc.Oracle("chainart", "ref"), orc.Oracle("chain", "ref")
    w = a.build(8, cfg.scene, 5)
    wa, wb = w.copy(), w.copy()
    for step in range(1, 121):
        a.apply(wa, cfg.scene, 5, 0, step)
        b.apply(wb, cfg.scene, 5, 0, step)
        a.batch_step(wa, cfg.dt, cfg.substeps)
        b.batch_step(wb, cfg.dt, cfg.substeps)
        if step == 20:
            assert np.array_equal(wa, wb)
    assert not np.array_equal(wa, wb)
