"""Every narrowphase pair type on the GPU against the reference.

The 54 known answers of tests/golden/kats.npz (two shapes, every pair type
of sphere / capsule / box, in touching, overlapping, edge and separated
poses; manifolds computed by the reference's b3_collide_pair, reference
src/puffysics/05_collision.inl:472-534) are stepped once, as worlds, through
the three device paths that generate contacts: the tile step of the batched
engine (worlds re-laid at the box-stack capacities), the small-world step
(the known answers' own capacities 2/2/4/2) and the header's per-thread
b3_step.  Each result must equal the reference's CPU step byte for byte, and
its contact the known answer's manifold (count, normal, features).  The
capsule scene's rollouts then exercise sphere-capsule and capsule-capsule
contacts under the solver for 60 steps.
"""
import os

import numpy as np
import pytest
import torch

import oracle as orc
from puffysics_b200 import engine, layout
from puffysics_b200.configs import CONFIGS, SCENE_HOVER, SCENE_STACK

pytestmark = pytest.mark.gpu
GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")
KAT_CAPS = (2, 2, 4, 2)
DT, SUBSTEPS = 1.0 / 60.0, 4
TYPES = {0: "sphere", 1: "capsule", 2: "box"}


def kat_worlds(o, caps, scene):
    """The known answers' two bodies and shapes in worlds of `caps` whose
    header comes from a seeded scene world (b3_world_init values); the
    bodies get unit mass and an isotropic inverse inertia of 2."""
    k = np.load(os.path.join(GOLDEN, "kats.npz"))
    kv = layout.view(k["worlds"], KAT_CAPS)
    n = len(k["worlds"])
    out = np.repeat(o.build(1, scene, 1), n, 0)
    v = layout.view(out, caps)
    v["body_count"], v["shape_count"], v["contact_count"], v["joint_count"] = 2, 2, 0, 0
    v["bodies"][:, :2] = kv["bodies"][:, :2]
    v["shapes"][:, :2] = kv["shapes"][:, :2]
    v["bodies"]["inv_mass"][:, :2] = 1.0
    v["bodies"]["inv_inertia"][:, :2] = 2.0
    v["bodies"]["inv_i_world"][:, :2] = 2.0 * np.eye(3, dtype=np.float32)
    return out, k


def check_against_answers(got, caps, k):
    """The stepped worlds' contacts are the known manifolds; returns the
    pair types that produced one."""
    v = layout.view(got, caps)
    sv = v["shapes"]["type"]
    seen = set()
    for i in range(len(got)):
        cnt = int(k["count"][i])
        if cnt == 0:
            continue
        assert v["contact_count"][i] == 1, i
        c = v["contacts"][i, 0]
        assert (c["shape_a"], c["shape_b"], c["point_count"]) == (0, 1, cnt), i
        assert np.array_equal(c["normal"], k["normal"][i]), i
        assert np.array_equal(c["points"]["feature"][:cnt], k["feature"][i][:cnt]), i
        seen.add(tuple(sorted((TYPES[int(sv[i, 0])], TYPES[int(sv[i, 1])]))))
    return seen


ALL_PAIRS = {tuple(sorted((a, b))) for a in TYPES.values() for b in TYPES.values()}


@pytest.mark.parametrize("path", ["tile", "small", "per_thread"])
def test_every_pair_type_matches_reference(path, oracle_kind, gpu_lib):
    if path == "tile":
        cfg = CONFIGS["stack"]
        caps, o, scene = cfg.caps, orc.Oracle("stack", oracle_kind), SCENE_STACK
    else:
        caps, o, scene = KAT_CAPS, orc.Oracle("hovertask", oracle_kind), SCENE_HOVER
    worlds, k = kat_worlds(o, caps, scene)
    dev = torch.from_numpy(worlds.copy()).cuda()
    if path == "tile":
        assert engine.step_launches(caps, len(worlds)) >= 1 and engine.step_launches(caps, 1 << 20) > 1
        rc = engine.batch_step_gpu(dev, DT, SUBSTEPS, caps=caps, joint_iters=o.joint_iters,
                                   relax_iters=o.relax_iters)
    elif path == "small":
        assert engine.step_launches(caps, 1 << 20) == 1     # the small-world kernel
        rc = engine.batch_step_gpu(dev, DT, SUBSTEPS, caps=caps, joint_iters=o.joint_iters,
                                   relax_iters=o.relax_iters)
    else:
        rc = engine.thread_step_gpu("hovertask", dev, DT, SUBSTEPS)
    assert rc == 0
    torch.cuda.synchronize()
    assert o.batch_step(worlds, DT, SUBSTEPS) == 1
    got = dev.cpu().numpy()
    for i in range(len(got)):
        assert np.array_equal(got[i], worlds[i]), "known answer %d differs from the reference step" % i
    assert check_against_answers(got, caps, k) == ALL_PAIRS


def pair_types(raw, caps):
    v = layout.view(raw, caps)
    st = v["shapes"]["type"]
    out = {}
    for w in range(len(raw)):
        for c in v["contacts"][w, :int(v["contact_count"][w])]:
            key = tuple(sorted((TYPES[int(st[w, c["shape_a"]])], TYPES[int(st[w, c["shape_b"]])])))
            out[key] = out.get(key, 0) + 1
    return out


@pytest.mark.parametrize("path", ["batched", "per_thread"])
def test_capsule_scene_rollout(path, oracle_kind, gpu_lib):
    """Capsules and spheres falling into a walled bin: 60 steps, byte-equal
    to the reference every step, with sphere-capsule and capsule-capsule
    contacts along the way."""
    cfg = CONFIGS["capsule"]
    o = orc.Oracle("capsule", oracle_kind)
    host = o.build(128, cfg.scene, 606)
    dev = torch.from_numpy(host.copy()).cuda()
    seen = {}
    for s in range(1, 61):
        assert o.batch_step(host, cfg.dt, cfg.substeps) == 1
        if path == "batched":
            rc = engine.batch_step_gpu(dev, cfg.dt, cfg.substeps, caps=cfg.caps, joint_iters=cfg.joint_iters)
        else:
            rc = engine.thread_step_gpu("capsule", dev, cfg.dt, cfg.substeps)
        assert rc == 0
        torch.cuda.synchronize()
        got = dev.cpu().numpy()
        if not np.array_equal(got, host):
            bad = np.where((got != host).any(1))[0]
            raise AssertionError("%d worlds differ at step %d (first %d)" % (len(bad), s, bad[0]))
        for key, c in pair_types(got, cfg.caps).items():
            seen[key] = seen.get(key, 0) + c
    assert seen.get(("capsule", "capsule"), 0) > 0 and seen.get(("capsule", "sphere"), 0) > 0, seen
    assert seen.get(("box", "capsule"), 0) > 0 and seen.get(("sphere", "sphere"), 0) > 0, seen
