"""Generate the golden fixtures of tests/golden/ from the reference itself.

    python tests/golden/gen_golden.py [name ...]   # needs oracle/_ref (make -C oracle REF_DIR=...)

The reference ships no tests or golden vectors for its stepping path, so the
fixtures are outputs of the reference's own CPU code (b3_batch_step from
b3_batch.cuh / puffysics.cuh, compiled here into oracle/_ref) on the seeded
scenes of puffysics_b200/scenes/b3_scenes.h:

  <cfg>.npz   init / step1 / step60: AoS world bytes of a few worlds before,
              after 1 and after 60 steps, each step preceded by the scene's
              generated actions (seed SEED, world indices 0..n-1).
  kats.npz    narrowphase known answers: two-shape worlds (hovertask
              capacities 2/2/4/2) in touching, overlapping, edge and separated
              poses for every shape pair type, with the reference manifold.
"""
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(ROOT, "oracle"))

from oracle import Oracle  # noqa: E402
from puffysics_b200 import layout  # noqa: E402
from puffysics_b200.configs import CONFIGS  # noqa: E402

SEED = 20261201
WORLDS = {"hover": 8, "stack": 8, "chain": 8, "pile": 4, "bounce": 8, "capsule": 8}


def rollout(name):
    cfg = CONFIGS[name]
    orc = Oracle(name, "ref")
    n = WORLDS[name]
    w = orc.build(n, cfg.scene, SEED)
    init = w.copy()
    out = {}
    for step in range(1, 61):
        orc.apply(w, cfg.scene, SEED, 0, step)
        assert orc.batch_step(w, cfg.dt, cfg.substeps) == 1
        if step in (1, 60):
            out["step%d" % step] = w.copy()
    np.savez_compressed(os.path.join(HERE, name + ".npz"), init=init, step1=out["step1"], step60=out["step60"],
                        seed=SEED, caps=np.array(cfg.caps), dt=cfg.dt, substeps=cfg.substeps,
                        joint_iters=cfg.joint_iters)


def quat(axis, angle):
    axis = np.asarray(axis, np.float64)
    axis = axis / np.linalg.norm(axis)
    s = np.sin(angle / 2)
    return np.array([axis[0] * s, axis[1] * s, axis[2] * s, np.cos(angle / 2)], np.float32)


def kat_world(caps, a, b):
    """Two dynamic bodies at the origin-relative poses a, b = (type, pos,
    quat, radius, half)."""
    raw = np.zeros((1, layout.world_bytes(*caps)), np.uint8)
    v = layout.view(raw, caps)[0]
    v["body_count"] = 2
    v["shape_count"] = 2
    for k, (typ, pos, q, rad, half) in enumerate((a, b)):
        v["bodies"]["position"][k] = pos
        v["bodies"]["rotation"][k] = q
        v["bodies"]["center"][k] = pos
        v["bodies"]["delta_rot"][k] = [0, 0, 0, 1]
        v["bodies"]["type"][k] = 2
        v["bodies"]["flags"][k] = 0x1000
        v["shapes"]["body"][k] = k
        v["shapes"]["type"][k] = typ
        v["shapes"]["local_rot"][k] = [0, 0, 0, 1]
        v["shapes"]["radius"][k] = rad
        v["shapes"]["half"][k] = half
        v["shapes"]["category"][k] = ~np.uint64(0)
        v["shapes"]["mask"][k] = ~np.uint64(0)
    return raw[0]


def kats():
    orc = Oracle("hovertask", "ref")
    caps = (2, 2, 4, 2)
    rng = np.random.default_rng(SEED)
    S, C, B = 0, 1, 2
    worlds = []
    for ta in (S, C, B):
        for tb in (S, C, B):
            for trial in range(6):
                ra, rb = 0.3 + 0.2 * rng.random(2)
                ha = (0.2 + 0.4 * rng.random(3)).astype(np.float32)
                hb = (0.2 + 0.4 * rng.random(3)).astype(np.float32)
                if ta == C:
                    ha = np.array([0, 0.2 + 0.3 * rng.random(), 0], np.float32)
                if tb == C:
                    hb = np.array([0, 0.2 + 0.3 * rng.random(), 0], np.float32)
                qa = quat(rng.normal(size=3), rng.uniform(0, np.pi)) if trial % 3 else quat([0, 1, 0], 0.0)
                qb = quat(rng.normal(size=3), rng.uniform(0, np.pi)) if trial % 2 else quat([0, 1, 0], 0.0)
                d = rng.normal(size=3)
                d /= np.linalg.norm(d)
                reach = (ra if ta != B else np.linalg.norm(ha)) + (rb if tb != B else np.linalg.norm(hb))
                dist = reach * (0.55, 0.8, 0.95, 1.0, 1.02, 0.3)[trial]
                pa = np.zeros(3, np.float32)
                pb = (d * dist).astype(np.float32)
                worlds.append(kat_world(caps, (ta, pa, qa, ra, ha), (tb, pb, qb, rb, hb)))
    worlds = np.stack(worlds)
    res = [orc.collide(w, 0, 1) for w in worlds]
    counts = np.array([r[0] for r in res], np.int32)
    normal = np.stack([r[1] for r in res])
    pa = np.zeros((len(res), 4, 3), np.float32)
    pb = np.zeros((len(res), 4, 3), np.float32)
    sep = np.zeros((len(res), 4), np.float32)
    feat = np.zeros((len(res), 4), np.uint32)
    for i, r in enumerate(res):
        pa[i, :r[0]] = r[2]
        pb[i, :r[0]] = r[3]
        sep[i, :r[0]] = r[4]
        feat[i, :r[0]] = r[5]
    np.savez_compressed(os.path.join(HERE, "kats.npz"), worlds=worlds, count=counts, normal=normal, pa=pa, pb=pb,
                        sep=sep, feature=feat, caps=np.array(caps))
    return counts


if __name__ == "__main__":
    names = sys.argv[1:] or list(WORLDS) + ["kats"]
    for name in names:
        if name == "kats":
            c = kats()
            print("kats:", len(c), "with contact:", int((c > 0).sum()))
        else:
            rollout(name)
