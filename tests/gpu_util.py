"""Shared helpers of the GPU tests: drive the CUDA engine and an oracle side
by side on the same seeded worlds and actions."""
import numpy as np

from puffysics_b200 import engine, layout, synth

# Tolerances for the atan2f-dependent (revolute) configuration: one step within
# abs/rel 1e-4, 60 steps within abs/rel 1e-3.
TOL_1STEP = 1e-4
TOL_60STEP = 1e-3


class Pair:
    """The same worlds on the GPU (torch uint8 tensor) and on a CPU oracle."""

    def __init__(self, cfg, oracle, host_worlds, seed, first=0):
        import torch
        self.cfg, self.o, self.seed, self.first = cfg, oracle, seed, first
        self.host = host_worlds.copy()
        self.dev = torch.from_numpy(host_worlds.copy()).cuda()
        kind, idx, nv = cfg.action
        self.vals = torch.zeros((len(host_worlds), max(nv, 1)), dtype=torch.float32, device="cuda")

    def step(self, step, active=None):
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
        rc = engine.batch_step_gpu(self.dev, cfg.dt, cfg.substeps, active=act_dev, caps=cfg.caps,
                                   joint_iters=cfg.joint_iters, relax_iters=cfg.relax_iters, flags=cfg.flags)
        assert rc == 0
        torch.cuda.synchronize()

    def got(self):
        return self.dev.cpu().numpy()


def contact_keys(raw, caps):
    """Per world: tuple of (shape_a, shape_b, point_count, features) of live contacts."""
    v = layout.view(raw, caps)
    keys = []
    for w in v:
        n = int(w["contact_count"])
        c = w["contacts"][:n]
        keys.append(tuple((int(a), int(b), int(k), tuple(int(f) for f in feats[:k]))
                          for a, b, k, feats in zip(c["shape_a"], c["shape_b"], c["point_count"],
                                                    c["points"]["feature"])))
    return keys


def state_close(got, want, caps, tol):
    """Body pose / velocity agreement within abs+rel `tol`; returns (ok, max abs err)."""
    g, w = layout.view(got, caps), layout.view(want, caps)
    err = 0.0
    ok = True
    for f in ("position", "rotation", "lin_vel", "ang_vel"):
        a, b = g["bodies"][f].astype(np.float64), w["bodies"][f].astype(np.float64)
        d = np.abs(a - b)
        err = max(err, float(d.max()))
        ok &= bool((d <= tol + tol * np.abs(b)).all())
    return ok, err
