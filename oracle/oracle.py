"""ctypes loader for the CPU parity oracles.

TEST INFRASTRUCTURE, NOT PRODUCT CODE.  Only tests/, __graft_entry__.smoke()
and the CPU-baseline leg of bench.py use this module.

Two oracles share one interface (see oracle/shim.c):
  kind="ref"  -- the reference's own C implementation (b3_batch_step from
                 b3_batch.cuh / puffysics.cuh) compiled in this container into
                 oracle/_ref/libb3ref_<cfg>.so;
  kind="port" -- the restatement oracle/port/b3port.c, compiled into
                 oracle/_build/libb3port_<cfg>.so (buildable anywhere with gcc).
Worlds are numpy uint8 arrays of shape (count, stride) holding the AoS
B3World bytes of the configuration's capacities.
"""
import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))

_c_p = ctypes.c_void_p
_u8p = ctypes.POINTER(ctypes.c_ubyte)


def lib_path(cfg, kind):
    sub = "_ref" if kind == "ref" else "_build"
    return os.path.join(HERE, sub, "libb3%s_%s.so" % (kind, cfg))


def build_oracles(quiet=True, ref_dir=None):
    """Compile the port oracles, and the reference ones when a reference
    checkout is given (`ref_dir`, else the PUFFYSICS_REF environment
    variable).  Returns the make exit status."""
    ref_dir = ref_dir or os.environ.get("PUFFYSICS_REF")
    cmd = ["make", "-C", HERE, "-j8"] + (["REF_DIR=" + ref_dir] if ref_dir else [])
    out = subprocess.run(cmd, capture_output=quiet)
    return out.returncode


def available(cfg, kind):
    return os.path.exists(lib_path(cfg, kind))


def _ptr(a):
    return None if a is None else a.ctypes.data_as(_c_p)


class Oracle:
    def __init__(self, cfg, kind="ref"):
        path = lib_path(cfg, kind)
        if kind == "port" and not os.path.exists(path):
            build_oracles()
        if not os.path.exists(path):
            raise FileNotFoundError(path)
        self.cfg, self.kind = cfg, kind
        self.lib = lib = ctypes.CDLL(path)
        p = kind + "_"
        self._f = lambda name: getattr(lib, p + name)
        f = self._f
        f("world_bytes").restype = ctypes.c_size_t
        f("config_signature").restype = ctypes.c_ulonglong
        f("joint_iters").restype = ctypes.c_int
        f("relax_iters").restype = ctypes.c_int
        f("build").argtypes = [_c_p, ctypes.c_int, ctypes.c_int, ctypes.c_ulonglong, ctypes.c_ulonglong]
        f("build").restype = ctypes.c_int
        f("batch_step").argtypes = [_c_p, ctypes.c_size_t, ctypes.c_size_t, ctypes.c_int, ctypes.c_float,
                                    ctypes.c_int, _c_p]
        f("batch_step").restype = ctypes.c_int
        f("batch_restore").argtypes = [_c_p, ctypes.c_size_t, ctypes.c_size_t, ctypes.c_int, _c_p, _c_p]
        f("batch_restore").restype = ctypes.c_int
        f("step_world").argtypes = [_c_p, ctypes.c_float, ctypes.c_int]
        f("apply").argtypes = [_c_p, ctypes.c_size_t, ctypes.c_size_t, ctypes.c_int, ctypes.c_int,
                               ctypes.c_ulonglong, ctypes.c_ulonglong, ctypes.c_ulonglong, _c_p]
        f("apply_values").argtypes = [_c_p, ctypes.c_size_t, ctypes.c_size_t, ctypes.c_int, ctypes.c_int,
                                      ctypes.c_int, _c_p, ctypes.c_int, _c_p]
        f("collide").argtypes = [_c_p, ctypes.c_int, ctypes.c_int] + [_c_p] * 5
        f("collide").restype = ctypes.c_int
        f("run_mt").argtypes = [_c_p, ctypes.c_int, ctypes.c_int, ctypes.c_ulonglong, ctypes.c_ulonglong,
                                ctypes.c_ulonglong, ctypes.c_int, ctypes.c_float, ctypes.c_int, ctypes.c_int]
        f("run_mt").restype = ctypes.c_double
        self.world_bytes = int(f("world_bytes")())
        self.signature = int(f("config_signature")())
        self.joint_iters = int(f("joint_iters")())
        self.relax_iters = int(f("relax_iters")())

    # ---- scene construction
    def build(self, n, scene, seed, first=0):
        w = np.zeros((n, self.world_bytes), dtype=np.uint8)
        rc = self._f("build")(_ptr(w), n, scene, seed, first)
        if rc != 0:
            raise RuntimeError("scene build failed at world %d" % (-1 - rc))
        return w

    # ---- stepping
    def batch_step(self, data, dt, substeps, active=None, stride=None, offset=0, count=None):
        """b3_batch_step on a (count, stride) uint8 array; returns 1 / 0."""
        stride = data.shape[1] if stride is None else stride
        count = data.shape[0] if count is None else count
        return self._f("batch_step")(_ptr(data), stride, offset, count, dt, substeps, _ptr(active))

    def batch_restore(self, data, initial, reset=None, stride=None, offset=0, count=None):
        stride = data.shape[1] if stride is None else stride
        count = data.shape[0] if count is None else count
        return self._f("batch_restore")(_ptr(data), stride, offset, count, _ptr(initial), _ptr(reset))

    def apply(self, data, scene, seed, first, step, active=None, stride=None, offset=0):
        stride = data.shape[1] if stride is None else stride
        self._f("apply")(_ptr(data), stride, offset, data.shape[0], scene, seed, first, step, _ptr(active))

    def apply_values(self, data, kind, index, values, active=None, stride=None, offset=0):
        values = np.ascontiguousarray(values, dtype=np.float32)
        stride = data.shape[1] if stride is None else stride
        self._f("apply_values")(_ptr(data), stride, offset, data.shape[0], kind, index, _ptr(values),
                                values.shape[1], _ptr(active))

    def collide(self, world, sa, sb):
        normal = np.zeros(3, np.float32)
        pa = np.zeros(12, np.float32)
        pb = np.zeros(12, np.float32)
        sep = np.zeros(4, np.float32)
        feat = np.zeros(4, np.uint32)
        n = self._f("collide")(_ptr(world), sa, sb, _ptr(normal), _ptr(pa), _ptr(pb), _ptr(sep), _ptr(feat))
        return n, normal, pa[:3 * n].reshape(n, 3), pb[:3 * n].reshape(n, 3), sep[:n], feat[:n]

    def run_mt(self, worlds, scene, seed, first, step0, steps, dt, substeps, threads):
        return self._f("run_mt")(_ptr(worlds), worlds.shape[0], scene, seed, first, step0, steps, dt,
                                 substeps, threads)


class HoverOracle:
    """The reference's hover task on the CPU (oracle/_ref/libb3ref_hoverenv.so,
    hover_task.h compiled from the reference), over (n, task_bytes) uint8
    arrays; logs are float32 (n, 5)."""

    def __init__(self):
        path = os.path.join(HERE, "_ref", "libb3ref_hoverenv.so")
        if not os.path.exists(path):
            raise FileNotFoundError(path)
        L = ctypes.CDLL(path)
        L.refhover_task_bytes.restype = ctypes.c_size_t
        vp = ctypes.c_void_p
        L.refhover_init.argtypes = [vp, ctypes.c_int, ctypes.c_float, ctypes.c_float, ctypes.c_float, ctypes.c_int,
                                    ctypes.c_int, ctypes.c_uint]
        L.refhover_step.argtypes = [vp, vp, ctypes.c_int, vp, vp, vp, vp]
        self.L = L
        self.task_bytes = L.refhover_task_bytes()

    def init(self, n, seed, target_height=2.0, thrust=10.0, dt=1.0 / 60.0, substeps=4, horizon=256):
        t = np.zeros((n, self.task_bytes), dtype=np.uint8)
        self.L.refhover_init(_ptr(t), n, target_height, thrust, dt, substeps, horizon, seed)
        return t, np.zeros((n, 5), dtype=np.float32)

    def step(self, tasks, logs, actions):
        n = tasks.shape[0]
        obs = np.zeros((n, 3), dtype=np.float32)
        rew = np.zeros(n, dtype=np.float32)
        term = np.zeros(n, dtype=np.float32)
        a = np.ascontiguousarray(actions, dtype=np.float32)
        self.L.refhover_step(_ptr(tasks), _ptr(logs), n, _ptr(a), _ptr(obs), _ptr(rew), _ptr(term))
        return obs, rew, term
