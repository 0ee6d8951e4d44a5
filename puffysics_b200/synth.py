"""Seeded synthetic inputs of the benchmark configurations.

Host: worlds are built by the C scene generators (scenes/b3_scenes.h,
compiled per capacity configuration into _lib/libb3scenes_<cfg>.so) through
the public world-building API.  Device: per-step actions and reset masks come
from b3x_scene_actions_gpu / b3x_scene_reset_gpu, bit-identical to the host
generators.  No public dataset is involved: the configurations are
parameterised scenes.
"""
import ctypes
import os

import numpy as np

from . import build as _build
from . import engine

_vp = ctypes.c_void_p


class SceneLib:
    def __init__(self, cfg):
        path = _build.scenes_lib(cfg.name)
        if not os.path.exists(path):
            _build.build()
        self.cfg = cfg
        self.lib = L = ctypes.CDLL(path)
        L.b3s_world_bytes.restype = ctypes.c_size_t
        L.b3s_signature.restype = ctypes.c_ulonglong
        L.b3s_build_batch.argtypes = [_vp, ctypes.c_size_t, ctypes.c_int, ctypes.c_int, ctypes.c_ulonglong,
                                      ctypes.c_ulonglong]
        L.b3s_build_batch.restype = ctypes.c_int
        L.b3s_actions_batch.argtypes = [_vp, ctypes.c_int, ctypes.c_int, ctypes.c_ulonglong, ctypes.c_ulonglong,
                                        ctypes.c_ulonglong]
        L.b3s_actions_batch.restype = ctypes.c_int
        L.b3s_reset_batch.argtypes = [_vp, ctypes.c_int, ctypes.c_ulonglong, ctypes.c_ulonglong, ctypes.c_ulonglong]
        self.world_bytes = int(L.b3s_world_bytes())
        assert int(L.b3s_signature()) == cfg.signature, "scene library capacity mismatch"

    def build(self, n, seed, first=0, stride=None):
        """(n, stride) uint8 host array of freshly built worlds."""
        stride = self.world_bytes if stride is None else stride
        out = np.zeros((n, stride), dtype=np.uint8)
        rc = self.lib.b3s_build_batch(out.ctypes.data, stride, n, self.cfg.scene, seed, first)
        if rc != 0:
            raise RuntimeError("scene build failed at world %d" % (-1 - rc))
        return out

    def actions(self, n, seed, first, step):
        kind, index, nv = self.cfg.action
        out = np.zeros((n, max(nv, 1)), dtype=np.float32)
        if nv:
            self.lib.b3s_actions_batch(out.ctypes.data, n, self.cfg.scene, seed, first, step)
        return out[:, :nv]

    def reset_mask(self, n, seed, first, step):
        out = np.zeros(n, dtype=np.uint8)
        self.lib.b3s_reset_batch(out.ctypes.data, n, seed, first, step)
        return out


def actions_gpu(out, n, scene, seed, first, step, stream=None):
    """Fill a float32 CUDA tensor (n, values per world) with the step's actions."""
    L = engine.lib()
    L.b3x_scene_actions_gpu.argtypes = [_vp, ctypes.c_int, ctypes.c_int, ctypes.c_ulonglong, ctypes.c_ulonglong,
                                        ctypes.c_ulonglong, _vp]
    L.b3x_scene_actions_gpu.restype = ctypes.c_int
    return L.b3x_scene_actions_gpu(ctypes.c_void_p(out.data_ptr()), n, scene, seed, first, step,
                                   engine._stream(stream))


def reset_gpu(out, n, seed, first, step, stream=None):
    """Fill a uint8 CUDA tensor (n,) with the scale-out reset mask of the step."""
    L = engine.lib()
    L.b3x_scene_reset_gpu.argtypes = [_vp, ctypes.c_int, ctypes.c_ulonglong, ctypes.c_ulonglong,
                                      ctypes.c_ulonglong, _vp]
    L.b3x_scene_reset_gpu.restype = ctypes.c_int
    return L.b3x_scene_reset_gpu(ctypes.c_void_p(out.data_ptr()), n, seed, first, step, engine._stream(stream))
