"""The PufferLib hover environment fused into one launch per step
(libb3hover.so, puffysics_b200/csrc/b3x_hover_env.cu), over ctypes.

Environments live in a torch uint8 device tensor of shape (n, env_bytes());
actions are float32 (n,), observations float32 (n, 3), rewards and terminals
float32 (n,).  Functions return cudaError_t codes (0 success, 1 invalid
arguments, nothing launched).  There is no CPU path: loading fails loudly when
the library is missing.
"""
import ctypes
import os

_PKG = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_PKG, "_lib", "libb3hover.so")
OBS = 3
# hover_default_config (reference examples/pufferlib/puffysics_hover/hover_task.h:41-44)
DEFAULT = dict(target_height=2.0, thrust=10.0, dt=1.0 / 60.0, substeps=4, horizon=256)

_lib = None


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError("%s is not built; run python -m puffysics_b200.build" % LIB_PATH)
        L = ctypes.CDLL(LIB_PATH)
        sz, vp, fp = ctypes.c_size_t, ctypes.c_void_p, ctypes.c_float
        for f in ("b3x_hover_env_bytes", "b3x_hover_task_offset", "b3x_hover_task_bytes", "b3x_hover_log_offset"):
            getattr(L, f).restype = sz
        L.b3x_hover_signature.restype = ctypes.c_ulonglong
        L.b3x_hover_init_gpu.argtypes = [vp, ctypes.c_int, fp, fp, fp, ctypes.c_int, ctypes.c_int, ctypes.c_uint, vp]
        L.b3x_hover_reset_gpu.argtypes = [vp, ctypes.c_int, vp, vp, vp, vp]
        L.b3x_hover_step_gpu.argtypes = [vp, ctypes.c_int, vp, vp, vp, vp, vp]
        L.b3x_hover_step_in_place_gpu.argtypes = [vp, ctypes.c_int, vp, vp, vp, vp, vp]
        for f in ("b3x_hover_init_gpu", "b3x_hover_reset_gpu", "b3x_hover_step_gpu", "b3x_hover_step_in_place_gpu"):
            getattr(L, f).restype = ctypes.c_int
        _lib = L
    return _lib


def env_bytes():
    return lib().b3x_hover_env_bytes()


def _p(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _s(stream):
    if stream is None:
        import torch
        stream = torch.cuda.current_stream()
    return ctypes.c_void_p(stream.cuda_stream)


def init(envs, seed, stream=None, **config):
    c = dict(DEFAULT, **config)
    return lib().b3x_hover_init_gpu(_p(envs), envs.shape[0], c["target_height"], c["thrust"], c["dt"],
                                    c["substeps"], c["horizon"], seed, _s(stream))


def reset(envs, obs, rewards, terminals, stream=None):
    return lib().b3x_hover_reset_gpu(_p(envs), envs.shape[0], _p(obs), _p(rewards), _p(terminals), _s(stream))


def step(envs, actions, obs, rewards, terminals, stream=None, in_place=False):
    f = lib().b3x_hover_step_in_place_gpu if in_place else lib().b3x_hover_step_gpu
    return f(_p(envs), envs.shape[0], _p(actions), _p(obs), _p(rewards), _p(terminals), _s(stream))


def tasks(envs_host):
    """The HoverTask bytes of each environment (numpy (n, task_bytes))."""
    o, b = lib().b3x_hover_task_offset(), lib().b3x_hover_task_bytes()
    return envs_host[:, o:o + b]


def logs(envs_host):
    """Episode statistics (perf, score, episode_return, episode_length, n), float32 (n, 5)."""
    o = lib().b3x_hover_log_offset()
    return envs_host[:, o:o + 20].copy().view("<f4")
