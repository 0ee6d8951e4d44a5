"""Host-side mirror of the C-ABI (include/puffysics_b200.h) over ctypes.

Names, argument meaning and return codes follow the reference batch API
(reference b3_batch.cuh:12-99): functions return cudaError_t codes
(0 = success, 1 = cudaErrorInvalidValue) and never raise for invalid
arguments; nothing is launched or written when they return 1.

Worlds are torch uint8 tensors on a CUDA device of shape (count, stride);
torch is used only for device memory and streams.  There is no CPU path:
loading fails loudly if libpuffysics_b200.so is missing.
"""
import ctypes
import os

from . import layout

_PKG = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_PKG, "_lib", "libpuffysics_b200.so")

CUDA_SUCCESS = 0
CUDA_ERROR_INVALID_VALUE = 1

ACTION_FORCE, ACTION_TORQUE, ACTION_LINEAR_IMPULSE, ACTION_JOINT_TARGET = 0, 1, 2, 3


class B3Batch(ctypes.Structure):
    _fields_ = [("data", ctypes.c_void_p), ("stride", ctypes.c_size_t), ("world_offset", ctypes.c_size_t),
                ("count", ctypes.c_int)]


_lib = None


def lib():
    """The loaded C-ABI library (raises if it has not been built)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError("libpuffysics_b200.so is not built (%s); run python -m puffysics_b200.build"
                               % LIB_PATH)
        L = ctypes.CDLL(LIB_PATH)
        vp, u8p = ctypes.c_void_p, ctypes.c_void_p
        L.b3x_batch_step_gpu.argtypes = [B3Batch, ctypes.c_float, ctypes.c_int, u8p, vp, ctypes.c_ulonglong,
                                         ctypes.c_int, ctypes.c_int]
        L.b3x_batch_step_gpu.restype = ctypes.c_int
        L.b3x_batch_step_gpu_flags.argtypes = [B3Batch, ctypes.c_float, ctypes.c_int, u8p, vp, ctypes.c_ulonglong,
                                               ctypes.c_int, ctypes.c_int, ctypes.c_int]
        L.b3x_batch_step_gpu_flags.restype = ctypes.c_int
        L.b3x_batch_step_gpu_ws.argtypes = [B3Batch, ctypes.c_float, ctypes.c_int, u8p, vp, ctypes.c_ulonglong,
                                            ctypes.c_int, ctypes.c_int, vp, ctypes.c_size_t]
        L.b3x_batch_step_gpu_ws.restype = ctypes.c_int
        L.b3x_batch_step_gpu_noalloc.argtypes = [B3Batch, ctypes.c_float, ctypes.c_int, u8p, vp,
                                                 ctypes.c_ulonglong, ctypes.c_int, ctypes.c_int]
        L.b3x_batch_step_gpu_noalloc.restype = ctypes.c_int
        L.b3x_workspace_bytes.argtypes = [ctypes.c_ulonglong, ctypes.c_int]
        L.b3x_workspace_bytes.restype = ctypes.c_size_t
        L.b3x_workspace_slot_bytes.argtypes = [ctypes.c_ulonglong]
        L.b3x_workspace_slot_bytes.restype = ctypes.c_size_t
        L.b3x_reserve_workspace.argtypes = [vp, ctypes.c_ulonglong]
        L.b3x_reserve_workspace.restype = ctypes.c_int
        L.b3x_release_workspaces.argtypes = []
        L.b3x_release_workspaces.restype = ctypes.c_int
        L.b3x_reserved_bytes.argtypes = [vp]
        L.b3x_reserved_bytes.restype = ctypes.c_size_t
        L.b3x_fault_flags.argtypes = [ctypes.c_int]
        L.b3x_fault_flags.restype = ctypes.c_int
        L.b3x_step_launches.argtypes = [ctypes.c_ulonglong, ctypes.c_int, ctypes.c_int]
        L.b3x_step_launches.restype = ctypes.c_int
        L.b3x_batch_restore_gpu.argtypes = [B3Batch, vp, u8p, vp, ctypes.c_ulonglong]
        L.b3x_batch_restore_gpu.restype = ctypes.c_int
        L.b3x_batch_apply_gpu.argtypes = [B3Batch, ctypes.c_int, ctypes.c_int, vp, ctypes.c_int, u8p, vp,
                                          ctypes.c_ulonglong]
        L.b3x_batch_apply_gpu.restype = ctypes.c_int
        L.b3x_batch_observe_gpu.argtypes = [B3Batch, ctypes.c_int, vp, vp, ctypes.c_ulonglong]
        L.b3x_batch_observe_gpu.restype = ctypes.c_int
        L.b3x_engine_bytes.argtypes = [ctypes.c_ulonglong, ctypes.c_int]
        L.b3x_engine_bytes.restype = ctypes.c_size_t
        for name in ("b3x_engine_bind", "b3x_engine_sync_to_aos"):
            f = getattr(L, name)
            f.argtypes = [vp, ctypes.c_int, B3Batch, u8p, vp, ctypes.c_ulonglong]
            f.restype = ctypes.c_int
        L.b3x_engine_step.argtypes = [vp, ctypes.c_int, ctypes.c_float, ctypes.c_int, u8p, vp, ctypes.c_ulonglong,
                                      ctypes.c_int, ctypes.c_int, ctypes.c_int]
        L.b3x_engine_step.restype = ctypes.c_int
        L.b3x_engine_apply.argtypes = [vp, ctypes.c_int, ctypes.c_int, ctypes.c_int, vp, ctypes.c_int, u8p, vp,
                                       ctypes.c_ulonglong]
        L.b3x_engine_apply.restype = ctypes.c_int
        L.b3x_engine_observe.argtypes = [vp, ctypes.c_int, ctypes.c_int, vp, vp, ctypes.c_ulonglong]
        L.b3x_engine_observe.restype = ctypes.c_int
        L.b3x_world_bytes.argtypes = [ctypes.c_ulonglong]
        L.b3x_world_bytes.restype = ctypes.c_size_t
        L.b3x_version.restype = ctypes.c_char_p
        _lib = L
    return _lib


def _ptr(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def _stream(stream):
    if stream is None:
        import torch
        stream = torch.cuda.current_stream()
    return ctypes.c_void_p(stream.cuda_stream if hasattr(stream, "cuda_stream") else int(stream))


def make_batch(worlds, stride=None, offset=0, count=None):
    """B3Batch over a (count, stride) uint8 tensor (or raw pointer ints)."""
    if isinstance(worlds, int) or worlds is None:
        return B3Batch(worlds, stride or 0, offset, count or 0)
    return B3Batch(worlds.data_ptr() if worlds.numel() else None,
                   worlds.shape[1] if stride is None else stride, offset,
                   worlds.shape[0] if count is None else count)


def batch_step_gpu(worlds, dt, substeps, active=None, stream=None, caps=None, joint_iters=2, relax_iters=None,
                   stride=None, offset=0, count=None, workspace=None, flags=0):
    """Step the selected worlds once (b3_batch_step_gpu; `flags` selects the
    reference's alternative step modes, b3x_batch_step_gpu_flags).  Returns a
    cudaError_t code."""
    sig = layout.signature(*caps)
    relax_iters = joint_iters if relax_iters is None else relax_iters
    b = make_batch(worlds, stride, offset, count)
    if flags:
        assert workspace is None, "the mode entry point uses the library's workspace"
        return lib().b3x_batch_step_gpu_flags(b, dt, substeps, _ptr(active), _stream(stream), sig, joint_iters,
                                              relax_iters, flags)
    if workspace is not None:
        return lib().b3x_batch_step_gpu_ws(b, dt, substeps, _ptr(active), _stream(stream), sig, joint_iters,
                                           relax_iters, _ptr(workspace), workspace.numel() * workspace.element_size())
    return lib().b3x_batch_step_gpu(b, dt, substeps, _ptr(active), _stream(stream), sig, joint_iters, relax_iters)


def batch_restore_gpu(worlds, initial, reset=None, stream=None, caps=None, stride=None, offset=0, count=None):
    """Copy snapshots over the selected worlds (b3_batch_restore_gpu)."""
    b = make_batch(worlds, stride, offset, count)
    return lib().b3x_batch_restore_gpu(b, _ptr(initial), _ptr(reset), _stream(stream), layout.signature(*caps))


def batch_apply_gpu(worlds, kind, index, values, active=None, stream=None, caps=None, stride=None, offset=0):
    """Apply per-world forces / torques / impulses / joint targets (values: float32 (count, k))."""
    b = make_batch(worlds, stride, offset)
    return lib().b3x_batch_apply_gpu(b, kind, index, _ptr(values), values.shape[1], _ptr(active), _stream(stream),
                                     layout.signature(*caps))


def batch_observe_gpu(worlds, body, out, stream=None, caps=None, stride=None, offset=0):
    """Gather position/rotation/lin_vel/ang_vel (13 floats) of one body per world."""
    b = make_batch(worlds, stride, offset)
    return lib().b3x_batch_observe_gpu(b, body, _ptr(out), _stream(stream), layout.signature(*caps))


def workspace_bytes(caps, device=0):
    """Workspace of one launch per resident wave (what reserve_workspace takes)."""
    return lib().b3x_workspace_bytes(layout.signature(*caps), device)


def workspace_slot_bytes(caps):
    """One tile's (32 worlds') workspace slot."""
    return lib().b3x_workspace_slot_bytes(layout.signature(*caps))


def reserve_workspace(caps, stream=None):
    """Set-up: reserve the step's workspace for `stream` (the only device
    allocation the library makes); later steps on that stream use it."""
    return lib().b3x_reserve_workspace(_stream(stream), layout.signature(*caps))


def release_workspaces():
    """Free every workspace reserved on the current device."""
    return lib().b3x_release_workspaces()


def reserved_bytes(stream=None):
    return lib().b3x_reserved_bytes(_stream(stream))


def fault_flags(clear=False):
    """Nonzero if a step abandoned a tile because a bounded wait gave up."""
    return lib().b3x_fault_flags(1 if clear else 0)


def step_launches(caps, count, device=0):
    """Kernel launches of one batch_step_gpu call over `count` worlds."""
    return lib().b3x_step_launches(layout.signature(*caps), count, device)


def world_bytes(caps):
    return lib().b3x_world_bytes(layout.signature(*caps))


# ---- resident world columns (b3x_engine_*) --------------------------------------------
class Columns:
    """Worlds resident in HBM as structure-of-arrays across worlds (the
    b3x_engine_* entry points): a uint8 device tensor of b3x_engine_bytes and
    the world count.  bind / sync_to_aos move worlds from / to an AoS batch;
    step / apply / observe work on the columns directly."""

    def __init__(self, caps, count, device=None):
        import torch
        self.caps, self.count = tuple(caps), count
        self.sig = layout.signature(*caps)
        nbytes = lib().b3x_engine_bytes(self.sig, count)
        self.store = torch.empty(max(nbytes, 16), dtype=torch.uint8, device=device or "cuda")

    def _p(self):
        return ctypes.c_void_p(self.store.data_ptr())

    def bind(self, worlds, select=None, stream=None, stride=None, offset=0):
        return lib().b3x_engine_bind(self._p(), self.count, make_batch(worlds, stride, offset), _ptr(select),
                                     _stream(stream), self.sig)

    def sync_to_aos(self, worlds, select=None, stream=None, stride=None, offset=0):
        return lib().b3x_engine_sync_to_aos(self._p(), self.count, make_batch(worlds, stride, offset), _ptr(select),
                                            _stream(stream), self.sig)

    def step(self, dt, substeps, active=None, stream=None, joint_iters=2, relax_iters=None, flags=0):
        relax_iters = joint_iters if relax_iters is None else relax_iters
        return lib().b3x_engine_step(self._p(), self.count, dt, substeps, _ptr(active), _stream(stream), self.sig,
                                     joint_iters, relax_iters, flags)

    def apply(self, kind, index, values, active=None, stream=None):
        return lib().b3x_engine_apply(self._p(), self.count, kind, index, _ptr(values), values.shape[1],
                                      _ptr(active), _stream(stream), self.sig)

    def observe(self, body, out, stream=None):
        return lib().b3x_engine_observe(self._p(), self.count, body, _ptr(out), _stream(stream), self.sig)


# ---- per-thread device b3_step (include/puffysics.cuh) ------------------------------
_thread_libs = {}


def thread_lib(name):
    """libb3thread_<name>.so: launchers of the header's per-thread device
    b3_step compiled with the capacities of configuration `name` (raises if it
    has not been built)."""
    if name not in _thread_libs:
        path = os.path.join(_PKG, "_lib", "libb3thread_%s.so" % name)
        if not os.path.exists(path):
            raise RuntimeError("%s is not built; run python -m puffysics_b200.build" % path)
        L = ctypes.CDLL(path)
        L.b3x_thread_signature.restype = ctypes.c_ulonglong
        L.b3x_thread_joint_iters.restype = ctypes.c_int
        L.b3x_thread_relax_iters.restype = ctypes.c_int
        L.b3x_thread_step_gpu.argtypes = [B3Batch, ctypes.c_float, ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p]
        L.b3x_thread_step_gpu.restype = ctypes.c_int
        L.b3x_thread_step_worlds_gpu.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_float, ctypes.c_int,
                                                 ctypes.c_void_p]
        L.b3x_thread_step_worlds_gpu.restype = ctypes.c_int
        L.b3x_thread_scene_apply_gpu.argtypes = [B3Batch, ctypes.c_int, ctypes.c_ulonglong, ctypes.c_ulonglong,
                                                 ctypes.c_ulonglong, ctypes.c_void_p]
        L.b3x_thread_scene_apply_gpu.restype = ctypes.c_int
        if hasattr(L, "b3x_thread_shim_step_gpu"):
            L.b3x_thread_shim_step_gpu.argtypes = [B3Batch, ctypes.c_float, ctypes.c_int, ctypes.c_void_p,
                                                   ctypes.c_void_p]
            L.b3x_thread_shim_step_gpu.restype = ctypes.c_int
        _thread_libs[name] = L
    return _thread_libs[name]


def thread_step_gpu(name, worlds, dt, substeps, active=None, stream=None, stride=None, offset=0, count=None):
    """Step the selected worlds with one thread per world (device b3_step over
    a batch, b3_batch_step_gpu semantics).  Returns a cudaError_t code."""
    b = make_batch(worlds, stride, offset, count)
    return thread_lib(name).b3x_thread_step_gpu(b, dt, substeps, _ptr(active), _stream(stream))


def thread_scene_apply_gpu(name, worlds, scene, seed, first, step, stream=None):
    """The benchmark scene's actions of `step` applied to every world, one
    launch with the header's b3_apply_* (benchmark input of the per-thread
    path).  Returns a cudaError_t code."""
    b = make_batch(worlds, None, 0, None)
    return thread_lib(name).b3x_thread_scene_apply_gpu(b, scene, seed, first, step, _stream(stream))


def thread_step_worlds_gpu(name, worlds, dt, substeps, stream=None):
    """b3_step_kernel over contiguous worlds (a (count, sizeof(B3World)) tensor)."""
    return thread_lib(name).b3x_thread_step_worlds_gpu(_ptr(worlds) if worlds.numel() else None, worlds.shape[0],
                                                       dt, substeps, _stream(stream))
