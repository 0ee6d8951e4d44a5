"""The allocation-free step entry point (b3x_batch_step_gpu_noalloc).

It exists for callers that cannot allocate device memory when they step
(framework-owned or plugin-host-owned device memory, real-time loops that
cannot risk an allocation's synchronisation): its workspace is a fixed 64 MiB
array inside the library.  This file is collected last on purpose, so that a
run stopping at the first failure has run every other test before it; it must
also pass alone in a fresh process.  The checks: two calls in a row through
the C-ABI give the same worlds as the regular entry point (whose results the
parity tests tie to the reference), within the parity tolerance — bit-exact
for this contact-only scene; a batch with more tiles than the array has
slots (several launches reusing the array) matches the regular entry point
and the reference's CPU step; a capacity configuration whose tile slot does
not fit the array is rejected with nothing written.
"""
import ctypes

import numpy as np
import pytest
import torch

import oracle as orc
from puffysics_b200 import build, engine, layout, synth
from puffysics_b200.configs import CONFIGS

pytestmark = pytest.mark.gpu
NOALLOC_BYTES = 64 << 20


def noalloc_step(L, worlds, cfg, stream, dt=None):
    b = engine.make_batch(worlds)
    return L.b3x_batch_step_gpu_noalloc(b, cfg.dt if dt is None else dt, cfg.substeps, None,
                                        ctypes.c_void_p(stream.cuda_stream), layout.signature(*cfg.caps), 8, 8)


def test_noalloc_step_matches_regular_step():
    build.build()
    L = engine.lib()
    cfg = CONFIGS["stack"]
    host = synth.SceneLib(cfg).build(2048, 77)
    regular = torch.from_numpy(host.copy()).cuda()
    fixed = torch.from_numpy(host.copy()).cuda()
    stream = torch.cuda.current_stream()
    for call in range(2):
        assert engine.batch_step_gpu(regular, cfg.dt, cfg.substeps, caps=cfg.caps, joint_iters=8) == 0
        rc = noalloc_step(L, fixed, cfg, stream)
        assert rc == 0, rc
        torch.cuda.synchronize()
        assert np.array_equal(fixed.cpu().numpy(), regular.cpu().numpy()), "call %d differs" % call
    # same validation as the regular entry point: nothing written on bad input
    before = fixed.cpu().numpy()
    assert noalloc_step(L, fixed, cfg, stream, dt=float("nan")) == engine.CUDA_ERROR_INVALID_VALUE
    torch.cuda.synchronize()
    assert np.array_equal(fixed.cpu().numpy(), before)


def test_noalloc_batch_larger_than_the_array():
    """8,192 stack worlds are 256 tiles; the 64 MiB array holds fewer slots,
    so one call runs several launches over the same array."""
    build.build()
    L = engine.lib()
    cfg = CONFIGS["stack"]
    n = 8192
    assert (n + 31) // 32 > NOALLOC_BYTES // engine.workspace_slot_bytes(cfg.caps)
    kind = "ref" if orc.available("stack", "ref") else "port"
    o = orc.Oracle("stack", kind)
    host = synth.SceneLib(cfg).build(n, 5)
    regular = torch.from_numpy(host.copy()).cuda()
    fixed = torch.from_numpy(host.copy()).cuda()
    stream = torch.cuda.current_stream()
    ref = host.copy()
    for call in range(2):
        assert engine.batch_step_gpu(regular, cfg.dt, cfg.substeps, caps=cfg.caps, joint_iters=8) == 0
        assert noalloc_step(L, fixed, cfg, stream) == 0
        o.batch_step(ref, cfg.dt, cfg.substeps)
        torch.cuda.synchronize()
        got = fixed.cpu().numpy()
        assert np.array_equal(got, regular.cpu().numpy()), "call %d differs from the regular entry" % call
        assert np.array_equal(got, ref), "call %d differs from the reference" % call
    assert engine.fault_flags() == 0


def test_noalloc_rejects_a_slot_larger_than_the_array():
    """Capacities of 5,000 contacts make one tile's slot larger than 64 MiB:
    cudaErrorInvalidValue, nothing launched, the worlds untouched."""
    build.build()
    L = engine.lib()
    caps = (2, 2, 5000, 1)
    assert engine.workspace_slot_bytes(caps) > NOALLOC_BYTES
    wb = layout.world_bytes(*caps)
    host = np.random.default_rng(0).integers(0, 256, size=(2, wb), dtype=np.uint8)
    worlds = torch.from_numpy(host.copy()).cuda()
    stream = torch.cuda.current_stream()
    b = engine.make_batch(worlds)
    rc = L.b3x_batch_step_gpu_noalloc(b, 1.0 / 60.0, 4, None, ctypes.c_void_p(stream.cuda_stream),
                                      layout.signature(*caps), 8, 8)
    assert rc == engine.CUDA_ERROR_INVALID_VALUE
    torch.cuda.synchronize()
    assert np.array_equal(worlds.cpu().numpy(), host)
