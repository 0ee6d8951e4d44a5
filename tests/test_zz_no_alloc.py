"""The allocation-free step entry point (b3x_batch_step_gpu_noalloc).

It exists for callers that cannot allocate device memory when they step
(framework-owned or plugin-host-owned device memory, real-time loops that
cannot risk an allocation's synchronisation): its workspace is a fixed array
inside the library.  This file is collected last on purpose, so that a run
stopping at the first failure has run every other test before it; it must
also pass alone in a fresh process.  The check: two calls in a row through
the C-ABI give the same worlds as the regular entry point (whose results the
parity tests tie to the reference), within the parity tolerance — bit-exact
for this contact-only scene.
"""
import ctypes

import numpy as np
import pytest
import torch

from puffysics_b200 import build, engine, layout, synth
from puffysics_b200.configs import CONFIGS

pytestmark = pytest.mark.gpu


def test_noalloc_step_matches_regular_step():
    build.build()
    L = engine.lib()
    cfg = CONFIGS["stack"]
    host = synth.SceneLib(cfg).build(2048, 77)
    regular = torch.from_numpy(host.copy()).cuda()
    fixed = torch.from_numpy(host.copy()).cuda()
    stream = torch.cuda.current_stream()
    sig = layout.signature(*cfg.caps)
    for call in range(2):
        assert engine.batch_step_gpu(regular, cfg.dt, cfg.substeps, caps=cfg.caps, joint_iters=8) == 0
        b = engine.make_batch(fixed)
        rc = L.b3x_batch_step_gpu_noalloc(b, cfg.dt, cfg.substeps, None, ctypes.c_void_p(stream.cuda_stream),
                                          sig, 8, 8)
        assert rc == 0, rc
        torch.cuda.synchronize()
        assert np.array_equal(fixed.cpu().numpy(), regular.cpu().numpy()), "call %d differs" % call
    # same validation as the regular entry point: nothing written on bad input
    before = fixed.cpu().numpy()
    b = engine.make_batch(fixed)
    assert L.b3x_batch_step_gpu_noalloc(b, float("nan"), 4, None, ctypes.c_void_p(stream.cuda_stream),
                                        sig, 8, 8) == engine.CUDA_ERROR_INVALID_VALUE
    torch.cuda.synchronize()
    assert np.array_equal(fixed.cpu().numpy(), before)
