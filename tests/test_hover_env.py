"""The hover environment fused into one launch per step (libb3hover.so)
against the reference's own hover task (examples/pufferlib/puffysics_hover/
hover_task.h compiled on the CPU, oracle/_ref/libb3ref_hoverenv.so).

Bar: bit-exact.  Observations, rewards and terminals equal the reference's
after every step, and the whole HoverTask (world, rng, tick, episode return)
and the episode log are byte-identical after a run that crosses the 256-step
horizon (every environment resets at least once).
"""
import ctypes

import numpy as np
import pytest

import oracle as orc
from puffysics_b200 import build, hover_env


def _ref_or_skip():
    try:
        return orc.HoverOracle()
    except FileNotFoundError:
        pytest.skip("reference hover task not built (oracle/_ref)")


@pytest.fixture(scope="module")
def built():
    build.build()
    return hover_env.lib()


def test_exports_and_task_layout(built):
    L = built
    for f in ("b3x_hover_init_gpu", "b3x_hover_reset_gpu", "b3x_hover_step_gpu", "b3x_hover_step_in_place_gpu",
              "b3x_hover_env_bytes", "b3x_hover_task_bytes", "b3x_hover_task_offset", "b3x_hover_log_offset",
              "b3x_hover_signature"):
        assert hasattr(L, f)
    assert L.b3x_hover_signature() == 2 | (2 << 16) | (4 << 32) | (2 << 48)
    assert hover_env.env_bytes() % 8 == 0
    ref = _ref_or_skip()
    assert L.b3x_hover_task_bytes() == ref.task_bytes


def test_argument_checks_need_no_device(built):
    L = built
    n1 = ctypes.c_void_p(8)
    assert L.b3x_hover_init_gpu(None, 4, 2.0, 10.0, 1 / 60, 4, 256, 1, None) == 1
    assert L.b3x_hover_init_gpu(n1, -1, 2.0, 10.0, 1 / 60, 4, 256, 1, None) == 1
    assert L.b3x_hover_init_gpu(n1, 4, 2.0, 10.0, 0.0, 4, 256, 1, None) == 1
    assert L.b3x_hover_init_gpu(n1, 4, 2.0, 10.0, 1 / 60, 0, 256, 1, None) == 1
    assert L.b3x_hover_init_gpu(ctypes.c_void_p(12), 4, 2.0, 10.0, 1 / 60, 4, 256, 1, None) == 1
    assert L.b3x_hover_step_gpu(n1, 4, None, n1, n1, n1, None) == 1
    assert L.b3x_hover_step_in_place_gpu(n1, 4, n1, n1, n1, None, None) == 1
    assert L.b3x_hover_reset_gpu(n1, -2, n1, n1, n1, None) == 1
    assert L.b3x_hover_step_gpu(None, 0, None, None, None, None, None) == 0


def test_reference_hover_task_runs_episodes():
    """The oracle itself: every environment ends an episode within the
    horizon and the per-environment log counts it."""
    ref = _ref_or_skip()
    tasks, logs = ref.init(16, 3)
    done_any = np.zeros(16, bool)
    rng = np.random.default_rng(0)
    for _ in range(260):
        _, rew, term = ref.step(tasks, logs, rng.integers(0, 3, 16).astype(np.float32))
        assert np.isfinite(rew).all()
        done_any |= term == 1.0
    assert done_any.all()
    assert (logs[:, 4] >= 1).all()


def _actions(step, n):
    return np.random.default_rng(1000 + step).integers(0, 3, n).astype(np.float32)


@pytest.mark.gpu
@pytest.mark.parametrize("in_place", [False, True])
def test_fused_env_step_matches_reference(in_place, built):
    import torch
    ref = _ref_or_skip()
    n, seed = 101, 17
    envs = torch.zeros((n, hover_env.env_bytes()), dtype=torch.uint8, device="cuda")
    assert hover_env.init(envs, seed) == 0
    tasks, logs = ref.init(n, seed)
    torch.cuda.synchronize()
    assert np.array_equal(hover_env.tasks(envs.cpu().numpy()), tasks)
    obs = torch.zeros((n, 3), dtype=torch.float32, device="cuda")
    rew = torch.zeros(n, dtype=torch.float32, device="cuda")
    term = torch.zeros(n, dtype=torch.float32, device="cuda")
    act = torch.zeros(n, dtype=torch.float32, device="cuda")
    resets = 0
    for s in range(300):
        a = _actions(s, n)
        act.copy_(torch.from_numpy(a))
        assert hover_env.step(envs, act, obs, rew, term, in_place=in_place) == 0
        o_ref, r_ref, t_ref = ref.step(tasks, logs, a)
        torch.cuda.synchronize()
        assert np.array_equal(obs.cpu().numpy(), o_ref), s
        assert np.array_equal(rew.cpu().numpy(), r_ref), s
        assert np.array_equal(term.cpu().numpy(), t_ref), s
        resets += int(t_ref.sum())
    host = envs.cpu().numpy()
    assert np.array_equal(hover_env.tasks(host), tasks)
    assert np.array_equal(hover_env.logs(host), logs)
    assert resets >= n


@pytest.mark.gpu
def test_reset_writes_first_observation(built):
    import torch
    ref = _ref_or_skip()
    n = 40
    envs = torch.zeros((n, hover_env.env_bytes()), dtype=torch.uint8, device="cuda")
    assert hover_env.init(envs, 5) == 0
    obs = torch.full((n, 3), 7.0, device="cuda")
    rew = torch.full((n,), 7.0, device="cuda")
    term = torch.full((n,), 7.0, device="cuda")
    assert hover_env.reset(envs, obs, rew, term) == 0
    torch.cuda.synchronize()
    tasks, _ = ref.init(n, 5)
    o = obs.cpu().numpy()
    assert (rew.cpu().numpy() == 0).all() and (term.cpu().numpy() == 0).all()
    assert (o[:, 2] == 0).all() and (o[:, 1] == 0).all()
    # a reset draws the next jitter from the environment's rng: heights differ from init's
    assert not np.array_equal(hover_env.tasks(envs.cpu().numpy()), tasks)
    assert (np.abs(o[:, 0]) <= 0.5).all()
