"""Benchmark: physics-only env-steps/s of the batched rigid-body step on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config stack]
    python -m torch.distributed.run --nproc-per-node N ... bench.py --gpus N
    python bench.py --impl reference        # the reference's CPU b3_batch_step

A step = the scene's per-step actions applied to every world, then one
b3_batch_step_gpu of every world (worlds x steps / s, substeps not counted,
reference README.md:149-152).  One process per GPU; each rank owns a
contiguous shard of independent worlds (weak scaling: the configuration's
world count per GPU; `scaleout` keeps 1,048,576 worlds in total).  No
collective runs inside the timed region.  Rank 0 prints one JSON line.

value    device-resident: actions generated on the device, worlds resident in
         HBM -- by default as structure-of-arrays columns across worlds
         (b3x_engine_*, bound once from the seeded AoS worlds before the
         timing; --path aos: the drop-in b3x_batch_step_gpu on the caller's
         AoS worlds, which the line also reports as `aos_path`); per-step
         CUDA events on the launching stream, L2 flushed between timed steps
         (outside the events) unless the world array is larger than twice
         L2, max over ranks.
e2e      through the C-ABI with host buffers: each step copies that step's
         actions from pinned host memory, applies them, steps, gathers one
         observation per world and copies it back, then synchronises.
roofline the step kernel alone, its CUDA-event duration against the
         algorithmic bytes of a world-step (the byte model below), plus the
         fp32 work per world-step against one add or mul per lane per clock.
configs  (one GPU) the configurations quoted over a fixed window of steps
         from their seeded state -- C4 pile: steps 1-240 from the seeded
         drop -- each with its own value, roofline, e2e and CPU baseline;
         warm-up steps run first and the seeded worlds are then restored.
"""
import argparse
import json
import os
import statistics
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

from puffysics_b200.configs import CONFIGS  # noqa: E402

METRIC = "physics-only env-steps/sec (worlds×steps/s) at 1/2/4/8 B200; % HBM roofline"
UNIT = "env-steps/s"
SEED = 1
L2_BYTES = 126e6
STATE_ONLY = 4       # B3X_STEP_STATE_ONLY

# Algorithmic bytes of one world-step, read + write, minimal SoA model:
# dynamic body 196 B (pose+velocity 52 r / 52 w, force+torque 24 r / 24 w,
# constants 44 r), other body 44 B, shape 84 B, contact 136 B (warm cache
# 68 r / 68 w), joint 208 B (constants 112 r, impulses 48 r / 48 w).
BYTES_DYN_BODY, BYTES_BODY, BYTES_SHAPE, BYTES_CONTACT, BYTES_JOINT = 196, 44, 84, 136, 208

# fp32 operations of one world-step per scene (fadd + fmul + 2 x ffma of one
# step-kernel launch, counted by ncu on the benchmark workloads and committed
# under profiles/ with the commands that made them); None for scenes not
# counted.
FLOPS_FILE = os.path.join(ROOT, "profiles", "flops_per_world_step.md")
TRAFFIC_FILE_FMT = os.path.join(ROOT, "profiles", "%s_%s.md")      # (kernel, scene)

WORKLOAD = {"hover": "C1 hover (4,096 worlds/GPU)", "stack": "C2 box stack (16,384 worlds/GPU)",
            "chain": "C3 capsule chain (16,384 worlds/GPU)",
            "pile": "C4 pile (65,536 worlds/GPU, steps 1-240 from the seeded drop)",
            "scaleout": "C5 scale-out (1,048,576 C2 worlds in total, 1% reset per step)",
            "stackil": "C2 box stack in the B3_INTERLEAVE_CONTACTS mode (16,384 worlds/GPU)"}


def parse_args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=1000)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--config", default="stack", choices=sorted(WORKLOAD))
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--worlds", type=int, default=0, help="override worlds per GPU")
    ap.add_argument("--e2e-steps", type=int, default=200)
    ap.add_argument("--cpu-seconds", type=float, default=10.0, help="CPU baseline sample budget")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-graph", action="store_true", help="e2e with direct calls instead of a CUDA graph")
    ap.add_argument("--no-per-thread-path", action="store_true",
                    help="skip the timing of the per-thread device b3_step after the main measurement")
    ap.add_argument("--path", default="columns", choices=["columns", "columns_state_only", "aos"],
                    help="world layout of the headline: the AoS drop-in, or resident columns (b3x_engine_*), "
                         "optionally with the state-only write-back")
    ap.add_argument("--no-other-paths", action="store_true",
                    help="measure only the headline's world layout (no aos / columns comparison runs)")
    ap.add_argument("--extra-configs", default="pile",
                    help="comma list of configurations measured after the main one on one GPU ('' for none)")
    return ap.parse_args()


def read_number(path, key):
    """`key = number` from a committed profile summary, else None."""
    try:
        for line in open(path):
            if line.strip().startswith(key):
                return float(line.split("=", 1)[1].split()[0].replace(",", ""))
    except (OSError, ValueError, IndexError):
        pass
    return None


def host_threads():
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


def cpu_model():
    try:
        for line in open("/proc/cpuinfo"):
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


def window_of(cfg, name):
    """Steps from the seeded state a configuration is quoted over (0: open,
    the timed steps follow the warm-up)."""
    return cfg.steps if name == "pile" else 0


def per_gpu_worlds(cfg, name, world, override=0):
    return override or (cfg.worlds // world if name == "scaleout" else cfg.worlds)


def l2_rule(world_array):
    """(flush between timed steps?, note): a world array larger than twice
    the 126 MB L2 cannot stay resident; smaller ones are evicted by writing a
    256 MiB buffer outside the events."""
    if world_array < L2_BYTES * 2:
        return True, ("flushed between timed steps (256 MiB write outside the events); world array %.0f MB"
                      % (world_array / 1e6))
    return False, ("no flush: the world array (%.0f MB), read and written every step, is larger than twice "
                   "the 126 MB L2" % (world_array / 1e6))


def workload_config(cfg, name, per_gpu, world):
    """The `config` object of both arms' lines (identical keys and values)."""
    from puffysics_b200 import layout
    win = window_of(cfg, name)
    return {"workload": WORKLOAD[name], "scene": cfg.name, "worlds_per_gpu": per_gpu, "worlds": per_gpu * world,
            "dt": cfg.dt, "substeps": cfg.substeps, "solver_iters": cfg.joint_iters, "caps": list(cfg.caps),
            "timed_steps": ("steps 1-%d from the seeded state" % win) if win else "the steps after the warm-up",
            "l2": l2_rule(per_gpu * layout.world_bytes(*cfg.caps))[1],
            "parallelism": "dp%d (contiguous world shards, no per-step collective)" % world}


def cpu_reference_run(cfg, steps, warmup, budget_s, window=0):
    """Time the reference's CPU b3_batch_step (oracle/_ref) or, where it was
    not built, its restatement (oracle/port) over all host threads.  With a
    window, a sample of the configuration's worlds runs steps 1..window from
    the seeded state, the sample sized (by a calibration over the same
    window) to fill about budget_s seconds.  Otherwise, with steps=None the
    step count is chosen to fill budget_s on the configuration's full world
    count, else the world sample is sized."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as orc
    kind = "reference" if orc.available(cfg.name, "ref") else "port"
    o = orc.Oracle(cfg.name, "ref" if kind == "reference" else "port")
    threads = host_threads()
    if window:
        probe = o.build(threads, cfg.scene, SEED)
        t = o.run_mt(probe, cfg.scene, SEED, 0, 1, window, cfg.dt, cfg.substeps, threads)
        worlds = int(budget_s / max(t / len(probe), 1e-9))
        worlds = max(threads, min(cfg.worlds, worlds))
        w = o.build(worlds, cfg.scene, SEED)
        secs = o.run_mt(w, cfg.scene, SEED, 0, 1, window, cfg.dt, cfg.substeps, threads)
        steps = window
        desc = "steps 1-%d from the seeded state" % window
    else:
        # calibrate: a few steps over a small sample
        probe = o.build(threads * 8, cfg.scene, SEED)
        t = o.run_mt(probe, cfg.scene, SEED, 0, 1, 3, cfg.dt, cfg.substeps, threads)
        per_world_step = max(t, 1e-6) / (3 * len(probe))
        if steps is None:
            worlds = min(cfg.worlds, 262144)
            steps = int(min(2000, max(3, budget_s / (per_world_step * worlds))))
        else:
            worlds = int(budget_s / max(per_world_step * max(steps, 1), 1e-12))
            worlds = max(threads, min(cfg.worlds, worlds))
        w = o.build(worlds, cfg.scene, SEED)
        if warmup:
            o.run_mt(w, cfg.scene, SEED, 0, 1, warmup, cfg.dt, cfg.substeps, threads)
        secs = o.run_mt(w, cfg.scene, SEED, 0, 1 + warmup, steps, cfg.dt, cfg.substeps, threads)
        desc = "%d steps after %d warm-up steps" % (steps, warmup)
    value = worlds * steps / secs
    return {"value": value, "unit": UNIT, "cores": threads, "kind": kind, "ms_per_step": secs * 1e3 / steps,
            "sample": "%d of the configuration's worlds x %s, %s, contiguous partitions, one pthread per host "
                      "thread, %.2f s" % (worlds, desc, cpu_model(), secs)}


def time_steps(one, k, warmup, flush, stream, restart=None):
    """`warmup` calls of one(), then (restart() if given: back to the seeded
    state) k timed calls, CUDA events on `stream` around each, L2 flushed
    between them outside the events when `flush` is given; returns the
    summed milliseconds."""
    import torch
    for _ in range(max(warmup, 3)):
        one()
    torch.cuda.synchronize()
    if restart is not None:
        restart()
        torch.cuda.synchronize()
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(k)]
    for e0, e1 in ev:
        if flush is not None:
            flush.zero_()
        e0.record(stream)
        one()
        e1.record(stream)
    torch.cuda.synchronize()
    return sum(e0.elapsed_time(e1) for e0, e1 in ev)


def _steps_for_budget(one, steps, warmup, budget_s):
    """Warm-up calls (all but one untimed, the last one timed by the wall
    clock) and the number of timed steps that fits budget_s."""
    import torch
    for _ in range(max(warmup, 3) - 1):
        one()
    torch.cuda.synchronize()
    t0 = time.time()
    one()
    torch.cuda.synchronize()
    return int(max(3, min(steps or 100, budget_s / max(time.time() - t0, 1e-4))))


def reference_gpu_run(cfg, steps, warmup, budget_s=60.0, window=0):
    """Time the reference's own GPU batch step (b3_batch_step_gpu: one thread
    per AoS world, oracle/_ref/libb3refgpu_<cfg>.so built from the reference
    sources with its stock nvcc flags) on this GPU: the scene's actions
    (applied with the reference's b3_apply_* in a per-world kernel) plus one
    b3_batch_step_gpu per step, CUDA events on the launching stream, the
    same warm-up, timed steps (or window) and L2 rule as this library's arm.
    None when there is no GPU or the library was not built."""
    import ctypes
    try:
        import torch
        if not torch.cuda.is_available():
            return None
    except ImportError:
        return None
    path = os.path.join(ROOT, "oracle", "_ref", "libb3refgpu_%s.so" % cfg.name)
    if not os.path.exists(path):
        return None
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as orc
    L = ctypes.CDLL(path)
    vp, sz = ctypes.c_void_p, ctypes.c_size_t
    L.refgpu_world_bytes.restype = sz
    L.refgpu_batch_step.argtypes = [vp, sz, sz, ctypes.c_int, ctypes.c_float, ctypes.c_int, vp, vp]
    L.refgpu_batch_step.restype = ctypes.c_int
    L.refgpu_apply.argtypes = [vp, sz, sz, ctypes.c_int, ctypes.c_int, ctypes.c_ulonglong, ctypes.c_ulonglong,
                               ctypes.c_ulonglong, vp]
    L.refgpu_apply.restype = ctypes.c_int
    n = min(cfg.worlds, 131072)
    kind = "ref" if orc.available(cfg.name, "ref") else "port"
    host = orc.Oracle(cfg.name, kind).build(n, cfg.scene, SEED)
    wb = host.shape[1]
    assert wb == L.refgpu_world_bytes()
    dev = torch.device("cuda", torch.cuda.current_device())
    worlds = torch.from_numpy(host).to(dev)
    seeded = worlds.clone() if window else None
    del host
    stream = torch.cuda.current_stream(dev)
    sp = ctypes.c_void_p(stream.cuda_stream)
    step_no = [0]

    def one():
        step_no[0] += 1
        assert L.refgpu_apply(worlds.data_ptr(), wb, 0, n, cfg.scene, SEED, 0, step_no[0], sp) == 0
        assert L.refgpu_batch_step(worlds.data_ptr(), wb, 0, n, cfg.dt, cfg.substeps, None, sp) == 0

    def restart():
        worlds.copy_(seeded)
        step_no[0] = 0

    if window:
        k = window
        for _ in range(max(warmup, 3) - 1):
            one()
    else:
        k = _steps_for_budget(one, steps, warmup, budget_s)
    flush = torch.empty(256 * 1024 * 1024, dtype=torch.uint8, device=dev) if n * wb < L2_BYTES * 2 else None
    ms = time_steps(one, k, 1, flush, stream, restart if window else None)
    return {"value": n * k / (ms / 1e3), "unit": UNIT, "ms_per_step": ms / k, "worlds": n, "steps": k,
            "l2": "flushed between timed steps" if flush is not None else "world array larger than twice L2",
            "timed_steps": ("steps 1-%d from the seeded state" % window) if window else "after the warm-up",
            "kernel": "reference b3_batch_step_gpu (b3_batch.cuh:63-89), one thread per world, nvcc -O3 sm_100a",
            "note": "the reference's GPU kernel on this GPU, timed like the step (actions + step, events)"}


HOVER_ENVS = 4096    # puffysics_hover.ini [vec] total_agents


def fused_env_run(steps, warmup, stream):
    """The PufferLib hover environment step fused into one launch
    (libb3hover.so): action, physics, reward, terminal, log, automatic reset
    and observation of 4,096 environments per step."""
    import torch
    from puffysics_b200 import hover_env
    n = HOVER_ENVS
    dev = torch.device("cuda", torch.cuda.current_device())
    envs = torch.zeros((n, hover_env.env_bytes()), dtype=torch.uint8, device=dev)
    assert hover_env.init(envs, SEED, stream) == 0
    obs = torch.zeros((n, 3), dtype=torch.float32, device=dev)
    rew = torch.zeros(n, dtype=torch.float32, device=dev)
    term = torch.zeros(n, dtype=torch.float32, device=dev)
    g = torch.Generator(device=dev)
    g.manual_seed(SEED)
    acts = torch.randint(0, 3, (16, n), generator=g, device=dev).float()
    k_no = [0]

    def one():
        k_no[0] += 1
        assert hover_env.step(envs, acts[k_no[0] % 16], obs, rew, term, stream) == 0

    flush = torch.empty(256 * 1024 * 1024, dtype=torch.uint8, device=dev)
    ms = time_steps(one, steps, warmup, flush, stream) / steps
    return {"value": n / (ms / 1e3), "unit": UNIT, "ms_per_step": ms, "envs": n, "steps": steps,
            "kernel": "b3x_hover_step_gpu: environments staged in shared memory, eight per 32-thread block",
            "l2": "flushed between timed steps"}


def reference_gpu_env_run(steps, warmup):
    """The reference hover adapter's step kernel shape (puffysics_hover.cu:40-43:
    one thread per environment in place) over the reference's hover_task.h,
    oracle/_ref/libb3refgpu_hoverenv.so; same environments and actions as
    fused_env_run."""
    import ctypes
    import torch
    path = os.path.join(ROOT, "oracle", "_ref", "libb3refgpu_hoverenv.so")
    if not torch.cuda.is_available() or not os.path.exists(path):
        return None
    L = ctypes.CDLL(path)
    vp = ctypes.c_void_p
    L.refhover_task_bytes.restype = ctypes.c_size_t
    L.refhover_gpu_init.argtypes = [vp, ctypes.c_int, ctypes.c_float, ctypes.c_float, ctypes.c_float, ctypes.c_int,
                                    ctypes.c_int, ctypes.c_uint, vp]
    L.refhover_gpu_step.argtypes = [vp, vp, ctypes.c_int, vp, vp, vp, vp, vp]
    n = HOVER_ENVS
    dev = torch.device("cuda", torch.cuda.current_device())
    stream = torch.cuda.current_stream(dev)
    sp = ctypes.c_void_p(stream.cuda_stream)
    tasks = torch.zeros((n, L.refhover_task_bytes()), dtype=torch.uint8, device=dev)
    logs = torch.zeros((n, 5), dtype=torch.float32, device=dev)
    assert L.refhover_gpu_init(tasks.data_ptr(), n, 2.0, 10.0, 1.0 / 60.0, 4, 256, SEED, sp) == 0
    obs = torch.zeros((n, 3), dtype=torch.float32, device=dev)
    rew = torch.zeros(n, dtype=torch.float32, device=dev)
    term = torch.zeros(n, dtype=torch.float32, device=dev)
    g = torch.Generator(device=dev)
    g.manual_seed(SEED)
    acts = torch.randint(0, 3, (16, n), generator=g, device=dev).float()
    k_no = [0]

    def one():
        k_no[0] += 1
        assert L.refhover_gpu_step(tasks.data_ptr(), logs.data_ptr(), n, acts[k_no[0] % 16].data_ptr(),
                                   obs.data_ptr(), rew.data_ptr(), term.data_ptr(), sp) == 0

    flush = torch.empty(256 * 1024 * 1024, dtype=torch.uint8, device=dev)
    ms = time_steps(one, steps, warmup, flush, stream) / steps
    return {"value": n / (ms / 1e3), "unit": UNIT, "ms_per_step": ms, "envs": n, "steps": steps,
            "kernel": "reference hover task (hover_task.h) in the adapter's kernel shape, one thread per "
                      "environment in place, nvcc -O3 sm_100a", "l2": "flushed between timed steps"}


def thread_path_run(cfg, n, steps, warmup, stream, budget_s=60.0, window=0, adapter=False):
    """Time this library's per-thread device b3_step (include/puffysics.cuh,
    one thread per world, libb3thread_<cfg>.so; with `adapter`, the same
    header built with nvcc's default contraction as an adapter builds it,
    libb3thread_<cfg>_adapter.so) over the stretch of the scene the reference
    GPU kernel is timed on: freshly built worlds, the scene's actions from
    step 1 (one launch, like the reference arm's action kernel), the same
    warm-up, timed steps (or window) and L2 rule; CUDA events on `stream`
    around each step."""
    import torch
    from puffysics_b200 import engine, synth
    name = cfg.name + ("_adapter" if adapter else "")
    try:
        engine.thread_lib(name)
    except RuntimeError:
        return None
    dev = torch.device("cuda", torch.cuda.current_device())
    w = torch.from_numpy(synth.SceneLib(cfg).build(n, SEED)).to(dev)
    seeded = w.clone() if window else None
    nv = cfg.action[2]
    step_no = [0]

    def one():
        step_no[0] += 1
        if nv:
            assert engine.thread_scene_apply_gpu(name, w, cfg.scene, SEED, 0, step_no[0], stream) == 0
        assert engine.thread_step_gpu(name, w, cfg.dt, cfg.substeps, stream=stream) == 0

    def restart():
        w.copy_(seeded)
        step_no[0] = 0

    if window:
        k = window
        for _ in range(max(warmup, 3) - 1):
            one()
    else:
        k = _steps_for_budget(one, steps, warmup, budget_s)
    flush = torch.empty(256 * 1024 * 1024, dtype=torch.uint8, device=dev) if w.numel() < L2_BYTES * 2 else None
    ms = time_steps(one, k, 1, flush, stream, restart if window else None)
    del w, seeded
    return {"value": n * k / (ms / 1e3), "unit": UNIT, "ms_per_step": ms / k, "worlds": n, "steps": k,
            "l2": "flushed between timed steps" if flush is not None else "world array larger than twice L2",
            "timed_steps": ("steps 1-%d from the seeded state" % window) if window else "after the warm-up",
            "kernel": "per-thread device b3_step of include/puffysics.cuh (one thread per world), "
                      + ("built with nvcc's default contraction, as an adapter compiles the header"
                         if adapter else "the parity build (-fmad=false: bit-exact with the CPU reference)")}


class ClockSampler:
    """NVML clocks and throttle reasons sampled every 20 ms (read only)."""

    REASONS = {0x1: "gpu_idle", 0x2: "applications_clocks_setting", 0x4: "sw_power_cap", 0x8: "hw_slowdown",
               0x20: "sw_thermal_slowdown", 0x40: "hw_thermal_slowdown", 0x80: "hw_power_brake_slowdown"}

    def __init__(self, device):
        self.samples, self.reasons, self.ok = [], set(), False
        try:
            import pynvml
            pynvml.nvmlInit()
            self.nv = pynvml
            self.h = pynvml.nvmlDeviceGetHandleByIndex(device)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
            self.ok = True
        except Exception:
            self.max_mhz = None
        self._stop = threading.Event()

    def _run(self):
        nv = self.nv
        while not self._stop.is_set():
            try:
                self.samples.append(nv.nvmlDeviceGetClockInfo(self.h, nv.NVML_CLOCK_SM))
                get = getattr(nv, "nvmlDeviceGetCurrentClocksEventReasons", None) or \
                    nv.nvmlDeviceGetCurrentClocksThrottleReasons
                r = get(self.h)
                for bit, name in self.REASONS.items():
                    if r & bit:
                        self.reasons.add(name)
            except Exception:
                pass
            time.sleep(0.02)

    def __enter__(self):
        if self.ok:
            self.t = threading.Thread(target=self._run, daemon=True)
            self.t.start()
        return self

    def __exit__(self, *exc):
        if self.ok:
            self._stop.set()
            self.t.join()

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": sorted(self.reasons), "samples": 0}
        return {"sm_mhz": statistics.median(self.samples), "sm_max_mhz": self.max_mhz,
                "reasons": sorted(self.reasons - {"gpu_idle"}), "samples": len(self.samples)}


def run_ours(name, args, rank, world, local, dev, barrier, path="columns"):
    """This library's arm on one configuration: the device-resident timed
    steps (the headline's K after W warm-up steps, or a configuration's
    window from its seeded state), then the end-to-end steps through host
    buffers.  path "columns": the worlds resident as structure-of-arrays
    columns (b3x_engine_*: bound once from the seeded AoS worlds, outside the
    timing); "aos": the drop-in b3x_batch_step_gpu on the AoS worlds.
    Returns the per-rank timings and the final state's counts."""
    import torch
    from puffysics_b200 import engine, layout, shard, synth
    cfg = CONFIGS[name]
    window = window_of(cfg, name)
    per_gpu = per_gpu_worlds(cfg, name, world, args.worlds if name == args.config else 0)
    first = rank * per_gpu
    caps = cfg.caps
    kind, aidx, nv = cfg.action

    scenes = synth.SceneLib(cfg)
    worlds = torch.from_numpy(scenes.build(per_gpu, SEED, first=first)).to(dev)
    seeded = worlds.clone() if (cfg.reset_fraction or window) else None
    stream = torch.cuda.current_stream(dev)
    cols = engine.Columns(caps, per_gpu, device=dev) if path.startswith("columns") else None
    # the state-only write-back (b3x_engine_step's B3X_STEP_STATE_ONLY)
    step_flags = cfg.flags | (STATE_ONLY if path == "columns_state_only" else 0)
    if cols is not None:
        assert cols.bind(worlds, stream=stream) == 0
    # set-up: the step's workspace for this stream (the step itself never allocates)
    assert engine.reserve_workspace(caps, stream) == 0
    vals = torch.zeros((per_gpu, max(nv, 1)), dtype=torch.float32, device=dev)
    reset = torch.zeros(per_gpu, dtype=torch.uint8, device=dev)
    world_array = per_gpu * layout.world_bytes(*caps)
    need_flush, _ = l2_rule(world_array)
    flush = torch.empty(256 * 1024 * 1024, dtype=torch.uint8, device=dev) if need_flush else None
    step_no = [0]
    step_launches = engine.step_launches(caps, per_gpu, local)

    def one_step(ev=None):
        """Actions (+ reset) then the step, all on `stream`; returns kernels launched."""
        step_no[0] += 1
        s = step_no[0]
        launches = 0
        if cfg.reset_fraction:
            assert synth.reset_gpu(reset, per_gpu, SEED, first, s, stream) == 0
            if cols is not None:
                assert cols.bind(seeded, select=reset, stream=stream) == 0
            else:
                assert engine.batch_restore_gpu(worlds, seeded, reset, stream, caps) == 0
            launches += 2
        if nv:
            assert synth.actions_gpu(vals, per_gpu, cfg.scene, SEED, first, s, stream) == nv
            if cols is not None:
                assert cols.apply(kind, aidx, vals, stream=stream) == 0
            else:
                assert engine.batch_apply_gpu(worlds, kind, aidx, vals, None, stream, caps) == 0
            launches += 2
        if ev is not None:
            ev.record(stream)
        if cols is not None:
            rc = cols.step(cfg.dt, cfg.substeps, None, stream, cfg.joint_iters, cfg.relax_iters, flags=step_flags)
        else:
            rc = engine.batch_step_gpu(worlds, cfg.dt, cfg.substeps, None, stream, caps, cfg.joint_iters,
                                       cfg.relax_iters, flags=cfg.flags)
        assert rc == 0, rc
        return launches + step_launches

    def restart():
        if cols is not None:
            assert cols.bind(seeded, stream=stream) == 0
        else:
            worlds.copy_(seeded)
        step_no[0] = 0

    for _ in range(max(args.warmup, 3)):
        one_step()
    torch.cuda.synchronize(dev)
    if window:
        restart()
    K = window or args.steps
    ev0 = [torch.cuda.Event(enable_timing=True) for _ in range(K)]
    evk = [torch.cuda.Event(enable_timing=True) for _ in range(K)]
    ev1 = [torch.cuda.Event(enable_timing=True) for _ in range(K)]
    launches = 0
    barrier()
    torch.cuda.synchronize(dev)
    sampler = ClockSampler(local)
    with sampler:
        for i in range(K):
            if flush is not None:
                flush.zero_()                  # evict L2 between timed steps (outside the events)
            ev0[i].record(stream)
            launches += one_step(evk[i])
            ev1[i].record(stream)
        torch.cuda.synchronize(dev)
    barrier()
    t_local = sum(ev0[i].elapsed_time(ev1[i]) for i in range(K))
    k_local = sum(evk[i].elapsed_time(ev1[i]) for i in range(K))

    # diagnostics of the final state (outside the timed region)
    if cols is not None:
        # (after state-only steps the header counts and bodies read here are whole)
        assert cols.sync_to_aos(worlds, stream=stream) == 0
    final = worlds.cpu().numpy()
    stats = shard.world_stats(final, caps)
    v = layout.view(final, caps)
    counts = {"dyn": float((v["bodies"]["type"][:, :] == 2).sum(1).mean()), "body": float(v["body_count"].mean()),
              "shape": float(v["shape_count"].mean()), "contact": float(v["contact_count"].mean()),
              "joint": float(v["joint_count"].mean())}
    del final, v

    # e2e through the C-ABI with host buffers (pinned), synchronising per step
    E = window or min(args.e2e_steps, K)
    h_act = torch.zeros((per_gpu, max(nv, 1)), dtype=torch.float32).pin_memory()
    h_obs = torch.zeros((per_gpu, 13), dtype=torch.float32).pin_memory()
    d_obs = torch.zeros((per_gpu, 13), dtype=torch.float32, device=dev)
    obs_body = aidx if kind in (0, 1, 2) else caps[0] - 1
    obs_body = min(obs_body, int(counts["body"]) - 1)
    act_src = [torch.from_numpy(scenes.actions(per_gpu, SEED, first, step_no[0] + 1 + i)).contiguous()
               for i in range(min(E, 4))] if nv else []

    def e2e_ops(s):
        """One environment step through the C-ABI on stream s: the actions
        from pinned host memory, apply, step, observe, observations back."""
        if nv:
            vals.copy_(h_act[:, :nv], non_blocking=True)
            if cols is not None:
                assert cols.apply(kind, aidx, vals, stream=s) == 0
            else:
                assert engine.batch_apply_gpu(worlds, kind, aidx, vals, None, s, caps) == 0
        if cols is not None:
            assert cols.step(cfg.dt, cfg.substeps, None, s, cfg.joint_iters, cfg.relax_iters, flags=step_flags) == 0
            assert cols.observe(obs_body, d_obs, stream=s) == 0
        else:
            assert engine.batch_step_gpu(worlds, cfg.dt, cfg.substeps, None, s, caps, cfg.joint_iters,
                                         cfg.relax_iters, flags=cfg.flags) == 0
            assert engine.batch_observe_gpu(worlds, obs_body, d_obs, s, caps) == 0
        h_obs.copy_(d_obs, non_blocking=True)

    # The step's calls are captured once in a CUDA graph and replayed every
    # step (the host writes that step's actions into the pinned buffer first,
    # then waits for the observations).  The capture stream gets its own
    # workspace reservation first (set-up, outside the timing), and one
    # direct call runs on it before the capture.  Falls back to direct calls
    # if capture is refused.
    gstream = torch.cuda.Stream(dev)
    gstream.wait_stream(stream)
    assert engine.reserve_workspace(caps, gstream) == 0
    graph, e2e_mode = None, "direct calls"
    with torch.cuda.stream(gstream):
        e2e_ops(gstream)
    gstream.synchronize()
    if not args.no_graph:
        try:
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph, stream=gstream):
                e2e_ops(gstream)
            e2e_mode = "one CUDA graph replay"
        except RuntimeError:
            graph = None
            torch.cuda.synchronize(dev)
    if window:
        restart()
    barrier()
    torch.cuda.synchronize(dev)
    e_start, e_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(gstream):
        e_start.record(gstream)
        for i in range(E):
            if nv:
                h_act[:, :nv].copy_(act_src[i % len(act_src)])
            if graph is not None:
                graph.replay()
            else:
                e2e_ops(gstream)
            gstream.synchronize()
        e_end.record(gstream)
    torch.cuda.synchronize(dev)
    e2e_local = e_start.elapsed_time(e_end)
    del graph
    assert engine.release_workspaces() == 0
    if path.startswith("columns"):
        e2e_path = ("pinned H2D actions -> b3x_engine_apply -> b3x_engine_step -> b3x_engine_observe -> D2H "
                    "(%s), stream synchronised every step" % e2e_mode)
    else:
        e2e_path = ("pinned H2D actions -> b3x_batch_apply_gpu -> b3x_batch_step_gpu -> b3x_batch_observe_gpu -> "
                    "D2H (%s), stream synchronised every step" % e2e_mode)
    del cols
    return {"name": name, "cfg": cfg, "per_gpu": per_gpu, "K": K, "E": E, "window": window, "path": path,
            "e2e_path": e2e_path,
            "t": t_local, "k": k_local, "e2e": e2e_local, "launches": launches, "step_launches": step_launches,
            "stats": stats, "counts": counts, "clocks": sampler.summary(),
            "bi": per_gpu * nv * 4, "bo": per_gpu * 13 * 4, "e2e_mode": e2e_mode}


def roofline(res, kern_s, local):
    """HBM roofline of the step kernel (algorithmic bytes / event time) and
    the fp32 work against one add or mul per lane per clock."""
    from puffysics_b200 import engine
    cfg, per_gpu, c = res["cfg"], res["per_gpu"], res["counts"]
    bytes_world = (c["dyn"] * BYTES_DYN_BODY + (c["body"] - c["dyn"]) * BYTES_BODY + c["shape"] * BYTES_SHAPE
                   + c["contact"] * BYTES_CONTACT + c["joint"] * BYTES_JOINT)
    alg_bytes = bytes_world * per_gpu
    peaks = {}
    try:
        peaks = json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json")))
    except (OSError, ValueError):
        pass
    hbm_peak = peaks.get("hbm_gbs") or 6650.0
    achieved = alg_bytes / kern_s / 1e9
    # worlds small enough to be stepped whole in shared memory take the
    # small-world kernel: one launch for any batch size
    small_path = engine.step_launches(cfg.caps, 1 << 20, local) == 1
    kname = "small_step_kernel" if small_path else "step_kernel"
    if res["path"].startswith("columns"):
        kname += "_columns"
    traffic = read_number(TRAFFIC_FILE_FMT % (kname, cfg.name), "dram_bytes_per_world_step")
    flops_ws = read_number(FLOPS_FILE, "%s_flops_per_world_step" % cfg.name)
    sm_max = (peaks.get("sm_max_mhz") or 1965.0)
    fp32_peak = 148 * 128 * sm_max * 1e6 / 1e12      # one fp32 add or mul per lane per clock
    roof = {"bound": "hbm", "achieved": achieved, "peak": hbm_peak, "unit": "GB/s", "frac": achieved / hbm_peak,
            "traffic": traffic * per_gpu / res["step_launches"] if traffic else None,
            "peak_source": "MEASURED_PEAKS.json hbm_gbs" if peaks.get("hbm_gbs") else "fallback 6650 GB/s",
            "kernel": ("b3x::small_step_kernel (worlds staged whole in shared memory, one thread per "
                       "world; %d launch per step)" if small_path else
                       "b3x::step_kernel (collide, solve and write-back phases; %d launch(es) per step)")
                      % res["step_launches"] + (" on the resident world columns" if res["path"].startswith("columns")
                                                else " on the caller's AoS worlds"),
            "kernel_ms": kern_s * 1e3,
            "traffic_source": "profiles/%s_%s.md" % (kname, cfg.name) if traffic else None,
            "algorithmic_bytes_per_launch": alg_bytes / res["step_launches"],
            "algorithmic_bytes_per_world_step": bytes_world,
            "per_launch": "achieved = algorithmic bytes of the step's launches / their summed event time; "
                          "traffic = ncu DRAM bytes of one launch"}
    if flops_ws:
        tf = flops_ws * per_gpu / kern_s / 1e12
        roof["fp32"] = {"achieved": tf, "peak": fp32_peak, "unit": "TFLOP/s", "frac": tf / fp32_peak,
                        "flops_per_world_step": flops_ws,
                        "peak_note": "148 SMs x 128 fp32 lanes x 1 add-or-mul per clock at max SM clock "
                                     "(the parity build contracts no multiply-add)"}
    return roof


def main():
    args = parse_args()
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    extras = [n for n in args.extra_configs.split(",") if n and n != args.config] if world == 1 else []
    cfg = CONFIGS[args.config]
    if args.impl == "reference":
        if rank != 0:
            return
        per_gpu = per_gpu_worlds(cfg, args.config, world, args.worlds)
        win = window_of(cfg, args.config)
        ref = cpu_reference_run(cfg, args.steps, args.warmup, budget_s=max(30.0, args.cpu_seconds), window=win)
        ref_gpu = reference_gpu_run(cfg, args.steps, args.warmup, window=win)
        ref_env = reference_gpu_env_run(args.steps, args.warmup) if cfg.name == "hover" else None
        line = {"impl": "reference", "metric": METRIC, "value": ref["value"], "unit": UNIT, "n_gpus": world,
                "steps": args.steps, "warmup": args.warmup,
                "ms_per_step": per_gpu * world / ref["value"] * 1e3, "higher_is_better": True,
                "scaling": "strong" if args.config == "scaleout" else "weak", "vs_baseline": None,
                "dtype": "f32", "data": "synthetic: seeded scenes (puffysics_b200/scenes/b3_scenes.h), "
                                        "actions from the same generator",
                "config": workload_config(cfg, args.config, per_gpu, world),
                "cpu_baseline": ref,
                "e2e": {"value": ref["value"], "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
                "ms_per_step_note": "the configuration's worlds / the CPU sample's env-steps/s",
                "reference_gpu": ref_gpu}
        if ref_env:
            line["reference_gpu_env"] = ref_env
        if extras:
            line["configs"] = {}
            for name in extras:
                c = CONFIGS[name]
                w = window_of(c, name)
                r = cpu_reference_run(c, None, 2, budget_s=args.cpu_seconds, window=w)
                pg = per_gpu_worlds(c, name, 1)
                line["configs"][name] = {
                    "value": r["value"], "unit": UNIT, "ms_per_step": pg / r["value"] * 1e3,
                    "config": workload_config(c, name, pg, 1), "cpu_baseline": r,
                    "e2e": {"value": r["value"], "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
                    "reference_gpu": reference_gpu_run(c, args.steps, args.warmup, window=w)}
        print(json.dumps(line), flush=True)
        return

    import torch
    import torch.distributed as dist
    from puffysics_b200 import build, shard

    build.build()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=dev)

    def barrier():
        if world > 1:
            dist.barrier()

    res = run_ours(args.config, args, rank, world, local, dev, barrier, path=args.path)

    # reductions (after timing): max time over ranks, summed diagnostics
    t_max, k_max, e_max = res["t"], res["k"], res["e2e"]
    if world > 1:
        tt = torch.tensor([t_max, k_max, e_max], dtype=torch.float64, device=dev)
        dist.all_reduce(tt, op=dist.ReduceOp.MAX)
        t_max, k_max, e_max = tt.tolist()
    tot = shard.reduce_stats(res["stats"], device=dev)

    def measured(r, t, k, e, nranks):
        """The measurement fields of one run (t, k, e: max-over-ranks ms)."""
        total = r["per_gpu"] * nranks
        return {"value": total * r["K"] / (t / 1e3), "unit": UNIT, "steps": r["K"], "warmup": args.warmup,
                "ms_per_step": t / r["K"], "world_path": r["path"],
                "roofline": roofline(r, k / r["K"] / 1e3, local),
                "e2e": {"value": total * r["E"] / (e / 1e3), "unit": UNIT, "h2d_bytes_per_step": r["bi"],
                        "d2h_bytes_per_step": r["bo"], "steps": r["E"], "path": r["e2e_path"]},
                "gpu_launches": r["launches"], "clocks": r["clocks"]}

    others = [] if args.no_other_paths else [p for p in ("aos", "columns", "columns_state_only") if p != args.path]
    if rank == 0:
        per_gpu = res["per_gpu"]
        stream = torch.cuda.current_stream(dev)
        line = {"metric": METRIC, "n_gpus": world,
                "higher_is_better": True,
                "scaling": "strong" if args.config == "scaleout" else "weak", "vs_baseline": None, "dtype": "f32",
                "data": "synthetic: seeded scenes (puffysics_b200/scenes/b3_scenes.h), on-device actions",
                "config": workload_config(res["cfg"], args.config, per_gpu, world)}
        line.update(measured(res, t_max, k_max, e_max, world))
        line["diagnostics"] = {"worlds": int(tot[0]), "contacts": int(tot[1]), "overflowed_worlds": int(tot[2]),
                               "dropped_contacts": int(tot[3]), "mean_contacts": res["counts"]["contact"],
                               "mean_bodies": res["counts"]["body"]}
        if world == 1:
            for other in others:
                r2 = run_ours(args.config, args, 0, 1, local, dev, barrier, path=other)
                line[other + "_path"] = measured(r2, r2["t"], r2["k"], r2["e2e"], 1)
        if world == 1 and not args.no_per_thread_path:
            line["per_thread_path"] = thread_path_run(res["cfg"], per_gpu, res["K"], args.warmup, stream,
                                                      window=res["window"])
            line["per_thread_path_adapter_build"] = thread_path_run(res["cfg"], per_gpu, res["K"], args.warmup,
                                                                    stream, window=res["window"], adapter=True)
            if res["cfg"].name == "hover":
                line["fused_env"] = fused_env_run(res["K"], args.warmup, stream)
        if world == 1 and not args.no_cpu_baseline:
            line["cpu_baseline"] = cpu_reference_run(res["cfg"], steps=None, warmup=2, budget_s=args.cpu_seconds,
                                                     window=res["window"])
        if extras:
            line["configs"] = {}
            for name in extras:
                r = run_ours(name, args, 0, 1, local, dev, barrier, path=args.path)
                sub = {"config": workload_config(r["cfg"], name, r["per_gpu"], 1)}
                sub.update(measured(r, r["t"], r["k"], r["e2e"], 1))
                sub["diagnostics"] = {"mean_contacts": r["counts"]["contact"], "mean_bodies": r["counts"]["body"],
                                      "overflowed_worlds": int(r["stats"][2]), "dropped_contacts": int(r["stats"][3])}
                for other in others:
                    r2 = run_ours(name, args, 0, 1, local, dev, barrier, path=other)
                    sub[other + "_path"] = measured(r2, r2["t"], r2["k"], r2["e2e"], 1)
                if not args.no_per_thread_path:
                    sub["per_thread_path"] = thread_path_run(r["cfg"], r["per_gpu"], r["K"], args.warmup, stream,
                                                             window=r["window"])
                    sub["per_thread_path_adapter_build"] = thread_path_run(r["cfg"], r["per_gpu"], r["K"],
                                                                           args.warmup, stream, window=r["window"],
                                                                           adapter=True)
                if not args.no_cpu_baseline:
                    sub["cpu_baseline"] = cpu_reference_run(r["cfg"], None, 2, budget_s=args.cpu_seconds,
                                                            window=r["window"])
                line["configs"][name] = sub
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
