"""C-ABI checks that need no GPU: the library builds for sm_100a, loads, and
exports every entry point include/puffysics_b200.h declares; the header's
struct layout equals the reference's for several capacity configurations."""
import ctypes
import os
import re
import subprocess

import numpy as np
import pytest

import oracle as orc
from puffysics_b200 import build, layout
from puffysics_b200.configs import CONFIGS

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "puffysics_b200.h")


def declared_symbols():
    text = open(HEADER).read()
    return sorted(set(re.findall(r"B3X_API\s+[\w\s\*]+?\b(b3x_\w+)\s*\(", text)))


@pytest.fixture(scope="module")
def lib():
    return ctypes.CDLL(build.build())


def test_library_exports_every_declared_symbol(lib):
    names = declared_symbols()
    assert len(names) >= 9
    for n in names:
        assert hasattr(lib, n), "missing export " + n


def test_world_bytes_match_layout(lib):
    lib.b3x_world_bytes.restype = ctypes.c_size_t
    lib.b3x_world_bytes.argtypes = [ctypes.c_ulonglong]
    for cfg in CONFIGS.values():
        assert lib.b3x_world_bytes(cfg.signature) == layout.world_bytes(*cfg.caps)
    assert layout.world_bytes(9, 9, 32, 1) == 18360       # C2 size quoted for the reference
    assert layout.world_bytes(2, 2, 4, 1) == 3016
    assert lib.b3x_world_bytes(0) == 0                     # zero capacities: invalid


PROBE = r"""
#include <stdio.h>
#include <stddef.h>
#include "%s"
int main(void) {
    printf("%%zu %%zu %%zu %%zu %%zu %%llu\n", sizeof(B3World), offsetof(B3World, bodies), offsetof(B3World, shapes),
           offsetof(B3World, contacts), offsetof(B3World, joints), (unsigned long long)B3_CONFIG_SIGNATURE);
    return 0;
}
"""


@pytest.mark.parametrize("caps", [(2, 2, 4, 1), (9, 9, 32, 1), (12, 12, 32, 10), (37, 37, 128, 1),
                                  (80, 128, 128, 32), (3, 5, 7, 2)])
@pytest.mark.parametrize("lang", ["c", "c++"])
def test_header_layout(tmp_path, caps, lang):
    src = tmp_path / ("probe." + ("c" if lang == "c" else "cpp"))
    src.write_text(PROBE % HEADER)
    exe = tmp_path / "probe"
    cc = "gcc" if lang == "c" else "g++"
    defs = ["-DB3_MAX_BODIES=%d" % caps[0], "-DB3_MAX_SHAPES=%d" % caps[1], "-DB3_MAX_CONTACTS=%d" % caps[2],
            "-DB3_MAX_JOINTS=%d" % caps[3]]
    subprocess.run([cc, "-Wall", "-Werror", "-Wno-unused-function"] + defs + [str(src), "-o", str(exe), "-lm"],
                   check=True)
    size, ob, os_, oc, oj, sig = map(int, subprocess.run([str(exe)], capture_output=True, text=True,
                                                         check=True).stdout.split())
    dt = layout.world_dtype(*caps)
    assert size == dt.itemsize
    assert (ob, os_, oc, oj) == tuple(dt.fields[k][1] for k in ("bodies", "shapes", "contacts", "joints"))
    assert sig == layout.signature(*caps)


def test_compat_include_names(tmp_path):
    """Adapters include "puffysics.cuh" / "b3_batch.cuh"; both resolve to this
    library's header in include/."""
    src = tmp_path / "adapter.c"
    src.write_text('#include "b3_batch.cuh"\n#include "puffysics.cuh"\n'
                   "int main(void){B3World w; b3_world_init(&w); B3BodyDef d = b3_default_body();"
                   "int b = b3_create_body(&w, &d); B3Batch bt = {&w, sizeof(B3World), 0, 1};"
                   "return !(b == 0 && b3_batch_valid(bt) && b3_batch_world(bt, 0) == &w);}\n")
    exe = tmp_path / "adapter"
    subprocess.run(["gcc", "-DB3_MAX_BODIES=4", "-DB3_MAX_SHAPES=4", "-DB3_MAX_CONTACTS=8", "-DB3_MAX_JOINTS=1",
                    "-I" + os.path.join(ROOT, "include"), str(src), "-o", str(exe), "-lm"], check=True)
    assert subprocess.run([str(exe)]).returncode == 0


@pytest.mark.parametrize("name", ["hover", "stack", "chain", "pile", "default", "stacksmall"])
def test_product_scene_builder_matches_reference_builder(name):
    from puffysics_b200.synth import SceneLib
    cfg = CONFIGS[name]
    kind = "ref" if orc.available(name, "ref") else "port"
    if kind == "port":
        orc.build_oracles()
    ours = SceneLib(cfg).build(6, 4242, first=10)
    theirs = orc.Oracle(name, kind).build(6, cfg.scene, 4242, first=10)
    assert np.array_equal(ours, theirs)


THREAD_EXPORTS = ["b3x_thread_signature", "b3x_thread_joint_iters", "b3x_thread_relax_iters",
                  "b3x_thread_step_gpu", "b3x_thread_step_worlds_gpu"]


@pytest.mark.parametrize("name", sorted(build.THREAD_CONFIGS))
def test_thread_libraries_export_launchers(lib, name):
    """libb3thread_<cfg>.so (include/puffysics.cuh's device b3_step) loads,
    exports its launchers, reports its capacities, and rejects invalid
    arguments before any device call."""
    from puffysics_b200 import engine
    L = engine.thread_lib(name)
    for n in THREAD_EXPORTS:
        assert hasattr(L, n)
    b, s, c, j, it = build.THREAD_CONFIGS[name]
    assert L.b3x_thread_signature() == layout.signature(b, s, c, j)
    assert L.b3x_thread_joint_iters() == it and L.b3x_thread_relax_iters() == it
    wb = layout.world_bytes(b, s, c, j)
    bad = [engine.B3Batch(None, wb, 0, 3), engine.B3Batch(None, wb, 0, -1), engine.B3Batch(64, wb - 8, 0, 1),
           engine.B3Batch(64, wb, 8, 1)]
    for bt in bad:
        assert L.b3x_thread_step_gpu(bt, 1 / 60, 4, None, None) == 1
    ok = engine.B3Batch(64, wb, 0, 1)
    assert L.b3x_thread_step_gpu(ok, float("inf"), 4, None, None) == 1
    assert L.b3x_thread_step_gpu(ok, 1 / 60, 0, None, None) == 1
    assert L.b3x_thread_step_gpu(engine.B3Batch(None, wb, 0, 0), 1 / 60, 4, None, None) == 0
    assert L.b3x_thread_step_worlds_gpu(None, -1, 1 / 60, 4, None) == 1
    assert L.b3x_thread_step_worlds_gpu(None, 0, 1 / 60, 4, None) == 0


def test_device_b3_step_in_adapter_kernels(tmp_path):
    """An adapter that calls b3_step from its own kernel, in two translation
    units that both include "puffysics.cuh", compiles for sm_100a and links
    (the header's device step has no duplicate external symbols)."""
    a = tmp_path / "env_a.cu"
    b = tmp_path / "env_b.cu"
    body = ('#include "puffysics.cuh"\n'
            "typedef struct Env { float reward; B3World world; } Env;\n"
            "__global__ void %s(Env* envs, int n) {\n"
            "  int i = blockIdx.x * blockDim.x + threadIdx.x;\n"
            "  if (i < n) { b3_apply_force(&envs[i].world, 1, b3_v(0, 1, 0));\n"
            "    b3_step(&envs[i].world, 1.0f / 60.0f, 4); envs[i].reward = envs[i].world.bodies[1].position.y; }\n"
            "}\n")
    a.write_text(body % "step_a" + "void launch_b(Env*, int);\n"
                 "void launch_a(Env* e, int n) { step_a<<<(n + 31) / 32, 32>>>(e, n);"
                 " b3_step_kernel<<<1, 32>>>(nullptr, 0, 0.0f, 1); launch_b(e, n); }\n")
    b.write_text(body % "step_b" + "void launch_b(Env* e, int n) { step_b<<<(n + 31) / 32, 32>>>(e, n); }\n"
                 "int main() { return 0; }\n")
    out = tmp_path / "adapter"
    cmd = [build.NVCC] + build.ARCH + ["-O1", "-std=c++17", "-DB3_MAX_BODIES=2", "-DB3_MAX_SHAPES=2",
                                       "-DB3_MAX_CONTACTS=4", "-DB3_MAX_JOINTS=1",
                                       "-I" + os.path.join(ROOT, "include"), str(a), str(b), "-o", str(out)]
    res = subprocess.run(cmd, capture_output=True, text=True)
    assert res.returncode == 0, res.stdout + res.stderr


def test_force_hook_adapter_uses_the_per_thread_step(tmp_path):
    """With B3_USER_FORCES defined, b3_batch_step_gpu compiles to the header's
    per-thread step (which runs the hook) and needs no library symbol."""
    src = tmp_path / "hooked.cu"
    src.write_text('#define B3_MAX_BODIES 2\n#define B3_MAX_SHAPES 2\n#define B3_MAX_CONTACTS 4\n'
                   '#define B3_MAX_JOINTS 1\n'
                   '#define B3_USER_FORCES(w, h) ((w)->bodies[0].force.y += 1.0f)\n'
                   '#include "b3_batch.cuh"\n'
                   'static_assert(B3_HAS_USER_FORCES, "hook seen");\n'
                   'int main() { B3Batch b = {nullptr, sizeof(B3World), 0, 0};\n'
                   '  return (int)b3_batch_step_gpu(b, 1.0f / 60.0f, 4, nullptr, 0); }\n')
    out = tmp_path / "hooked"
    cmd = [build.NVCC] + build.ARCH + ["-O1", "-std=c++17", "-I" + os.path.join(ROOT, "include"), str(src),
                                       "-o", str(out)]
    res = subprocess.run(cmd, capture_output=True, text=True)
    assert res.returncode == 0, res.stdout + res.stderr


def test_articulated_contacts_adapter_uses_the_per_thread_step(tmp_path):
    """With B3_ART_CONTACTS=1 the header accepts the macro, the device b3_step
    carries the articulated contact response and b3_batch_step_gpu compiles
    to that per-thread step (no library symbol needed)."""
    src = tmp_path / "art.cu"
    src.write_text('#define B3_MAX_BODIES 12\n#define B3_MAX_SHAPES 12\n#define B3_MAX_CONTACTS 32\n'
                   '#define B3_MAX_JOINTS 10\n#define B3_ART_CONTACTS 1\n'
                   '#include "b3_batch.cuh"\n'
                   'int main() { B3Batch b = {nullptr, sizeof(B3World), 0, 0};\n'
                   '  return (int)b3_batch_step_gpu(b, 1.0f / 60.0f, 4, nullptr, 0); }\n')
    out = tmp_path / "art"
    cmd = [build.NVCC] + build.ARCH + ["-O1", "-std=c++17", "-I" + os.path.join(ROOT, "include"), str(src),
                                       "-o", str(out)]
    res = subprocess.run(cmd, capture_output=True, text=True)
    assert res.returncode == 0, res.stdout + res.stderr
