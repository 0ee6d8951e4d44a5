"""Build libpuffysics_b200.so (sm_100a) in-tree with nvcc.

    python -m puffysics_b200.build [-v]

Flags that matter for parity: -fmad=false (no fused multiply-add
contraction), -prec-div=true / -prec-sqrt=true / -ftz=false (IEEE division,
square root and denormals).  With them every float expression of the step
rounds exactly like the reference's CPU build with -ffp-contract=off.
"""
import os
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
LIB_DIR = os.path.join(PKG, "_lib")
LIB = os.path.join(LIB_DIR, "libpuffysics_b200.so")
SOURCES = [os.path.join(PKG, "csrc", "b3x_step.cu"), os.path.join(PKG, "csrc", "b3x_scenes.cu")]
HEADERS = [os.path.join(ROOT, "include", "puffysics_b200.h"),
           os.path.join(PKG, "csrc", "b3x_math.cuh"),
           os.path.join(PKG, "csrc", "b3x_narrow.cuh"),
           os.path.join(PKG, "csrc", "b3x_layout.cuh"),
           os.path.join(PKG, "csrc", "b3x_solver.cuh"),
           os.path.join(PKG, "csrc", "b3x_phases.cuh"),
           os.path.join(PKG, "csrc", "b3x_world_step.cuh"),
           os.path.join(PKG, "csrc", "b3x_art.cuh"),
           os.path.join(PKG, "scenes", "b3_scenes.h")]
SCENES_SRC = os.path.join(PKG, "scenes", "b3_scenes_host.c")
THREAD_SRC = os.path.join(PKG, "csrc", "b3x_thread_step.cu")
THREAD_HEADERS = [os.path.join(ROOT, "include", "puffysics.cuh"),
                  os.path.join(PKG, "csrc", "b3x_world_step.cuh"), os.path.join(PKG, "csrc", "b3x_art.cuh")]
# the hover environment fused into one launch per step (libb3hover.so)
HOVER_SRC = os.path.join(PKG, "csrc", "b3x_hover_env.cu")
HOVER_LIB = os.path.join(LIB_DIR, "libb3hover.so")
HOVER_HEADERS = THREAD_HEADERS + [os.path.join(ROOT, "include", "b3x_staged.cuh")]
THREAD_HEADERS = THREAD_HEADERS + [os.path.join(PKG, "scenes", "b3_test_forces.h")]
# what the per-thread libraries include
THREAD_DEPS = THREAD_HEADERS + [os.path.join(ROOT, "include", "puffysics_b200.h"),
                                os.path.join(PKG, "csrc", "b3x_math.cuh"), os.path.join(PKG, "csrc", "b3x_narrow.cuh"),
                                os.path.join(PKG, "scenes", "b3_scenes.h")]
# capacity configurations the host scene builders are compiled for:
# name -> (bodies, shapes, contacts, joints)
SCENE_CONFIGS = {"hover": (2, 2, 4, 1), "stack": (9, 9, 32, 1), "chain": (12, 12, 32, 10),
                 "pile": (37, 37, 128, 1), "hovertask": (2, 2, 4, 2), "default": (80, 128, 128, 32),
                 "stacksmall": (9, 9, 4, 1), "bounce": (9, 9, 32, 1), "capsule": (17, 17, 64, 1), "stackil": (9, 9, 32, 1),
                 "chainil": (12, 12, 32, 10), "bouncenr": (9, 9, 32, 1), "bounceilnr": (9, 9, 32, 1),
                 "hoveruf": (2, 2, 4, 1), "chainart": (12, 12, 32, 10)}
# per-thread step launchers (include/puffysics.cuh's device b3_step): name ->
# (bodies, shapes, contacts, joints, B3_JOINT_ITERS), the capacities of the
# benchmark configurations and of the reference's defaults
THREAD_CONFIGS = {"hover": (2, 2, 4, 1, 8), "stack": (9, 9, 32, 1, 8), "chain": (12, 12, 32, 10, 8),
                  "pile": (37, 37, 128, 1, 8), "hovertask": (2, 2, 4, 2, 2), "default": (80, 128, 128, 32, 2),
                  "bounce": (9, 9, 32, 1, 8), "capsule": (17, 17, 64, 1, 8), "stackil": (9, 9, 32, 1, 8),
                  "chainil": (12, 12, 32, 10, 8), "chainart": (12, 12, 32, 10, 8),
                  "bouncenr": (9, 9, 32, 1, 8), "bounceilnr": (9, 9, 32, 1, 8), "hoveruf": (2, 2, 4, 1, 8)}
# the same header step built the way an adapter compiles it (nvcc's default
# floating-point contraction instead of the parity flags), for timing beside
# the reference kernel, which is built that way too: libb3thread_<name>_adapter.so
ADAPTER_THREAD_CONFIGS = ["hover", "stack", "chain", "pile"]
# the reference's mode macros of the per-thread configurations
THREAD_MODES = {"stackil": ["-DB3_INTERLEAVE_CONTACTS"], "chainil": ["-DB3_INTERLEAVE_CONTACTS"],
                "bouncenr": ["-DB3_SKIP_RESTITUTION"],
                "bounceilnr": ["-DB3_INTERLEAVE_CONTACTS", "-DB3_SKIP_RESTITUTION"],
                "hoveruf": ["-include", os.path.join(PKG, "scenes", "b3_test_forces.h")],
                "chainart": ["-DB3_ART_CONTACTS=1"]}
CC = os.environ.get("CC", "gcc")

NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc" if os.path.exists("/usr/local/cuda/bin/nvcc") else "nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
PARITY = ["-fmad=false", "-prec-div=true", "-prec-sqrt=true", "-ftz=false"]


def nvcc_cmd(out=LIB, extra=()):
    return ([NVCC] + ARCH + ["-lineinfo", "-O3", "-std=c++17"] + PARITY
            + ["-Xcompiler", "-fPIC,-fvisibility=hidden", "-shared", "-cudart", "static",
               "-I" + os.path.join(ROOT, "include"), "-I" + os.path.join(PKG, "csrc"),
               "-I" + os.path.join(PKG, "scenes")]
            + list(extra) + SOURCES + ["-o", out])


def thread_lib(name):
    return os.path.join(LIB_DIR, "libb3thread_%s.so" % name)


def thread_cmd(name):
    adapter = name.endswith("_adapter")
    cfg = name[:-len("_adapter")] if adapter else name
    b, s, c, j, it = THREAD_CONFIGS[cfg]
    caps = ["-DB3_MAX_BODIES=%d" % b, "-DB3_MAX_SHAPES=%d" % s, "-DB3_MAX_CONTACTS=%d" % c,
            "-DB3_MAX_JOINTS=%d" % j, "-DB3_JOINT_ITERS=%d" % it] + THREAD_MODES.get(cfg, [])
    return ([NVCC] + ARCH + ["-lineinfo", "-O3", "-std=c++17"] + ([] if adapter else PARITY)
            + ["-Xcompiler", "-fPIC,-fvisibility=hidden", "-shared", "-cudart", "static",
               "-I" + os.path.join(ROOT, "include"), "-I" + os.path.join(PKG, "csrc"),
               "-I" + os.path.join(PKG, "scenes")]
            + caps + [THREAD_SRC, "-o", thread_lib(name)])


def thread_lib_names():
    return list(THREAD_CONFIGS) + [n + "_adapter" for n in ADAPTER_THREAD_CONFIGS]


def hover_cmd():
    return ([NVCC] + ARCH + ["-lineinfo", "-O3", "-std=c++17"] + PARITY
            + ["-Xcompiler", "-fPIC,-fvisibility=hidden", "-shared", "-cudart", "static",
               "-I" + os.path.join(ROOT, "include"), "-I" + os.path.join(PKG, "csrc"), HOVER_SRC, "-o", HOVER_LIB])


def build_thread_libs(force=False):
    """The per-thread step launchers, one per capacity configuration, and the
    hover environment library, compiled concurrently."""
    deps = [THREAD_SRC, __file__] + THREAD_DEPS
    todo = [n for n in thread_lib_names() if force or _newer(thread_lib(n), deps)]
    cmds = {n: thread_cmd(n) for n in todo}
    if force or _newer(HOVER_LIB, [HOVER_SRC, __file__] + THREAD_DEPS + HOVER_HEADERS):
        cmds["hover environment"] = hover_cmd()
    procs = [(n, subprocess.Popen(c, stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True))
             for n, c in cmds.items()]
    errors = []
    for n, p in procs:
        out, _ = p.communicate()
        if p.returncode != 0:
            errors.append("library %s failed:\n%s\n%s" % (n, " ".join(cmds[n]), out))
    if errors:
        raise RuntimeError("\n".join(errors))


def scenes_lib(name):
    return os.path.join(LIB_DIR, "libb3scenes_%s.so" % name)


def _newer(out, deps):
    if not os.path.exists(out):
        return True
    t = os.path.getmtime(out)
    return any(os.path.getmtime(d) > t for d in deps)


def up_to_date():
    deps = SOURCES + HEADERS + [__file__]
    thread_deps = [THREAD_SRC, __file__] + THREAD_DEPS
    return (not _newer(LIB, deps) and not any(_newer(scenes_lib(n), [SCENES_SRC] + HEADERS) for n in SCENE_CONFIGS)
            and not any(_newer(thread_lib(n), thread_deps) for n in thread_lib_names())
            and not _newer(HOVER_LIB, [HOVER_SRC, __file__] + THREAD_DEPS + HOVER_HEADERS))


def build_scenes(force=False):
    """Host scene builders, one per capacity configuration (gcc, exact float
    expressions: -ffp-contract=off)."""
    for name, (b, s, c, j) in SCENE_CONFIGS.items():
        out = scenes_lib(name)
        if not force and not _newer(out, [SCENES_SRC] + HEADERS):
            continue
        cmd = [CC, "-O2", "-ffp-contract=off", "-fno-fast-math", "-fPIC", "-shared", "-std=gnu11",
               "-fvisibility=hidden", "-DB3_MAX_BODIES=%d" % b, "-DB3_MAX_SHAPES=%d" % s,
               "-DB3_MAX_CONTACTS=%d" % c, "-DB3_MAX_JOINTS=%d" % j,
               "-I" + os.path.join(ROOT, "include"), "-I" + os.path.join(PKG, "scenes"), SCENES_SRC, "-o", out,
               "-lm"]
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            raise RuntimeError("scene builder build failed:\n" + " ".join(cmd) + "\n" + res.stdout + res.stderr)


def build(force=False, verbose=False):
    """Compile the library if any source is newer than it; returns its path."""
    if not force and up_to_date():
        return LIB
    os.makedirs(LIB_DIR, exist_ok=True)
    build_scenes(force)
    build_thread_libs(force)
    if not force and not _newer(LIB, SOURCES + HEADERS + [__file__]):
        return LIB
    cmd = nvcc_cmd(extra=["-Xptxas", "-v"] if verbose else [])
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError("nvcc failed:\n" + " ".join(cmd) + "\n" + res.stdout + res.stderr)
    if verbose:
        sys.stdout.write(res.stdout + res.stderr)
    return LIB


if __name__ == "__main__":
    print(build(force=True, verbose="-v" in sys.argv))
