"""Generate tests/golden/mjcf_walker.npz: the MJCF test robot
(tests/fixtures/mjcf/walker.xml) loaded and spawned by the reference's MJCF
loader (mjcf.h, compiled from the reference checkout against this library's
include/), as AoS B3World bytes at the default capacities: the bind pose and
the "crouch" keyframe.

    python tests/golden/gen_mjcf.py     # PUFFYSICS_REF=<checkout> to name it
"""
import os
import subprocess
import sys
import tempfile

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
FIX = os.path.join(ROOT, "tests", "fixtures", "mjcf")
sys.path.insert(0, ROOT)
import __graft_entry__  # noqa: E402

# the reference checkout: PUFFYSICS_REF, else where the build driver mounts it
REF_DIR = os.environ.get("PUFFYSICS_REF") or __graft_entry__.REFERENCE_MOUNT


def spawn(include_dirs, keys, workdir):
    exe = os.path.join(workdir, "spawn")
    subprocess.run(["gcc", "-O2", "-std=gnu11", "-ffp-contract=off"] + ["-I" + d for d in include_dirs]
                   + [os.path.join(FIX, "spawn.c"), "-o", exe, "-lm"], check=True)
    out = []
    for k in keys:
        path = os.path.join(workdir, "w_%s.bin" % k)
        subprocess.run([exe, os.path.join(FIX, "walker.xml"), k, path], check=True, capture_output=True)
        out.append(np.fromfile(path, dtype=np.uint8))
    return np.stack(out)


def main():
    if not REF_DIR or not os.path.exists(os.path.join(REF_DIR, "mjcf.h")):
        sys.exit("reference checkout not found at %s" % REF_DIR)
    with tempfile.TemporaryDirectory() as d:
        worlds = spawn([os.path.join(ROOT, "include"), REF_DIR], ["-", "crouch"], d)
    np.savez_compressed(os.path.join(HERE, "mjcf_walker.npz"), worlds=worlds, keys=np.array(["bind", "crouch"]))
    print(worlds.shape)


if __name__ == "__main__":
    main()
