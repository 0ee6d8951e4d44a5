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
