"""Builds tests/ref_binding/attn_cuda_binding.cpp into an importable module.

The module links against the in-tree ``libgfx906_b200_attn.so`` the way the
reference links its kernel object into its extension
(deploy/gfx906_attn.py:78-83): g++ on the binding source, the library on the
link line, nothing else. Test infrastructure only; rebuilt when the source,
the library or the flags change.
"""

from __future__ import annotations

import importlib.util
import os
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
REPO = HERE.parents[1]
if str(REPO) not in sys.path:
    sys.path.insert(0, str(REPO))

from gfx906_b200 import build as pkg_build  # noqa: E402

NAME = "gfx906_ref_cuda_binding"
SRC = HERE / "attn_cuda_binding.cpp"
OUT = HERE / (NAME + ".so")


def build(force: bool = False) -> Path:
    lib = pkg_build.build_library()
    cflags, ldflags, tver = pkg_build._torch_flags()
    cflags = [f for f in cflags if not f.startswith("-DTORCH_EXTENSION_NAME=")] + [f"-DTORCH_EXTENSION_NAME={NAME}"]
    cxx = os.environ.get("CXX", "g++")
    rpath = "-Wl,-rpath,$ORIGIN/" + os.path.relpath(lib.parent, HERE)
    digest = pkg_build._digest([SRC, lib], cflags + ldflags + [tver, cxx, rpath])
    if not force and pkg_build._fresh(OUT, digest):
        return OUT
    tmp = OUT.with_name(OUT.name + ".tmp")
    cmd = [cxx, "-O2", "-std=c++17", "-fPIC", "-shared", str(SRC), "-o", str(tmp), *cflags,
           f"-L{lib.parent}", "-lgfx906_b200_attn", rpath, *ldflags]
    pkg_build._run(cmd, HERE / ".cxx.log")
    os.replace(tmp, OUT)
    pkg_build._stamp(OUT, digest)
    return OUT


def load():
    """Imports the built module (builds it first if needed)."""
    path = build()
    spec = importlib.util.spec_from_file_location(NAME, path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


if __name__ == "__main__":
    print(build(force="--force" in sys.argv))
