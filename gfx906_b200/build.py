"""In-tree build of the sm_100a attention library and its torch operator.

Two artefacts are built next to this file, so that they travel with the
source tree and no JIT cache is involved:

* ``libgfx906_b200_attn.so``: the C-ABI library (``include/gfx906_b200_attn.h``),
  compiled by nvcc for ``sm_100a`` only. It has no torch dependency; this is
  the object the reference's ``attn.cpp`` links against (the reference links
  ``attn_kernel.gfx906.o`` the same way, ``deploy/gfx906_attn.py:78-83``).
* ``_attn_ext<EXT_SUFFIX>``: the torch operator (``csrc/attn.cpp``), a pybind11
  module exposing ``attn(q, k, v, scale)``, linked to the library above.

Each artefact is rebuilt only when a hash of its sources, flags and compiler
changes (stored beside it as ``<artefact>.buildhash``); file modification
times are not trusted because source trees get copied between machines.
"""

from __future__ import annotations

import hashlib
import os
import shutil
import subprocess
import sys
import sysconfig
from pathlib import Path

PKG_DIR = Path(__file__).resolve().parent
REPO_DIR = PKG_DIR.parent
CSRC = PKG_DIR / "csrc"
INCLUDE = REPO_DIR / "include"

LIB_NAME = "libgfx906_b200_attn.so"
LIB_PATH = PKG_DIR / LIB_NAME
EXT_NAME = "_attn_ext"
EXT_PATH = PKG_DIR / (EXT_NAME + (sysconfig.get_config_var("EXT_SUFFIX") or ".so"))

# Every CUDA translation unit of the library.
CU_SOURCES = [CSRC / "attn_fwd_sm100.cu", CSRC / "attn_fwd_noalloc.cu"]
CU_HEADERS = [CSRC / "sm100_ptx.cuh", INCLUDE / "gfx906_b200_attn.h"]

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-lineinfo", "-O3", "-std=c++17",
    "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
    "-Xptxas", "-v",
]


class BuildError(RuntimeError):
    """A compiler invocation failed; the message carries the tail of its log."""


def nvcc_path() -> str:
    cand = shutil.which("nvcc")
    if cand:
        return cand
    for root in (os.environ.get("CUDA_HOME"), "/usr/local/cuda"):
        if root and Path(root, "bin", "nvcc").is_file():
            return str(Path(root, "bin", "nvcc"))
    raise BuildError("nvcc not found (set CUDA_HOME or put nvcc on PATH)")


def _digest(paths, extra) -> str:
    h = hashlib.sha256()
    for p in paths:
        h.update(str(Path(p).name).encode())
        h.update(Path(p).read_bytes())
    for e in extra:
        h.update(str(e).encode())
    return h.hexdigest()


def _fresh(target: Path, digest: str) -> bool:
    stamp = target.with_name(target.name + ".buildhash")
    return target.is_file() and stamp.is_file() and stamp.read_text().strip() == digest


def _stamp(target: Path, digest: str) -> None:
    target.with_name(target.name + ".buildhash").write_text(digest + "\n")


def _run(cmd, log_path: Path) -> str:
    res = subprocess.run(cmd, cwd=REPO_DIR, capture_output=True, text=True)
    log = " ".join(map(str, cmd)) + "\n" + res.stdout + res.stderr
    log_path.write_text(log)
    if res.returncode != 0:
        raise BuildError(f"build failed ({cmd[0]}):\n{log[-4000:]}")
    return log


def build_library(force: bool = False) -> Path:
    """Compile the C-ABI library (nvcc, sm_100a). Returns its path."""
    nvcc = nvcc_path()
    ver = subprocess.run([nvcc, "--version"], capture_output=True, text=True).stdout
    digest = _digest(CU_SOURCES + CU_HEADERS, NVCC_FLAGS + [ver])
    if not force and _fresh(LIB_PATH, digest):
        return LIB_PATH
    tmp = LIB_PATH.with_name(LIB_PATH.name + ".tmp")
    cmd = [nvcc, *NVCC_FLAGS, "-shared", "-o", str(tmp), *map(str, CU_SOURCES)]
    _run(cmd, PKG_DIR / ".nvcc.log")
    os.replace(tmp, LIB_PATH)
    _stamp(LIB_PATH, digest)
    return LIB_PATH


def _torch_flags():
    import torch
    from torch.utils import cpp_extension as ce

    inc = ce.include_paths(device_type="cuda")
    libs = ce.library_paths(device_type="cuda")
    abi = int(bool(torch._C._GLIBCXX_USE_CXX11_ABI))
    cflags = [f"-I{p}" for p in inc] + [f"-I{sysconfig.get_paths()['include']}"] + [
        f"-D_GLIBCXX_USE_CXX11_ABI={abi}",
        f"-DTORCH_EXTENSION_NAME={EXT_NAME}",
        "-DTORCH_API_INCLUDE_EXTENSION_H",
    ]
    ldflags = [f"-L{p}" for p in libs] + [f"-Wl,-rpath,{p}" for p in libs] + [
        "-lc10", "-lc10_cuda", "-ltorch", "-ltorch_cpu", "-ltorch_cuda", "-ltorch_python",
    ]
    return cflags, ldflags, torch.__version__


def build_extension(force: bool = False) -> Path:
    """Compile the torch operator module linked to the C-ABI library."""
    lib = build_library(force=force)
    cflags, ldflags, tver = _torch_flags()
    cxx = os.environ.get("CXX", "g++")
    src = CSRC / "attn.cpp"
    digest = _digest([src, INCLUDE / "gfx906_b200_attn.h", lib], cflags + ldflags + [tver, cxx])
    if not force and _fresh(EXT_PATH, digest):
        return EXT_PATH
    tmp = EXT_PATH.with_name(EXT_PATH.name + ".tmp")
    cmd = [cxx, "-O2", "-std=c++17", "-fPIC", "-shared", str(src), "-o", str(tmp), *cflags,
           f"-L{PKG_DIR}", "-lgfx906_b200_attn", "-Wl,-rpath,$ORIGIN", *ldflags]
    _run(cmd, PKG_DIR / ".cxx.log")
    os.replace(tmp, EXT_PATH)
    _stamp(EXT_PATH, digest)
    return EXT_PATH


def build_all(force: bool = False) -> None:
    build_library(force=force)
    build_extension(force=force)


if __name__ == "__main__":
    build_all(force="--force" in sys.argv)
    print(LIB_PATH)
    print(EXT_PATH)
