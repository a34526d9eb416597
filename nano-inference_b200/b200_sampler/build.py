"""Build the sampler's CUDA library in-tree (``b200_sampler/libns_sampler.so``).

    python -m b200_sampler.build          (from nano-inference_b200/)

nvcc cross-compiles for sm_100a only; no GPU is needed to build.  The library
is a plain shared object with a C ABI (``include/ns_sampler.h``); it links the
CUDA runtime statically and uses no torch headers.
"""
from __future__ import annotations

import glob
import os
import shutil
import subprocess
import sys

PKG_DIR = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG_DIR)                     # nano-inference_b200/
REPO = os.path.dirname(ROOT)
CSRC = os.path.join(ROOT, "csrc")
INCLUDE = os.path.join(REPO, "include")
LIB_NAME = "libns_sampler.so"
LIB_PATH = os.path.join(PKG_DIR, LIB_NAME)

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-std=c++17", "-lineinfo",
    "-Xcompiler", "-fPIC,-O2",
    "-shared",
]


def nvcc_path() -> str:
    p = shutil.which("nvcc")
    if p:
        return p
    cand = "/usr/local/cuda/bin/nvcc"
    if os.path.exists(cand):
        return cand
    raise RuntimeError("nvcc not found")


def sources():
    return sorted(glob.glob(os.path.join(CSRC, "*.cu")))


HISTPACK_SRC = os.path.join(CSRC, "histpack.c")


def histpack_path() -> str:
    import sysconfig
    return os.path.join(PKG_DIR, "_histpack" + sysconfig.get_config_var("EXT_SUFFIX"))


def build_histpack(force: bool = False) -> str:
    """Compile the host-side history packer (a CPython extension, plain C)."""
    import sysconfig
    out = histpack_path()
    if not force and os.path.exists(out) and os.path.getmtime(out) >= os.path.getmtime(HISTPACK_SRC):
        return out
    cc = shutil.which("gcc") or shutil.which("cc")
    if cc is None:
        raise RuntimeError("no C compiler for the history packer")
    tmp = out + ".tmp"
    cmd = [cc, "-O3", "-shared", "-fPIC", "-I", sysconfig.get_paths()["include"], "-o", tmp, HISTPACK_SRC]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError("gcc failed:\n" + r.stdout + r.stderr)
    os.replace(tmp, out)
    return out


def _deps():
    return sources() + glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(INCLUDE, "*.h"))


def needs_build() -> bool:
    if not os.path.exists(LIB_PATH):
        return True
    t = os.path.getmtime(LIB_PATH)
    return any(os.path.getmtime(p) > t for p in _deps())


def build(force: bool = False, verbose: bool = False) -> str:
    """Compile csrc/*.cu into the in-tree shared library (and the history
    packer); returns the library's path."""
    build_histpack(force)
    if not force and not needs_build():
        return LIB_PATH
    tmp = LIB_PATH + ".tmp"
    cmd = [nvcc_path(), *NVCC_FLAGS, "-I", INCLUDE, "-I", CSRC, "-o", tmp, *sources()]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
        print(" ".join(cmd), flush=True)
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError("nvcc failed:\n" + r.stdout + r.stderr)
    if verbose:
        print(r.stdout + r.stderr)
    os.replace(tmp, LIB_PATH)
    return LIB_PATH


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="-v" in sys.argv))
