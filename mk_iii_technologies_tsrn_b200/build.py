"""Build recipe for the in-tree CUDA library ``_tropical_b200.so`` (sm_100a).

Compiles every ``csrc/*.cu`` with nvcc for ``sm_100a`` only and links them
into one shared library next to this file.  The library exposes the C ABI
declared in ``include/tropical_b200.h``; Python reaches it through ctypes
(``_lib.py``).  Rebuilds only when a source or header is newer than the
library.  Run ``python -m mk_iii_technologies_tsrn_b200.build`` or call
:func:`build`.
"""
from __future__ import annotations

import glob
import os
import shutil
import subprocess
import sys

PKG_DIR = os.path.dirname(os.path.abspath(__file__))
REPO_DIR = os.path.dirname(PKG_DIR)
CSRC = os.path.join(PKG_DIR, "csrc")
INCLUDE = os.path.join(REPO_DIR, "include")
LIB_NAME = "_tropical_b200.so"
LIB_PATH = os.path.join(PKG_DIR, LIB_NAME)
BUILD_DIR = os.path.join(PKG_DIR, "_build")

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = [
    "-O3",
    "-lineinfo",
    "-std=c++17",
    "-Xcompiler",
    "-fPIC",
    "-Xcompiler",
    "-fvisibility=hidden",
    "--expt-relaxed-constexpr",
]


def _nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found; the tropical CUDA library cannot be built")


def _sources() -> list[str]:
    return sorted(glob.glob(os.path.join(CSRC, "*.cu")))


def _deps() -> list[str]:
    return (
        _sources()
        + glob.glob(os.path.join(CSRC, "*.cuh"))
        + glob.glob(os.path.join(INCLUDE, "*.h"))
        + [os.path.abspath(__file__)]
    )


def needs_build() -> bool:
    if not os.path.exists(LIB_PATH):
        return True
    lib_mtime = os.path.getmtime(LIB_PATH)
    return any(os.path.getmtime(p) > lib_mtime for p in _deps())


def build(force: bool = False, verbose: bool = False, ptxas_verbose: bool = False,
          extra_flags: list[str] | None = None, lib_path: str | None = None,
          build_dir: str | None = None) -> str:
    """Compile the library if needed and return its path.

    ``extra_flags`` (e.g. ``-DTP_TMA_TM=8``) and ``lib_path``/``build_dir`` build a
    variant library elsewhere without touching the in-tree one."""
    out_path = lib_path or LIB_PATH
    bdir = build_dir or BUILD_DIR
    if lib_path is None and not force and not needs_build():
        return LIB_PATH
    nvcc = _nvcc()
    os.makedirs(bdir, exist_ok=True)
    objs = []
    procs = []
    for src in _sources():
        obj = os.path.join(bdir, os.path.basename(src)[:-3] + ".o")
        cmd = [nvcc, *ARCH_FLAGS, *NVCC_FLAGS, *(extra_flags or []), "-I", INCLUDE, "-c", src,
               "-o", obj]
        if ptxas_verbose:
            cmd[1:1] = ["-Xptxas", "-v"]
        if verbose:
            print(" ".join(cmd), flush=True)
        procs.append((src, subprocess.Popen(cmd, stdout=subprocess.PIPE, stderr=subprocess.STDOUT)))
        objs.append(obj)
    failed = []
    for src, proc in procs:
        out, _ = proc.communicate()
        text = out.decode(errors="replace")
        if proc.returncode != 0:
            failed.append((src, text))
        elif (verbose or ptxas_verbose) and text.strip():
            print(text, flush=True)
    if failed:
        msg = "\n".join(f"--- {s}\n{t}" for s, t in failed)
        raise RuntimeError(f"nvcc failed:\n{msg}")
    tmp = out_path + ".tmp"
    link = [nvcc, *ARCH_FLAGS, "-shared", "-o", tmp, *objs, "-lcudart"]
    if verbose:
        print(" ".join(link), flush=True)
    res = subprocess.run(link, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"link failed:\n{res.stdout}\n{res.stderr}")
    os.replace(tmp, out_path)
    return out_path


if __name__ == "__main__":
    force = "--force" in sys.argv
    print(build(force=force, verbose="-v" in sys.argv, ptxas_verbose="--ptxas" in sys.argv))
