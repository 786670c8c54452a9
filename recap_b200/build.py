"""Build librecap_b200.so in-tree with nvcc for sm_100a.

Usage: ``python -m recap_b200.build`` (or ``recap_b200.build.build()``).  The library
is rebuilt when any source under ``recap_b200/csrc`` or ``include/`` is newer than it.
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

PACKAGE_DIR = Path(__file__).resolve().parent
REPO_DIR = PACKAGE_DIR.parent
CSRC = PACKAGE_DIR / "csrc"
INCLUDE = REPO_DIR / "include"
LIB_NAME = "librecap_b200.so"
LIB_PATH = PACKAGE_DIR / LIB_NAME
BUILD_DIR = PACKAGE_DIR / "_build"

SOURCES = ["layout.cu", "select.cu", "closure.cu", "cvk.cu", "coarse.cu", "fmha.cu", "refresh.cu", "selftest.cu",
           "exchange.cu", "capi.cu"]
ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = [
    "-O3",
    "-std=c++17",
    "-lineinfo",
    "-Xcompiler",
    "-fPIC",
    "--expt-relaxed-constexpr",
    "-Xptxas",
    "-v",
]


def _nvcc() -> str:
    cuda_home = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    cand = Path(cuda_home) / "bin" / "nvcc"
    if cand.exists():
        return str(cand)
    found = shutil.which("nvcc")
    if not found:
        raise RuntimeError("nvcc not found; set CUDA_HOME")
    return found


def _stale() -> bool:
    if not LIB_PATH.exists():
        return True
    built = LIB_PATH.stat().st_mtime
    inputs = list(CSRC.glob("*.cu")) + list(CSRC.glob("*.cuh")) + list(CSRC.glob("*.h"))
    inputs += list(INCLUDE.glob("*.h")) + [Path(__file__)]
    return any(p.stat().st_mtime > built for p in inputs)


def build(force: bool = False, verbose: bool = False, jobs: int | None = None) -> Path:
    """Compile every kernel source and link the shared library; returns its path."""
    if not force and not _stale():
        return LIB_PATH
    nvcc = _nvcc()
    BUILD_DIR.mkdir(exist_ok=True)
    objs = []
    procs = []
    for src in SOURCES:
        obj = BUILD_DIR / (Path(src).stem + ".o")
        objs.append(obj)
        cmd = [nvcc, *ARCH_FLAGS, *NVCC_FLAGS, "-I", str(INCLUDE), "-c", str(CSRC / src), "-o", str(obj)]
        procs.append((src, cmd, subprocess.Popen(cmd, stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True)))
    logs = []
    failed = []
    for src, cmd, p in procs:
        out, _ = p.communicate()
        logs.append(f"== {src}\n{out}")
        if p.returncode != 0:
            failed.append(src)
    (BUILD_DIR / "ptxas.log").write_text("\n".join(logs))
    if failed:
        raise RuntimeError("nvcc failed for " + ", ".join(failed) + "\n" + "\n".join(logs))
    tmp = LIB_PATH.with_suffix(".so.tmp")
    link = [nvcc, *ARCH_FLAGS, "-shared", "-o", str(tmp), *map(str, objs), "-lcudart_static", "-ldl", "-lrt", "-lpthread"]
    r = subprocess.run(link, stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True)
    if r.returncode != 0:
        raise RuntimeError("link failed:\n" + r.stdout)
    os.replace(tmp, LIB_PATH)
    if verbose:
        print("\n".join(logs))
    return LIB_PATH


if __name__ == "__main__":
    path = build(force="--force" in sys.argv, verbose="-v" in sys.argv)
    print(path)
