"""Builds libgorgon_b200.so in-tree with nvcc for sm_100a.

Sources live in ``csrc/``; objects go to ``_build/`` and the shared library to
``lib/``.  A source is recompiled when it, a header under ``csrc/`` or the
public header is newer than its object.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

PKG = Path(__file__).resolve().parent
CSRC = PKG / "csrc"
BUILD = PKG / "_build"
LIBDIR = PKG / "lib"
LIB = LIBDIR / "libgorgon_b200.so"
INCLUDE = PKG.parent / "include"

SOURCES = ["abi.cu", "tree_mask.cu", "attn_api.cu", "attn_simt.cu", "attn_tc.cu", "attn_pair.cu",
           "verify.cu", "kv_trim.cu", "cand_tree.cu"]

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-std=c++17", "-lineinfo", "--expt-relaxed-constexpr",
              "-Xcompiler", "-fPIC,-O3,-fvisibility=hidden", "-I", str(INCLUDE)]


def nvcc_path() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found: set NVCC or put the CUDA toolkit on PATH")


def _headers_mtime() -> float:
    hs = list(CSRC.glob("*.cuh")) + list(INCLUDE.glob("*.h"))
    return max((h.stat().st_mtime for h in hs), default=0.0)


def _compile(nvcc: str, src: Path, obj: Path, verbose: bool, ptxas_v: bool) -> str:
    cmd = [nvcc, *ARCH, *NVCC_FLAGS, "-c", str(src), "-o", str(obj)]
    if ptxas_v:
        cmd[1:1] = ["-Xptxas", "-v"]
    if verbose:
        print(" ".join(cmd), flush=True)
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed on {src.name}:\n{res.stdout}\n{res.stderr}")
    return res.stderr


def build(force: bool = False, verbose: bool = False, ptxas_v: bool = False, jobs: int | None = None) -> Path:
    """Compile every CUDA source and link the shared library; returns its path."""
    nvcc = nvcc_path()
    BUILD.mkdir(exist_ok=True)
    LIBDIR.mkdir(exist_ok=True)
    hdr = _headers_mtime()
    todo = []
    for name in SOURCES:
        src = CSRC / name
        obj = BUILD / (name[:-3] + ".o")
        if force or ptxas_v or not obj.exists() or obj.stat().st_mtime < max(src.stat().st_mtime, hdr):
            todo.append((src, obj))
    logs = []
    if todo:
        with ThreadPoolExecutor(max_workers=jobs or min(len(todo), os.cpu_count() or 4)) as ex:
            futs = [ex.submit(_compile, nvcc, s, o, verbose, ptxas_v) for s, o in todo]
            for f in futs:
                logs.append(f.result())
    objs = [str(BUILD / (n[:-3] + ".o")) for n in SOURCES]
    if todo or force or not LIB.exists():
        tmp = LIB.with_suffix(".so.tmp")
        cmd = [nvcc, *ARCH, "-shared", "--cudart", "static", "-o", str(tmp), *objs]
        if verbose:
            print(" ".join(cmd), flush=True)
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            raise RuntimeError(f"link failed:\n{res.stdout}\n{res.stderr}")
        os.replace(tmp, LIB)
    if ptxas_v:
        for log in logs:
            sys.stdout.write(log)
    return LIB


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose=True, ptxas_v="--ptxas-v" in sys.argv)
    print(LIB)
