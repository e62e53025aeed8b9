"""Build ``libnsm.so`` (the C-ABI library) in-tree with nvcc for sm_100a.

The library is a plain shared object with an ``extern "C"`` interface
(``include/nsm.h``); the Python package binds it with ctypes.  cudart is
linked statically so the library only needs the NVIDIA driver at run time.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
CSRC = PKG / "csrc"
LIB = PKG / "libnsm.so"
SOURCES = ["nsm_abi.cu", "nsm_router.cu", "nsm_decode.cu", "nsm_aux.cu", "nsm_static.cu", "nsm_union.cu", "nsm_exchange.cu",
           "nsm_lmhead.cu", "nsm_token.cu"]
GENCODE = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc_path() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found; the CUDA toolkit is required to build libnsm.so")


def _stale() -> bool:
    if not LIB.exists():
        return True
    mtime = LIB.stat().st_mtime
    deps = [CSRC / s for s in SOURCES] + list(CSRC.glob("*.cuh")) + list(CSRC.glob("*.h"))
    deps.append(PKG.parent / "include" / "nsm.h")
    return any(d.stat().st_mtime > mtime for d in deps if d.exists())


def build(force: bool = False, verbose: bool = False) -> Path:
    if not force and not _stale():
        return LIB
    nvcc = nvcc_path()
    objdir = PKG / "_build"
    objdir.mkdir(exist_ok=True)
    common = GENCODE + ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-Xcompiler", "-O3",
                        "-I", str(PKG.parent / "include")]
    objs = []
    cmds = []
    for src in SOURCES:
        obj = objdir / (Path(src).stem + ".o")
        cmds.append([nvcc, *common, "-c", str(CSRC / src), "-o", str(obj)])
        objs.append(str(obj))
    if verbose:
        for cmd in cmds:
            print(" ".join(cmd), file=sys.stderr)
    # the translation units are independent: compile them in parallel
    from concurrent.futures import ThreadPoolExecutor

    with ThreadPoolExecutor(max_workers=min(len(cmds), os.cpu_count() or 1)) as pool:
        for r in list(pool.map(lambda c: subprocess.run(c, capture_output=True, text=True), cmds)):
            if r.returncode != 0:
                raise RuntimeError(f"nvcc failed: {' '.join(r.args)}\n{r.stdout}{r.stderr}")
    tmp = LIB.with_suffix(".so.tmp")
    cmd = [nvcc, *GENCODE, "-shared", "-cudart", "static", "-o", str(tmp), *objs]
    if verbose:
        print(" ".join(cmd), file=sys.stderr)
    subprocess.run(cmd, check=True)
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose=True))
