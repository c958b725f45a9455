"""Build the native library ``arthip_b200/lib/libarthip_b200.so`` with nvcc (sm_100a).

Usage: ``python -m arthip_b200.build [--force]``. Every source is compiled with
``-gencode arch=compute_100a,code=sm_100a -lineinfo -O3``; objects are rebuilt when a
source or header is newer than the object. The library links the CUDA runtime
statically, so it loads next to PyTorch's own runtime without version coupling.
"""

from __future__ import annotations

import concurrent.futures as cf
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
CSRC = PKG / "csrc"
ROOT = PKG.parent
LIB_DIR = PKG / "lib"
OBJ_DIR = PKG / "_build"
LIB_NAME = "libarthip_b200.so"
LIB_PATH = LIB_DIR / LIB_NAME

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
COMMON = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC,-O3,-Wall", "-I", str(CSRC),
          "-I", str(ROOT / "include"), "--expt-relaxed-constexpr", "-diag-suppress", "177"]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found (set NVCC or put the CUDA toolkit on PATH)")


def sources() -> list[Path]:
    return sorted(list(CSRC.glob("*.cc")) + list(CSRC.glob("kernels/*.cu")))


def headers() -> list[Path]:
    return sorted(list(CSRC.rglob("*.h")) + list(CSRC.rglob("*.cuh")) + list((ROOT / "include").glob("*.h")))


def _compile(src: Path, force: bool) -> Path:
    obj = OBJ_DIR / (src.relative_to(CSRC).as_posix().replace("/", "__") + ".o")
    newest_dep = max([src.stat().st_mtime] + [h.stat().st_mtime for h in headers()])
    if not force and obj.exists() and obj.stat().st_mtime >= newest_dep:
        return obj
    cmd = [nvcc(), *ARCH, *COMMON, "-c", str(src), "-o", str(obj)]
    if src.suffix == ".cc":
        cmd[1:1] = ["-x", "cu"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src.name}:\n{r.stdout}\n{r.stderr}")
    return obj


def build(force: bool = False, verbose: bool = True) -> Path:
    OBJ_DIR.mkdir(parents=True, exist_ok=True)
    LIB_DIR.mkdir(parents=True, exist_ok=True)
    srcs = sources()
    with cf.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 4)) as ex:
        objs = list(ex.map(lambda s: _compile(s, force), srcs))
    if not force and LIB_PATH.exists() and LIB_PATH.stat().st_mtime >= max(o.stat().st_mtime for o in objs):
        return LIB_PATH
    cmd = [nvcc(), *ARCH, "-shared", "-o", str(LIB_PATH), *map(str, objs), "-cudart", "static"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    if verbose:
        print(f"[arthip_b200] built {LIB_PATH}")
    return LIB_PATH


if __name__ == "__main__":
    build(force="--force" in sys.argv)
