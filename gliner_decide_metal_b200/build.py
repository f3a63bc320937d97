"""Build recipe for the C-ABI library ``libgdc.so`` (sm_100a).

Compiles every ``csrc`` translation unit with nvcc for ``-gencode
arch=compute_100a,code=sm_100a`` (objects under ``_build/``) and links the shared
library in-tree next to this file, so it travels with the repository to the GPU host.
Usage: ``python gliner_decide_metal_b200/build.py [--force] [-j N]`` (a plain script: it does
not import the package, whose import loads the library this script builds).
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
BUILD = ROOT / "_build"
LIB = PKG / "libgdc.so"
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-std=c++17", "-lineinfo", "--expt-relaxed-constexpr", "-Xcompiler", "-fPIC,-O3,-Wall",
              "-Xptxas", "-O3", f"-I{ROOT / 'include'}", f"-I{CSRC}"]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found")


def sources():
    return sorted([p for p in CSRC.rglob("*.cu")] + [p for p in CSRC.rglob("*.cpp")])


def headers():
    return sorted(list(CSRC.rglob("*.h")) + list(CSRC.rglob("*.cuh")) + list((ROOT / "include").glob("*.h")))


def _compile(src: Path, force: bool, extra):
    obj = BUILD / (src.relative_to(CSRC).as_posix().replace("/", "__") + ".o")
    newest_dep = max([src.stat().st_mtime] + [h.stat().st_mtime for h in headers()])
    if not force and obj.exists() and obj.stat().st_mtime >= newest_dep:
        return obj, None
    cmd = [nvcc(), *ARCH, *NVCC_FLAGS, *extra, "-c", str(src), "-o", str(obj)]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        obj.unlink(missing_ok=True)
        return obj, f"ERROR $ {' '.join(cmd)}\n{r.stdout}\n{r.stderr}"
    return obj, (r.stderr if ("warning" in r.stderr.lower() or extra) else None)


def build(force: bool = False, jobs: int | None = None, verbose_ptxas: bool = False) -> Path:
    BUILD.mkdir(exist_ok=True)
    extra = ["-Xptxas", "-v"] if verbose_ptxas else []
    srcs = sources()
    objs = []
    errors = []
    with cf.ThreadPoolExecutor(max_workers=jobs or min(8, os.cpu_count() or 4)) as ex:
        for obj, msg in ex.map(lambda s: _compile(s, force, extra), srcs):
            objs.append(obj)
            if msg:
                if msg.startswith("ERROR"):
                    errors.append(msg)
                else:
                    print(msg, file=sys.stderr)
    if errors:
        raise RuntimeError("nvcc failed:\n" + "\n".join(errors))
    newest = max(o.stat().st_mtime for o in objs)
    if force or not LIB.exists() or LIB.stat().st_mtime < newest:
        cmd = [nvcc(), *ARCH, "-shared", "-o", str(LIB), *map(str, objs), "-lpthread", "-ldl", "-lrt"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n$ {' '.join(cmd)}\n{r.stdout}\n{r.stderr}")
    return LIB


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("-j", type=int, default=None)
    ap.add_argument("--ptxas-v", action="store_true")
    a = ap.parse_args()
    print(build(a.force, a.j, a.ptxas_v))
