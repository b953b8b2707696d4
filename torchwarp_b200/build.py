"""Ahead-of-time build of libtorchwarp_b200.so for sm_100a (no JIT, no torch headers).

    python -m torchwarp_b200.build          # build (incremental)
    python -m torchwarp_b200.build --force  # rebuild everything

Each ``csrc/*.cu`` is compiled to an object with
``nvcc -gencode arch=compute_100a,code=sm_100a -O3 -lineinfo`` and the
objects are linked into ``torchwarp_b200/_lib/libtorchwarp_b200.so``.  The
library depends only on the CUDA runtime.
"""

import argparse
import os
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

PKG = Path(__file__).resolve().parent
CSRC = PKG / "csrc"
OUT_DIR = PKG / "_lib"
LIB = OUT_DIR / "libtorchwarp_b200.so"
OBJ_DIR = PKG.parent / "_build" / "obj"
ROOT = PKG.parent

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr",
         "-Xptxas", "-warn-spills"]


def nvcc():
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found (set NVCC)")


def _headers():
    return sorted(CSRC.glob("*.cuh")) + sorted((ROOT / "include").glob("*.h"))


def _compile(src, force):
    obj = OBJ_DIR / (src.stem + ".o")
    newest_dep = max([src.stat().st_mtime] + [h.stat().st_mtime for h in _headers()])
    if not force and obj.exists() and obj.stat().st_mtime >= newest_dep:
        return obj, None
    cmd = [nvcc(), *ARCH, *FLAGS, "-I", str(ROOT / "include"), "-c", str(src), "-o", str(obj)]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        return obj, "{}\n{}{}".format(" ".join(cmd), r.stdout, r.stderr)
    return obj, None


def build(force=False, verbose=False):
    OBJ_DIR.mkdir(parents=True, exist_ok=True)
    OUT_DIR.mkdir(parents=True, exist_ok=True)
    sources = sorted(CSRC.glob("*.cu"))
    with ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 1)) as ex:
        results = list(ex.map(lambda s: _compile(s, force), sources))
    errors = [e for _, e in results if e]
    if errors:
        raise RuntimeError("nvcc failed:\n" + "\n".join(errors))
    objs = [o for o, _ in results]
    if force or not LIB.exists() or any(o.stat().st_mtime > LIB.stat().st_mtime for o in objs):
        # --no-undefined: a symbol missing from every object fails the build
        # here, not the first dlopen on a GPU box
        cmd = [nvcc(), *ARCH, "-shared", "-o", str(LIB), *map(str, objs), "-lcudart",
               "-Xlinker", "--no-undefined"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError("link failed:\n{}{}".format(r.stdout, r.stderr))
    if verbose:
        print("built", LIB)
    return LIB


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    args = ap.parse_args()
    try:
        build(force=args.force, verbose=True)
    except RuntimeError as e:
        print(e, file=sys.stderr)
        sys.exit(1)
