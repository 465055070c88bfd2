"""Build libinl_cuda.so in-tree for sm_100a with nvcc.

    python im-not-llm_b200/build.py            # incremental
    python im-not-llm_b200/build.py --clean    # from scratch

Objects go to im-not-llm_b200/_build/, the library to
im-not-llm_b200/libinl_cuda.so (both git-ignored; the .so travels with the
repository snapshot to the GPU box).
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
BUILD = PKG / "_build"
LIB = PKG / "libinl_cuda.so"

NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-std=c++17", "-O3", "-lineinfo", "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
         "-diag-suppress", "177", f"-I{ROOT / 'include'}", f"-I{CSRC}"]


def _sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu"))


def _headers() -> list[Path]:
    return sorted(CSRC.glob("*.h")) + sorted(CSRC.glob("*.cuh")) + sorted((ROOT / "include").glob("*.h"))


def _compile(src: Path) -> tuple[Path, str]:
    obj = BUILD / (src.stem + ".o")
    cmd = [NVCC, *ARCH, *FLAGS, "-c", str(src), "-o", str(obj)]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src.name}:\n{r.stderr}")
    return obj, r.stderr


def build(clean: bool = False, verbose: bool = False) -> Path:
    if clean and BUILD.exists():
        shutil.rmtree(BUILD)
    BUILD.mkdir(exist_ok=True)
    srcs = _sources()
    newest_header = max((h.stat().st_mtime for h in _headers()), default=0.0)
    todo = []
    for s in srcs:
        obj = BUILD / (s.stem + ".o")
        if not obj.exists() or obj.stat().st_mtime < max(s.stat().st_mtime, newest_header):
            todo.append(s)
    if todo:
        with cf.ThreadPoolExecutor(max_workers=min(len(todo), os.cpu_count() or 4)) as ex:
            for obj, log in ex.map(_compile, todo):
                if verbose and log.strip():
                    print(log, file=sys.stderr)
    objs = [BUILD / (s.stem + ".o") for s in srcs]
    if todo or not LIB.exists() or LIB.stat().st_mtime < max(o.stat().st_mtime for o in objs):
        cmd = [NVCC, *ARCH, "-shared", "-cudart", "static", "-o", str(LIB), *map(str, objs)]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stderr}")
    return LIB


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--clean", action="store_true")
    ap.add_argument("-v", "--verbose", action="store_true")
    a = ap.parse_args()
    print(build(clean=a.clean, verbose=a.verbose))
