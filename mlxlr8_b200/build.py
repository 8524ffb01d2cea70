"""Build the in-tree CUDA library ``libexlr8_b200.so`` for sm_100a.

    python -m mlxlr8_b200.build          # incremental
    python -m mlxlr8_b200.build --force  # rebuild everything

Each ``csrc/*.cu`` compiles to an object under ``_build/`` (in parallel); the
objects link into ``mlxlr8_b200/libexlr8_b200.so``.  nvcc cross-compiles, so
this works on a machine without a GPU.
"""

from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

PACKAGE = Path(__file__).resolve().parent
ROOT = PACKAGE.parent
CSRC = PACKAGE / "csrc"
INCLUDE = ROOT / "include"
BUILD = ROOT / "_build"
LIBRARY = PACKAGE / "libexlr8_b200.so"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr",
         "-Xptxas", "-warn-spills"]


def nvcc() -> str:
    for candidate in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if candidate and Path(candidate).exists():
            return candidate
    raise RuntimeError("nvcc not found: the CUDA toolkit is required to build libexlr8_b200.so")


def _sources():
    return sorted(CSRC.glob("*.cu"))


def _headers():
    return sorted(list(CSRC.glob("*.cuh")) + list(INCLUDE.glob("*.h")))


def _stale(target: Path, deps) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(d.stat().st_mtime > t for d in deps)


def _compile(src: Path, verbose: bool) -> Path:
    obj = BUILD / (src.stem + ".o")
    cmd = [nvcc(), *ARCH, *FLAGS, "-I", str(INCLUDE), "-c", str(src), "-o", str(obj)]
    if verbose:
        print(" ".join(cmd), flush=True)
    result = subprocess.run(cmd, capture_output=True, text=True)
    if result.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src.name}:\n{result.stdout}\n{result.stderr}")
    if result.stderr.strip() and verbose:
        print(result.stderr, file=sys.stderr)
    return obj


def build(force: bool = False, verbose: bool = False) -> Path:
    BUILD.mkdir(exist_ok=True)
    sources = _sources()
    headers = _headers()
    todo = [s for s in sources if force or _stale(BUILD / (s.stem + ".o"), [s, *headers])]
    if todo:
        with ThreadPoolExecutor(max_workers=min(len(todo), os.cpu_count() or 4)) as pool:
            list(pool.map(lambda s: _compile(s, verbose), todo))
    objects = [BUILD / (s.stem + ".o") for s in sources]
    if force or todo or _stale(LIBRARY, objects):
        cmd = [nvcc(), *ARCH, "-shared", "-o", str(LIBRARY), *map(str, objects), "-lcudart"]
        if verbose:
            print(" ".join(cmd), flush=True)
        result = subprocess.run(cmd, capture_output=True, text=True)
        if result.returncode != 0:
            raise RuntimeError(f"link failed:\n{result.stdout}\n{result.stderr}")
    return LIBRARY


def main() -> None:
    parser = argparse.ArgumentParser(description=__doc__)
    parser.add_argument("--force", action="store_true")
    parser.add_argument("--verbose", action="store_true")
    args = parser.parse_args()
    print(build(force=args.force, verbose=args.verbose))


if __name__ == "__main__":
    main()
