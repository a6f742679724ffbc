"""Build libace_b200.so in-tree with nvcc for sm_100a.

    python -m ace_kernels_b200.build [--force] [--debug]

Each translation unit under ``csrc/`` is compiled in parallel to an object file
under ``_build/``, then linked (CUDA runtime linked statically) into
``ace_kernels_b200/libace_b200.so``. No fast-math: the probability and bin-index
path relies on IEEE division and CUDA's accurate ``expf``.
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
CSRC = PKG / "csrc"
INCLUDE = PKG.parent / "include"
BUILD = PKG / "_build"
LIB = PKG / "libace_b200.so"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = [
    "-O3",
    "-std=c++17",
    "-lineinfo",
    "-Xcompiler",
    "-fPIC",
    "-Xptxas",
    "-v",
    f"-I{INCLUDE}",
]


def nvcc() -> str:
    path = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(path).exists():
        raise RuntimeError("nvcc not found: the CUDA toolkit is required to build")
    return path


def _sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu"))


def _headers() -> list[Path]:
    return sorted([*CSRC.glob("*.cuh"), *CSRC.glob("*.h"), *INCLUDE.glob("*.h")])


def _stale(target: Path, deps: list[Path]) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(d.stat().st_mtime > t for d in deps)


def _compile(src: Path, debug: bool) -> tuple[Path, str]:
    obj = BUILD / (src.stem + ".o")
    flags = list(NVCC_FLAGS)
    if debug:
        flags += ["-DACE_DEBUG"]
    cmd = [nvcc(), *ARCH, *flags, "-c", str(src), "-o", str(obj)]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed on {src.name}:\n{res.stdout}\n{res.stderr}")
    return obj, res.stderr


def build(force: bool = False, debug: bool = False, verbose: bool = False) -> Path:
    """Compile (if stale) and return the path of libace_b200.so."""
    srcs = _sources()
    deps = srcs + _headers() + [Path(__file__)]
    if not force and not _stale(LIB, deps):
        return LIB
    BUILD.mkdir(exist_ok=True)
    jobs = max(1, min(len(srcs), os.cpu_count() or 1))
    with cf.ThreadPoolExecutor(jobs) as pool:
        results = list(pool.map(lambda s: _compile(s, debug), srcs))
    if verbose:
        for obj, log in results:
            print(f"== {obj.name}\n{log}", file=sys.stderr)
    objs = [str(o) for o, _ in results]
    tmp = LIB.with_suffix(".so.tmp")
    cmd = [nvcc(), *ARCH, "-shared", "-cudart", "static", "-o", str(tmp), *objs]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"link failed:\n{res.stdout}\n{res.stderr}")
    os.replace(tmp, LIB)
    return LIB


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--debug", action="store_true")
    ap.add_argument("-v", "--verbose", action="store_true")
    args = ap.parse_args()
    print(build(force=args.force, debug=args.debug, verbose=args.verbose))


if __name__ == "__main__":
    main()
