"""Build the engine's shared library, drift_b200/libdrift_b200.so, for sm_100a.

    python -m drift_b200.build [-v]

Each .cu under csrc/ compiles to an object in csrc/_build/ (in parallel),
then nvcc links them into one self-contained .so (static cudart). The build is
skipped when the library is newer than every source. -fmad=false keeps every
multiply and add a separate rounding, as the JVM computes them.
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
BUILD = CSRC / "_build"
LIB = PKG / "libdrift_b200.so"
INCLUDE = PKG.parent / "include"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-fmad=false", "-Xcompiler", "-fPIC",
         "-Xcompiler", "-fvisibility=hidden", "--expt-relaxed-constexpr"]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found; the engine needs the CUDA toolkit to build")


def sources():
    return sorted(CSRC.glob("*.cu"))


def headers():
    return sorted(list(CSRC.glob("*.cuh")) + list(CSRC.glob("*.h")) + list(INCLUDE.glob("*.h")))


def up_to_date() -> bool:
    if not LIB.exists():
        return False
    t = LIB.stat().st_mtime
    return all(p.stat().st_mtime <= t for p in sources() + headers() + [Path(__file__)])


def build(verbose: bool = False, force: bool = False, extra_flags=()) -> Path:
    if not force and up_to_date():
        return LIB
    BUILD.mkdir(exist_ok=True)
    cc = nvcc()
    objs = []

    def compile_one(src: Path) -> Path:
        obj = BUILD / (src.stem + ".o")
        cmd = [cc, *ARCH, *FLAGS, *extra_flags, "-I", str(INCLUDE), "-c", str(src), "-o", str(obj)]
        if verbose:
            print(" ".join(cmd), flush=True)
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            raise RuntimeError(f"nvcc failed on {src.name}:\n{res.stdout}\n{res.stderr}")
        if verbose and (res.stdout or res.stderr):
            print(res.stdout, res.stderr, flush=True)
        return obj

    with cf.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 2)) as ex:
        objs = list(ex.map(compile_one, sources()))
    tmp = LIB.with_suffix(".so.tmp")
    cmd = [cc, *ARCH, "-shared", "-o", str(tmp), *map(str, objs), "-cudart", "static"]
    if verbose:
        print(" ".join(cmd), flush=True)
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"link failed:\n{res.stdout}\n{res.stderr}")
    os.replace(tmp, LIB)
    return LIB


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("-v", "--verbose", action="store_true")
    ap.add_argument("-f", "--force", action="store_true")
    ap.add_argument("--ptxas-info", action="store_true", help="print registers/spills per kernel")
    args = ap.parse_args()
    extra = ["-Xptxas", "-v"] if args.ptxas_info else []
    build(verbose=args.verbose or args.ptxas_info, force=args.force or args.ptxas_info,
          extra_flags=extra)
    print(LIB)
    return 0


if __name__ == "__main__":
    sys.exit(main())
