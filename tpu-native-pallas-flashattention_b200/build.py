"""Builds libpallas_flash_b200.so (sm_100a) in-tree with nvcc.

    python tpu-native-pallas-flashattention_b200/build.py [--force] [--jobs N]

The library is the product's native code; the Python package loads it from
``pallas_flash/libpallas_flash_b200.so``.  Sources are compiled as separate
relocatable objects in parallel and device-linked into one shared library.
"""

from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG_ROOT = Path(__file__).resolve().parent
CSRC = PKG_ROOT / "csrc"
OUT_DIR = PKG_ROOT / "pallas_flash"
LIB_NAME = "libpallas_flash_b200.so"
BUILD_DIR = PKG_ROOT / "_build"
INCLUDE = PKG_ROOT.parent / "include"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = [
    "-O3", "-std=c++17", "-lineinfo", "-rdc=true", "-Xcompiler", "-fPIC",
    "--expt-relaxed-constexpr",
    "-Xptxas", "-warn-spills",
]


def nvcc() -> str:
    cand = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(cand).exists():
        raise RuntimeError("nvcc not found; the CUDA toolkit is required to build pallas_flash")
    return cand


def sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu"))


def _deps() -> list[Path]:
    return sources() + sorted(CSRC.glob("*.cuh")) + sorted(CSRC.glob("*.h")) + sorted(INCLUDE.glob("*.h"))


def lib_path() -> Path:
    return OUT_DIR / LIB_NAME


def up_to_date() -> bool:
    lib = lib_path()
    if not lib.exists():
        return False
    t = lib.stat().st_mtime
    return all(p.stat().st_mtime <= t for p in _deps())


def _compile(src: Path, verbose: bool) -> Path:
    obj = BUILD_DIR / (src.stem + ".o")
    cmd = [nvcc(), *ARCH, *NVCC_FLAGS, "-I", str(INCLUDE), "-c", str(src), "-o", str(obj)]
    if verbose:
        cmd += ["-Xptxas", "-v"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed on {src.name}:\n{r.stdout}\n{r.stderr}")
    if verbose and (r.stdout or r.stderr):
        sys.stderr.write(r.stderr + r.stdout)
    return obj


def build(force: bool = False, jobs: int | None = None, verbose: bool = False) -> Path:
    """Compiles every CUDA source for sm_100a and links the shared library."""
    if not force and up_to_date():
        return lib_path()
    BUILD_DIR.mkdir(exist_ok=True)
    srcs = sources()
    jobs = jobs or min(len(srcs), os.cpu_count() or 1)
    with cf.ThreadPoolExecutor(max_workers=jobs) as ex:
        objs = list(ex.map(lambda s: _compile(s, verbose), srcs))
    tmp = lib_path().with_suffix(".so.tmp")
    cmd = [nvcc(), *ARCH, "-rdc=true", "-shared", "-Xcompiler", "-fPIC", *map(str, objs),
           "-o", str(tmp), "-lcudart"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    os.replace(tmp, lib_path())
    return lib_path()


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--jobs", type=int, default=None)
    ap.add_argument("--verbose", action="store_true", help="print ptxas resource usage")
    args = ap.parse_args()
    print(build(force=args.force, jobs=args.jobs, verbose=args.verbose))


if __name__ == "__main__":
    main()
