"""Build ``libboltz_b200.so`` in-tree with nvcc for sm_100a.

Usage: ``python -m boltz_lumi_b200.build [--force] [--jobs N]``.

The library is the C-ABI of ``include/boltz_b200.h``; it is built next to
this file so that it travels with the source tree.  Replaces the reference's
lazy ``torch.utils.cpp_extension.load`` of HIP sources (kernels/_build.py:9-34).
"""

import argparse
import concurrent.futures
import os
import shutil
import subprocess
import sys
from pathlib import Path

PACKAGE = Path(__file__).resolve().parent
ROOT = PACKAGE.parent
CSRC = PACKAGE / "csrc"
INCLUDE = ROOT / "include"
BUILD = PACKAGE / "_build"
LIBRARY = PACKAGE / "libboltz_b200.so"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = [
    "-O3",
    "-lineinfo",
    "-std=c++17",
    "--expt-relaxed-constexpr",
    "-Xcompiler",
    "-fPIC",
    "-Xcompiler",
    "-fvisibility=hidden",
    "-DBL_BUILDING_LIBRARY",
]


def nvcc() -> str:
    path = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(path).exists():
        raise RuntimeError("nvcc not found; the CUDA 12.9 toolkit is required to build libboltz_b200.so")
    return path


def sources():
    return sorted(CSRC.glob("*.cu"))


def headers():
    return sorted(CSRC.glob("*.cuh")) + sorted(INCLUDE.glob("*.h"))


def _stale(target: Path, deps) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(d.stat().st_mtime > t for d in deps)


def _compile(src: Path, force: bool, verbose: bool) -> Path:
    obj = BUILD / (src.stem + ".o")
    if force or _stale(obj, [src, *headers()]):
        cmd = [nvcc(), *ARCH, *FLAGS, f"-I{INCLUDE}", f"-I{CSRC}", "-c", str(src), "-o", str(obj)]
        if verbose:
            cmd.insert(1, "-Xptxas=-v")
        result = subprocess.run(cmd, capture_output=True, text=True)
        if result.returncode != 0:
            raise RuntimeError(f"nvcc failed for {src.name}:\n{result.stdout}\n{result.stderr}")
        if verbose:
            sys.stderr.write(result.stderr)
    return obj


def build(force: bool = False, jobs: int = 0, verbose: bool = False) -> Path:
    """Compile every ``csrc/*.cu`` and link the shared library; returns its path."""
    BUILD.mkdir(exist_ok=True)
    srcs = sources()
    jobs = jobs or min(len(srcs), os.cpu_count() or 1)
    with concurrent.futures.ThreadPoolExecutor(max_workers=jobs) as pool:
        objs = list(pool.map(lambda s: _compile(s, force, verbose), srcs))
    if force or _stale(LIBRARY, objs):
        tmp = LIBRARY.with_suffix(".so.tmp")
        cmd = [nvcc(), *ARCH, "-shared", "-o", str(tmp), *map(str, objs)]
        result = subprocess.run(cmd, capture_output=True, text=True)
        if result.returncode != 0:
            raise RuntimeError(f"link failed:\n{result.stdout}\n{result.stderr}")
        os.replace(tmp, LIBRARY)
    return LIBRARY


def main():
    parser = argparse.ArgumentParser(description=__doc__)
    parser.add_argument("--force", action="store_true")
    parser.add_argument("--jobs", type=int, default=0)
    parser.add_argument("--verbose", action="store_true", help="print ptxas register/spill reports")
    args = parser.parse_args()
    print(build(args.force, args.jobs, args.verbose))


if __name__ == "__main__":
    main()
