"""Builds libplm_native.so (the sm_100a kernels and the C ABI) in-tree with nvcc.

    python plm-anon_b200/csrc/build.py [--force] [--verbose]

Every ``*.cu`` in this directory is compiled to an object under ``_build/`` and linked into
``plm-anon_b200/plm/libplm_native.so``. Translation units listed in ``EXACT_FP`` are compiled with ``-fmad=false``:
their floating-point steps must match the CPU oracle bit for bit, so no multiply-add may be contracted. Objects are
rebuilt only when a source or header is newer than them.
"""

from __future__ import annotations

import argparse
import os
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

CSRC = Path(__file__).resolve().parent
BUILD = CSRC / "_build"
LIBRARY = CSRC.parent / "plm" / "libplm_native.so"
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
COMMON = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr", "-I", str(CSRC)]
EXACT_FP = {"voronoi.cu"}


def _newest_header() -> float:
    headers = list(CSRC.glob("*.cuh")) + list(CSRC.glob("*.h")) + list((CSRC.parent.parent / "include").glob("*.h"))
    return max((h.stat().st_mtime for h in headers), default=0.0)


def _compile(source: Path, verbose: bool) -> tuple[Path, str]:
    obj = BUILD / (source.stem + ".o")
    flags = ARCH + COMMON + (["-fmad=false"] if source.name in EXACT_FP else [])
    if verbose:
        flags += ["-Xptxas", "-v"]
    cmd = [NVCC, *flags, "-c", str(source), "-o", str(obj)]
    result = subprocess.run(cmd, capture_output=True, text=True)
    if result.returncode != 0:
        raise RuntimeError(f"nvcc failed on {source.name}:\n{result.stdout}\n{result.stderr}")
    return obj, result.stderr


def build(force: bool = False, verbose: bool = False) -> Path:
    BUILD.mkdir(exist_ok=True)
    sources = sorted(CSRC.glob("*.cu"))
    header_time = _newest_header()
    stale = [s for s in sources
             if force or not (BUILD / (s.stem + ".o")).exists()
             or (BUILD / (s.stem + ".o")).stat().st_mtime < max(s.stat().st_mtime, header_time)]
    with ThreadPoolExecutor(max_workers=max(1, min(len(stale), os.cpu_count() or 4))) as pool:
        for obj, log in pool.map(lambda s: _compile(s, verbose), stale):
            if verbose and log:
                print(f"--- {obj.name}\n{log}", file=sys.stderr)
    objects = [BUILD / (s.stem + ".o") for s in sources]
    if force or stale or not LIBRARY.exists() or LIBRARY.stat().st_mtime < max(o.stat().st_mtime for o in objects):
        cmd = [NVCC, *ARCH, "-shared", "-o", str(LIBRARY), *map(str, objects)]
        result = subprocess.run(cmd, capture_output=True, text=True)
        if result.returncode != 0:
            raise RuntimeError(f"link failed:\n{result.stdout}\n{result.stderr}")
    return LIBRARY


if __name__ == "__main__":
    parser = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    parser.add_argument("--force", action="store_true")
    parser.add_argument("--verbose", action="store_true")
    args = parser.parse_args()
    print(build(args.force, args.verbose))
