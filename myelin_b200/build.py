"""Build the myelin_b200 C-ABI library (``libmyelin_b200.so``) for sm_100a.

Every ``csrc/*.cu`` file is compiled by nvcc in parallel and linked into one
shared library inside the package directory, so that the built file travels
with the source tree. Rebuilds are incremental (by modification time).

Usage: ``python -m myelin_b200.build [--force] [--verbose]``.
"""

from __future__ import annotations

import argparse
import concurrent.futures
import os
import shutil
import subprocess
import sys
from pathlib import Path

PACKAGE_DIR = Path(__file__).resolve().parent
CSRC_DIR = PACKAGE_DIR / "csrc"
BUILD_DIR = PACKAGE_DIR / "_build"
LIB_DIR = PACKAGE_DIR / "_lib"
LIB_PATH = LIB_DIR / "libmyelin_b200.so"
INCLUDE_DIR = PACKAGE_DIR.parent / "include"

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = [
    "-O3",
    "-std=c++17",
    "-lineinfo",
    "--expt-relaxed-constexpr",
    "-Xcompiler",
    "-fPIC",
    "-Xptxas",
    "-warn-spills",
]


def nvcc_path() -> str:
    for candidate in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if candidate and Path(candidate).exists():
            return candidate
    raise RuntimeError("nvcc not found: the CUDA toolkit is required to build myelin_b200")


def _sources() -> list[Path]:
    return sorted(CSRC_DIR.glob("*.cu"))


def _headers() -> list[Path]:
    return sorted(CSRC_DIR.glob("*.cuh")) + sorted(INCLUDE_DIR.glob("*.h"))


def _compile(nvcc: str, src: Path, obj: Path, verbose: bool) -> str:
    cmd = [nvcc, *ARCH_FLAGS, *NVCC_FLAGS, "-c", str(src), "-o", str(obj)]
    if verbose:
        cmd += ["-Xptxas", "-v"]
    proc = subprocess.run(cmd, capture_output=True, text=True)
    if proc.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src.name}:\n{proc.stdout}\n{proc.stderr}")
    return proc.stdout + proc.stderr


def build(force: bool = False, verbose: bool = False) -> Path:
    """Compile and link the library; return its path."""

    nvcc = nvcc_path()
    BUILD_DIR.mkdir(exist_ok=True)
    LIB_DIR.mkdir(exist_ok=True)
    newest_header = max((h.stat().st_mtime for h in _headers()), default=0.0)
    jobs: list[tuple[Path, Path]] = []
    objects: list[Path] = []
    for src in _sources():
        obj = BUILD_DIR / (src.stem + ".o")
        objects.append(obj)
        stale = (
            force
            or not obj.exists()
            or obj.stat().st_mtime < max(src.stat().st_mtime, newest_header)
        )
        if stale:
            jobs.append((src, obj))
    if jobs:
        workers = min(len(jobs), os.cpu_count() or 4)
        with concurrent.futures.ThreadPoolExecutor(max_workers=workers) as pool:
            futures = {pool.submit(_compile, nvcc, s, o, verbose): s for s, o in jobs}
            for fut in concurrent.futures.as_completed(futures):
                log = fut.result()
                if verbose and log:
                    sys.stderr.write(f"--- {futures[fut].name}\n{log}")
    lib_stale = (
        force
        or bool(jobs)
        or not LIB_PATH.exists()
        or LIB_PATH.stat().st_mtime < max(o.stat().st_mtime for o in objects)
    )
    if lib_stale:
        tmp = LIB_PATH.with_suffix(".so.tmp")
        cmd = [nvcc, *ARCH_FLAGS, "-shared", "-o", str(tmp), *map(str, objects)]
        proc = subprocess.run(cmd, capture_output=True, text=True)
        if proc.returncode != 0:
            raise RuntimeError(f"link failed:\n{proc.stdout}\n{proc.stderr}")
        tmp.replace(LIB_PATH)
    return LIB_PATH


def main() -> None:
    parser = argparse.ArgumentParser(description=__doc__)
    parser.add_argument("--force", action="store_true")
    parser.add_argument("--verbose", action="store_true", help="print ptxas resource usage")
    args = parser.parse_args()
    path = build(force=args.force, verbose=args.verbose)
    print(path)


if __name__ == "__main__":
    main()
