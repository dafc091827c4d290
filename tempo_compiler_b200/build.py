"""Builds libtempo_b200.so in-tree from csrc/*.cu for sm_100a.

Each translation unit compiles in parallel (``nvcc -c``), then nvcc links the shared library with the static CUDA
runtime, so the library needs only the NVIDIA driver at run time. Rebuilds only when a source is newer than the
library.

    python -m tempo_compiler_b200.build [--force] [--verbose-ptxas]
"""

from __future__ import annotations

import argparse
import concurrent.futures
import fcntl
import os
import pathlib
import shutil
import subprocess
import sys

PACKAGE = pathlib.Path(__file__).resolve().parent
CSRC = PACKAGE / "csrc"
INCLUDE = PACKAGE.parent / "include"
LIBRARY = PACKAGE / "libtempo_b200.so"
BUILD = PACKAGE / "_build"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "-Xcompiler", "-O2", "-I", str(INCLUDE)]


def nvcc() -> str:
    found = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not pathlib.Path(found).exists():
        raise RuntimeError("nvcc not found: the B200 kernels cannot be built without the CUDA toolkit")
    return found


def sources() -> list[pathlib.Path]:
    return sorted(CSRC.glob("*.cu"))


def _stale() -> bool:
    if not LIBRARY.exists():
        return True
    built = LIBRARY.stat().st_mtime
    deps = sources() + sorted(CSRC.glob("*.cuh")) + sorted(CSRC.glob("*.hpp")) + sorted(INCLUDE.glob("*.h"))
    return any(path.stat().st_mtime > built for path in deps)


def _compile(source: pathlib.Path, verbose_ptxas: bool) -> tuple[pathlib.Path, str]:
    obj = BUILD / (source.stem + ".o")
    cmd = [nvcc(), *ARCH, *FLAGS, "-c", str(source), "-o", str(obj)]
    if verbose_ptxas:
        cmd += ["-Xptxas", "-v"]
    result = subprocess.run(cmd, capture_output=True, text=True)
    if result.returncode != 0:
        raise RuntimeError(f"nvcc failed on {source.name}:\n{result.stdout}\n{result.stderr}")
    return obj, result.stderr


def build(force: bool = False, verbose_ptxas: bool = False) -> pathlib.Path:
    """Compiles the library if it is missing or stale and returns its path."""
    if not force and not verbose_ptxas and not _stale():
        return LIBRARY
    BUILD.mkdir(exist_ok=True)
    # Several processes (one per GPU) may find the library stale at once: one builds, the others wait for it and
    # then find it fresh. The lock also keeps them from writing the same object files.
    with open(BUILD / ".lock", "w") as lock:
        fcntl.flock(lock, fcntl.LOCK_EX)
        if not force and not verbose_ptxas and not _stale():
            return LIBRARY
        return _build_locked(verbose_ptxas)


def _build_locked(verbose_ptxas: bool) -> pathlib.Path:
    workers = min(len(sources()), os.cpu_count() or 4)
    with concurrent.futures.ThreadPoolExecutor(max_workers=workers) as pool:
        results = list(pool.map(lambda s: _compile(s, verbose_ptxas), sources()))
    if verbose_ptxas:
        for _, log in results:
            sys.stderr.write(log)
    tmp = LIBRARY.with_suffix(f".so.{os.getpid()}.tmp")
    cmd = [nvcc(), *ARCH, "-shared", "-o", str(tmp), *[str(obj) for obj, _ in results]]
    result = subprocess.run(cmd, capture_output=True, text=True)
    if result.returncode != 0:
        raise RuntimeError(f"nvcc link failed:\n{result.stdout}\n{result.stderr}")
    os.replace(tmp, LIBRARY)
    return LIBRARY


def main() -> int:
    parser = argparse.ArgumentParser(description=__doc__)
    parser.add_argument("--force", action="store_true")
    parser.add_argument("--verbose-ptxas", action="store_true")
    args = parser.parse_args()
    print(build(force=args.force, verbose_ptxas=args.verbose_ptxas))
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
