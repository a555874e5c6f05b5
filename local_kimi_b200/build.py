"""Build recipe for the in-tree CUDA library ``libkimi_b200.so``.

Compiles every ``csrc/*.cu`` for sm_100a with nvcc into one shared library
next to this file.  The library exports the C ABI declared in
``include/kimi_b200.h``; nothing here links torch.  Run as
``python -m local_kimi_b200.build`` or call :func:`build`.
"""

from __future__ import annotations

import fcntl
import os
import shutil
import subprocess
import sys
from pathlib import Path

PACKAGE_DIR = Path(__file__).resolve().parent
REPO_DIR = PACKAGE_DIR.parent
CSRC = PACKAGE_DIR / "csrc"
LIB_NAME = "libkimi_b200.so"
LIB_PATH = PACKAGE_DIR / LIB_NAME
BUILD_DIR = REPO_DIR / "_build"

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = [
    "-O3",
    "-lineinfo",
    "-std=c++17",
    "--expt-relaxed-constexpr",
    "-Xcompiler",
    "-fPIC",
    "-Xcompiler",
    "-fvisibility=hidden",
]


def _nvcc() -> str:
    for candidate in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if candidate and Path(candidate).exists():
            return candidate
    raise RuntimeError("nvcc not found; set NVCC or add the CUDA toolkit to PATH")


def sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu"))


def _stale(target: Path, inputs: list[Path]) -> bool:
    if not target.exists():
        return True
    mtime = target.stat().st_mtime
    return any(path.stat().st_mtime > mtime for path in inputs)


def build(verbose: bool = False, force: bool = False, ptxas_verbose: bool = False) -> Path:
    """Compile the library if any source or header is newer than it.

    Safe to call from several processes at once (the ranks of a torchrun
    launch each call it): the build runs under an exclusive lock on a file in
    the build directory, and the staleness check is repeated once the lock is
    held, so one process compiles and the others find the library current.
    """
    headers = sorted(CSRC.glob("*.cuh")) + sorted((REPO_DIR / "include").glob("*.h"))
    srcs = sources()
    if not force and not _stale(LIB_PATH, srcs + headers):
        return LIB_PATH
    BUILD_DIR.mkdir(exist_ok=True)
    with open(BUILD_DIR / ".build.lock", "w") as lock:
        fcntl.flock(lock, fcntl.LOCK_EX)
        try:
            if not force and not _stale(LIB_PATH, srcs + headers):
                return LIB_PATH
            return _compile(srcs, headers, verbose, force, ptxas_verbose)
        finally:
            fcntl.flock(lock, fcntl.LOCK_UN)


def _compile(srcs: list[Path], headers: list[Path], verbose: bool, force: bool,
             ptxas_verbose: bool) -> Path:
    nvcc = _nvcc()
    objects = []
    for src in srcs:
        obj = BUILD_DIR / (src.stem + ".o")
        objects.append(obj)
        if not force and not _stale(obj, [src] + headers):
            continue
        cmd = [nvcc, *ARCH_FLAGS, *NVCC_FLAGS, "-I", str(REPO_DIR / "include"), "-c", str(src),
               "-o", str(obj)]
        if ptxas_verbose:
            cmd.insert(1, "-Xptxas=-v")
        if verbose:
            print(" ".join(cmd), file=sys.stderr)
        subprocess.run(cmd, check=True)
    tmp = LIB_PATH.with_suffix(f".so.tmp{os.getpid()}")
    cmd = [nvcc, *ARCH_FLAGS, "-shared", "-cudart", "static", "-o", str(tmp), *map(str, objects)]
    if verbose:
        print(" ".join(cmd), file=sys.stderr)
    subprocess.run(cmd, check=True)
    os.replace(tmp, LIB_PATH)
    return LIB_PATH


if __name__ == "__main__":
    force = "--force" in sys.argv
    path = build(verbose=True, force=force, ptxas_verbose="--ptxas" in sys.argv)
    print(path)
