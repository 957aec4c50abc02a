"""Build recipe for libnqt.so, the sm_100a kernels behind include/nqt.h.

Every ``csrc/*.cu`` file is compiled with nvcc for ``sm_100a`` only and the
objects are linked into ``libnqt.so`` next to this file (in-tree, so the
library travels with the source tree).  Objects go to ``_build/``.
A rebuild happens only when a source or header is newer than the library.
"""

from __future__ import annotations

import concurrent.futures
import os
import shutil
import subprocess
from pathlib import Path

PKG_DIR = Path(__file__).resolve().parent
REPO_DIR = PKG_DIR.parent
CSRC = PKG_DIR / "csrc"
BUILD_DIR = PKG_DIR / "_build"
LIB_PATH = PKG_DIR / "libnqt.so"

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = [
    *ARCH_FLAGS,
    "-lineinfo",
    "-O3",
    "-std=c++17",
    "-Xcompiler",
    "-fPIC",
    "--expt-relaxed-constexpr",
    f"-I{REPO_DIR / 'include'}",
]


def _nvcc() -> str:
    for candidate in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if candidate and Path(candidate).exists():
            return candidate
    raise RuntimeError("nvcc not found: set NVCC or put the CUDA toolkit on PATH")


def sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu"))


def _inputs() -> list[Path]:
    return [*sources(), *CSRC.glob("*.cuh"), *(REPO_DIR / "include").glob("*.h")]


def up_to_date() -> bool:
    if not LIB_PATH.exists():
        return False
    lib_time = LIB_PATH.stat().st_mtime
    return all(p.stat().st_mtime <= lib_time for p in _inputs())


def build(*, force: bool = False, verbose: bool = False) -> Path:
    """Compile all kernels and link libnqt.so; returns the library path."""

    if not force and up_to_date():
        return LIB_PATH
    nvcc = _nvcc()
    BUILD_DIR.mkdir(exist_ok=True)

    def compile_one(src: Path) -> Path:
        obj = BUILD_DIR / (src.stem + ".o")
        cmd = [nvcc, *NVCC_FLAGS, "-c", str(src), "-o", str(obj)]
        if verbose:
            cmd.insert(1, "-Xptxas=-v")
        proc = subprocess.run(cmd, capture_output=True, text=True)
        if proc.returncode != 0:
            raise RuntimeError(f"nvcc failed for {src.name}:\n{proc.stderr}")
        if verbose and proc.stderr:
            print(proc.stderr)
        return obj

    with concurrent.futures.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 1)) as pool:
        objects = list(pool.map(compile_one, sources()))
    tmp = LIB_PATH.with_suffix(".so.tmp")
    cmd = [nvcc, *ARCH_FLAGS, "-shared", "-o", str(tmp), *map(str, objects)]
    proc = subprocess.run(cmd, capture_output=True, text=True)
    if proc.returncode != 0:
        raise RuntimeError(f"link of libnqt.so failed:\n{proc.stderr}")
    os.replace(tmp, LIB_PATH)
    return LIB_PATH


if __name__ == "__main__":
    import sys

    print(build(force="--force" in sys.argv, verbose="-v" in sys.argv))
