"""Build the cachebridge_b200 native library (C ABI + sm_100a kernels).

Compiles every ``.cu`` file in this directory with nvcc for sm_100a into
``cachebridge_b200/libcachebridge_b200.so`` (in-tree, so it travels with the
repository snapshot). Usage: ``python -m cachebridge_b200.csrc.build [-v]``.
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
PACKAGE = HERE.parent
OUTPUT = PACKAGE / "libcachebridge_b200.so"
SOURCES = sorted(HERE.glob("*.cu"))
HEADERS = sorted(HERE.glob("*.cuh")) + [PACKAGE.parent / "include" / "cachebridge_b200.h"]

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
COMMON_FLAGS = [
    "-O3",
    "-lineinfo",
    "-std=c++17",
    "--expt-relaxed-constexpr",
    "-Xcompiler",
    "-fPIC",
    "-Xcompiler",
    "-fvisibility=hidden",
]


def nvcc_path() -> str:
    for candidate in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if candidate and Path(candidate).exists():
            return candidate
    raise RuntimeError("nvcc not found: the CUDA toolkit is required to build cachebridge_b200")


def up_to_date() -> bool:
    if not OUTPUT.exists():
        return False
    built = OUTPUT.stat().st_mtime
    return all(p.stat().st_mtime <= built for p in list(SOURCES) + HEADERS + [Path(__file__)])


def build(verbose: bool = False, force: bool = False) -> Path:
    """Compile the library if any source is newer than it; return its path."""
    if not force and up_to_date():
        return OUTPUT
    nvcc = nvcc_path()
    objdir = PACKAGE.parent / "_build"
    objdir.mkdir(exist_ok=True)
    objects = []
    for src in SOURCES:
        obj = objdir / (src.stem + ".o")
        cmd = [nvcc, *ARCH_FLAGS, *COMMON_FLAGS, "-c", str(src), "-o", str(obj)]
        if verbose:
            cmd.insert(1, "-Xptxas=-v")
        subprocess.run(cmd, check=True)
        objects.append(str(obj))
    tmp = OUTPUT.with_suffix(".so.tmp")
    subprocess.run(
        [nvcc, *ARCH_FLAGS, "-shared", "-Xcompiler", "-fPIC", *objects, "-o", str(tmp)],
        check=True,
    )
    os.replace(tmp, OUTPUT)
    return OUTPUT


if __name__ == "__main__":
    path = build(verbose="-v" in sys.argv, force="-f" in sys.argv or "-v" in sys.argv)
    print(path)
