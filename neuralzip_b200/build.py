"""Builds libnzb200.so in-tree (nvcc, sm_100a).

Run as ``python -m neuralzip_b200.build``. The library holds the host packer
(C++) and the tile decode kernel (CUDA) behind the C ABI of
``include/nz_b200.h``; it is written next to this file under ``_lib/`` so a
snapshot of the repository carries it.
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

PACKAGE = Path(__file__).resolve().parent
ROOT = PACKAGE.parent
CSRC = PACKAGE / "csrc"
OUTPUT = PACKAGE / "_lib" / "libnzb200.so"
SOURCES = ("nz_host.cpp", "nz_huff0.cpp", "nz_storage.cpp", "nz_setup.cpp", "nz_schedule.cpp", "nz_decode.cu")
HEADERS = (ROOT / "include" / "nz_b200.h", CSRC / "nz_internal.h")
ARCH = ("-gencode", "arch=compute_100a,code=sm_100a")


def nvcc():
    for candidate in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if candidate and Path(candidate).exists():
            return candidate
    raise RuntimeError("nvcc was not found; set NVCC or put CUDA's bin directory on PATH.")


def _stale():
    if not OUTPUT.exists():
        return True
    built = OUTPUT.stat().st_mtime
    inputs = [CSRC / name for name in SOURCES] + list(HEADERS) + [Path(__file__)]
    return any(path.stat().st_mtime > built for path in inputs)


def build(force=False, verbose=False, extra=()):
    """Compiles the library when a source is newer than it; returns its path."""
    if not force and not _stale():
        return OUTPUT
    OUTPUT.parent.mkdir(parents=True, exist_ok=True)
    tmp = OUTPUT.with_suffix(".so.tmp")
    command = [
        nvcc(), *ARCH, "-lineinfo", "-O3", "-std=c++17", "-shared",
        "-Xcompiler", "-fPIC,-O3,-pthread",
        "-Xptxas", "-v" if verbose else "-O3",
        f"-I{ROOT / 'include'}", f"-I{CSRC}",
        *extra,
        "-o", str(tmp),
        *(str(CSRC / name) for name in SOURCES),
    ]
    result = subprocess.run(command, capture_output=True, text=True)
    if result.returncode != 0:
        raise RuntimeError(f"nvcc failed ({result.returncode}):\n{result.stdout}\n{result.stderr}")
    if verbose:
        sys.stderr.write(result.stdout + result.stderr)
    os.replace(tmp, OUTPUT)
    return OUTPUT


if __name__ == "__main__":
    path = build(force="--force" in sys.argv, verbose="-v" in sys.argv)
    print(path)
