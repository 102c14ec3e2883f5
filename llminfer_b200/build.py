"""Build recipe for the CUDA backend library.

Compiles every CUDA and host source under csrc/ for sm_100a only and links
them, with the CUDA runtime linked statically, into
llminfer_b200/_lib/libllmi_cuda.so (in-tree, so the built library travels
with the repository snapshot).  Objects go to llminfer_b200/_build/.
Sources are recompiled when they, or any header, are newer than their object.
"""
from __future__ import annotations

import concurrent.futures
import os
import shutil
import subprocess
import sys
from pathlib import Path

PACKAGE = Path(__file__).resolve().parent
ROOT = PACKAGE.parent
CSRC = PACKAGE / "csrc"
BUILD = PACKAGE / "_build"
LIBDIR = PACKAGE / "_lib"
LIBRARY = LIBDIR / "libllmi_cuda.so"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
CUDA_FLAGS = ARCH + [
    "-O3", "-lineinfo", "-std=c++17", "--expt-relaxed-constexpr",
    "-Xcompiler", "-fPIC", "-Xptxas", "-warn-spills",
]
HOST_FLAGS = ["-O2", "-std=c++17", "-Xcompiler", "-fPIC", "-Xcompiler", "-fno-exceptions",
              "-Xcompiler", "-Wall"]
INCLUDES = ["-I", str(ROOT / "include"), "-I", str(CSRC)]


def nvcc() -> str:
    found = shutil.which("nvcc")
    if found:
        return found
    default = "/usr/local/cuda/bin/nvcc"
    if os.path.exists(default):
        return default
    raise RuntimeError("nvcc not found: the CUDA toolkit is required to build llminfer_b200")


def _sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu")) + sorted((CSRC / "host").glob("*.cpp"))


def _headers() -> list[Path]:
    return (sorted(CSRC.rglob("*.cuh")) + sorted(CSRC.rglob("*.h"))
            + sorted((ROOT / "include").glob("*.h")))


def _compile(src: Path, obj: Path, verbose: bool) -> None:
    flags = CUDA_FLAGS if src.suffix == ".cu" else HOST_FLAGS
    cmd = [nvcc(), *flags, *INCLUDES, "-c", str(src), "-o", str(obj)]
    if verbose:
        print(" ".join(cmd), flush=True)
    result = subprocess.run(cmd, capture_output=True, text=True)
    if result.returncode != 0:
        raise RuntimeError(f"compiling {src.name} failed:\n{result.stdout}\n{result.stderr}")
    if verbose and (result.stdout.strip() or result.stderr.strip()):
        print(result.stdout + result.stderr, flush=True)


def build(verbose: bool = False, force: bool = False) -> Path:
    """Builds (or refreshes) the library and returns its path."""
    BUILD.mkdir(exist_ok=True)
    LIBDIR.mkdir(exist_ok=True)
    newest_header = max((h.stat().st_mtime for h in _headers()), default=0.0)
    jobs = []
    objects = []
    for src in _sources():
        obj = BUILD / (src.name + ".o")
        objects.append(obj)
        stale = (force or not obj.exists()
                 or obj.stat().st_mtime < max(src.stat().st_mtime, newest_header))
        if stale:
            jobs.append((src, obj))
    with concurrent.futures.ThreadPoolExecutor(max_workers=max(1, min(8, os.cpu_count() or 1))) as pool:
        for fut in [pool.submit(_compile, s, o, verbose) for s, o in jobs]:
            fut.result()
    if jobs or not LIBRARY.exists():
        tmp = LIBRARY.with_suffix(".so.tmp")
        cmd = [nvcc(), *ARCH, "-shared", "-cudart", "static", "-o", str(tmp),
               *map(str, objects), "-lpthread", "-ldl", "-lrt"]
        if verbose:
            print(" ".join(cmd), flush=True)
        result = subprocess.run(cmd, capture_output=True, text=True)
        if result.returncode != 0:
            raise RuntimeError(f"linking failed:\n{result.stdout}\n{result.stderr}")
        os.replace(tmp, LIBRARY)
    return LIBRARY


if __name__ == "__main__":
    build(verbose="-v" in sys.argv, force="-f" in sys.argv)
    print(LIBRARY)
