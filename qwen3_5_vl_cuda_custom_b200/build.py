"""Ahead-of-time build of the sm_100a kernel library ``libq35b200.so``.

Each ``csrc/*.cu`` file is compiled separately by nvcc (in parallel, skipped
when the object is newer than its sources) and linked into one shared library
inside the package directory, so the built library travels with the source
tree.  The library exports only the ``extern "C"`` entry points declared in
``include/q35b200.h``; the CUDA runtime is linked statically, so the library
needs only the NVIDIA driver at run time.

Usage: ``python -m qwen3_5_vl_cuda_custom_b200.build [--force]``.
"""
from __future__ import annotations

import concurrent.futures as cf
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG_DIR = Path(__file__).resolve().parent
CSRC = PKG_DIR / "csrc"
BUILD_DIR = PKG_DIR / "_build"
LIB_NAME = "libq35b200.so"
LIB_PATH = PKG_DIR / LIB_NAME
INCLUDE_DIR = PKG_DIR.parent / "include"

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = [
    "-O3",
    "-std=c++17",
    "-lineinfo",
    "-Xcompiler", "-fPIC",
    "-Xcompiler", "-fvisibility=hidden",
    "--expt-relaxed-constexpr",
    "-Xptxas", "-v",
]


def _nvcc() -> str:
    cuda_home = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    cand = Path(cuda_home) / "bin" / "nvcc"
    if cand.exists():
        return str(cand)
    found = shutil.which("nvcc")
    if not found:
        raise RuntimeError("nvcc not found: set CUDA_HOME")
    return found


def _sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu"))


def _headers() -> list[Path]:
    return sorted(CSRC.glob("*.cuh")) + sorted(INCLUDE_DIR.glob("*.h"))


def _compile(src: Path, obj: Path, verbose: bool) -> str:
    cmd = [_nvcc(), *ARCH_FLAGS, *NVCC_FLAGS, "-I", str(INCLUDE_DIR), "-c",
           str(src), "-o", str(obj)]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed on {src.name}:\n{res.stdout}\n{res.stderr}")
    log = BUILD_DIR / (src.stem + ".ptxas.txt")
    log.write_text(res.stderr)
    if verbose:
        print(f"[q35b200] compiled {src.name}", file=sys.stderr)
    return res.stderr


def build(force: bool = False, verbose: bool = False) -> Path:
    """Compiles every kernel source and links ``libq35b200.so``; returns its path."""
    BUILD_DIR.mkdir(exist_ok=True)
    newest_header = max((h.stat().st_mtime for h in _headers()), default=0.0)
    jobs = []
    objs = []
    for src in _sources():
        obj = BUILD_DIR / (src.stem + ".o")
        objs.append(obj)
        stale = (force or not obj.exists()
                 or obj.stat().st_mtime < max(src.stat().st_mtime, newest_header))
        if stale:
            jobs.append((src, obj))
    if jobs:
        with cf.ThreadPoolExecutor(max_workers=min(len(jobs), os.cpu_count() or 4)) as ex:
            futs = [ex.submit(_compile, s, o, verbose) for s, o in jobs]
            for f in futs:
                f.result()
    lib_stale = (not LIB_PATH.exists() or jobs
                 or LIB_PATH.stat().st_mtime < max(o.stat().st_mtime for o in objs))
    if lib_stale:
        tmp = LIB_PATH.with_suffix(".so.tmp")
        cmd = [_nvcc(), *ARCH_FLAGS, "-shared", "-cudart", "static",
               *[str(o) for o in objs], "-o", str(tmp)]
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            raise RuntimeError(f"link failed:\n{res.stdout}\n{res.stderr}")
        os.replace(tmp, LIB_PATH)
        if verbose:
            print(f"[q35b200] linked {LIB_PATH}", file=sys.stderr)
    return LIB_PATH


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose=True)
