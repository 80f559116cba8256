"""Builds ``libsemx.so`` (the sm_100a kernels + C ABI) in-tree with nvcc.

Every ``csrc/*.cu`` file is compiled separately (in parallel) for
``-gencode arch=compute_100a,code=sm_100a`` and linked into one shared library next to
this file, so the library travels with the source tree. Rebuilds only when a source or
header is newer than the library, and recompiles only the sources whose object is older
than the source or any header. The CUDA runtime is linked statically; the driver is
resolved at first use, so the library also loads on machines without a GPU (for ABI
checks).
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

PKG_DIR = Path(__file__).resolve().parent
REPO_DIR = PKG_DIR.parent
CSRC = PKG_DIR / "csrc"
INCLUDE = REPO_DIR / "include"
BUILD_DIR = REPO_DIR / "_build"
LIB_PATH = PKG_DIR / "libsemx.so"

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
COMMON_FLAGS = [
    "-O3",
    "-lineinfo",
    "-std=c++17",
    "-Xcompiler",
    "-fPIC",
    "--expt-relaxed-constexpr",
    f"-I{INCLUDE}",
    f"-I{CSRC}",
]


def _nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found: the semx CUDA library cannot be built")


def sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu"))


def _headers() -> list[Path]:
    return sorted(CSRC.glob("*.cuh")) + sorted(INCLUDE.glob("*.h"))


def up_to_date() -> bool:
    if not LIB_PATH.exists():
        return False
    lib_m = LIB_PATH.stat().st_mtime
    return all(p.stat().st_mtime <= lib_m for p in sources() + _headers())


def _compile(src: Path, verbose_ptxas: bool) -> tuple[Path, str]:
    obj = BUILD_DIR / (src.stem + ".o")
    if not verbose_ptxas and obj.exists():
        obj_m = obj.stat().st_mtime
        if all(p.stat().st_mtime <= obj_m for p in [src] + _headers()):
            return obj, ""
    cmd = [_nvcc(), *ARCH_FLAGS, *COMMON_FLAGS, "-c", str(src), "-o", str(obj)]
    if verbose_ptxas:
        cmd += ["-Xptxas", "-v"]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src.name}:\n{res.stdout}\n{res.stderr}")
    return obj, res.stderr


def build(force: bool = False, verbose_ptxas: bool = False, quiet: bool = True) -> Path:
    """Compiles and links ``libsemx.so``; returns its path."""
    if not force and not verbose_ptxas and up_to_date():
        return LIB_PATH
    BUILD_DIR.mkdir(exist_ok=True)
    srcs = sources()
    with ThreadPoolExecutor(max_workers=min(8, len(srcs))) as ex:
        results = list(ex.map(lambda s: _compile(s, verbose_ptxas), srcs))
    if verbose_ptxas or not quiet:
        for (_, log), src in zip(results, srcs):
            if log.strip():
                print(f"== {src.name}\n{log}", file=sys.stderr)
    tmp = LIB_PATH.with_suffix(".so.tmp")
    cmd = [_nvcc(), *ARCH_FLAGS, "-shared", "-o", str(tmp), *[str(o) for o, _ in results]]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"link failed:\n{res.stdout}\n{res.stderr}")
    os.replace(tmp, LIB_PATH)
    return LIB_PATH


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose_ptxas="-v" in sys.argv, quiet=False)
    print(LIB_PATH)
