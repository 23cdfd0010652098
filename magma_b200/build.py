"""Builds libmagma_cuda.so in-tree with nvcc for sm_100a.

Each ``csrc/*.cu`` compiles to an object under ``magma_b200/_build/`` (in
parallel, skipped when the object is newer than its sources), then everything
links into ``magma_b200/libmagma_cuda.so`` with the CUDA runtime linked
statically. Run ``python -m magma_b200.build`` or call :func:`build`.
"""
from __future__ import annotations

import concurrent.futures as cf
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
CSRC = PKG / "csrc"
BUILD = PKG / "_build"
LIB = PKG / "libmagma_cuda.so"
INCLUDE = PKG.parent / "include"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = [
    "-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
    "--expt-relaxed-constexpr", "-DNDEBUG",
]


def _nvcc() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found: set NVCC or install the CUDA toolkit")


def _headers() -> list[Path]:
    return sorted(CSRC.glob("*.cuh")) + sorted(INCLUDE.glob("*.h"))


def _needs(obj: Path, deps: list[Path]) -> bool:
    if not obj.exists():
        return True
    t = obj.stat().st_mtime
    return any(d.stat().st_mtime > t for d in deps)


def _compile(nvcc: str, src: Path, obj: Path, verbose: bool) -> None:
    cmd = [nvcc, *ARCH, *NVCC_FLAGS, "-I", str(INCLUDE), "-c", str(src), "-o", str(obj)]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src.name}:\n{r.stdout}\n{r.stderr}")
    if verbose and r.stderr:
        sys.stderr.write(r.stderr)


def build(verbose: bool = False, jobs: int | None = None) -> Path:
    """Compiles every csrc/*.cu for sm_100a and links libmagma_cuda.so."""
    nvcc = _nvcc()
    BUILD.mkdir(exist_ok=True)
    headers = _headers()
    sources = sorted(CSRC.glob("*.cu"))
    todo = []
    objs = []
    for src in sources:
        obj = BUILD / (src.stem + ".o")
        objs.append(obj)
        if _needs(obj, [src, *headers]) or verbose:
            todo.append((src, obj))
    if todo:
        with cf.ThreadPoolExecutor(max_workers=jobs or min(8, os.cpu_count() or 4)) as ex:
            futs = [ex.submit(_compile, nvcc, s, o, verbose) for s, o in todo]
            for f in futs:
                f.result()
    if todo or _needs(LIB, objs):
        tmp = LIB.with_suffix(".so.tmp")
        cmd = [nvcc, *ARCH, "-shared", "-Xcompiler", "-fPIC", "-o", str(tmp), *map(str, objs),
               "-cudart", "static", "-lpthread", "-ldl", "-lrt"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
        os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    print(build(verbose="-v" in sys.argv))
