"""Builds libncm_cuda.so (the sm_100a kernels and their C ABI) in-tree.

Usage: python -m ncmorph_b200.build [--force]

Each ``csrc/*.cu`` translation unit is compiled with nvcc for sm_100a only
(``-gencode arch=compute_100a,code=sm_100a``) into ``_build/`` and linked
into ``ncmorph_b200/libncm_cuda.so``. Objects are rebuilt when their source
or any header under ``csrc/`` or ``include/`` is newer.
"""
from __future__ import annotations

import concurrent.futures as cf
import os
import pathlib
import shutil
import subprocess
import sys

PKG = pathlib.Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
INCLUDE = ROOT / "include"
BUILD = ROOT / "_build" / "ncm_cuda"
LIB = PKG / "libncm_cuda.so"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH + [
    "-O3",
    "-std=c++17",
    "-lineinfo",
    "-Xcompiler", "-fPIC",
    "-Xcompiler", "-fvisibility=hidden",
    "--expt-relaxed-constexpr",
    "-I", str(INCLUDE),
]


def nvcc() -> str:
    cand = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(cand):
        raise RuntimeError("nvcc not found; the CUDA toolkit is required to build libncm_cuda.so")
    return cand


def _newest_header() -> float:
    hs = list(CSRC.glob("*.cuh")) + list(CSRC.glob("*.h")) + list(INCLUDE.glob("*.h"))
    return max((h.stat().st_mtime for h in hs), default=0.0)


def _compile(src: pathlib.Path, obj: pathlib.Path, extra: list[str]) -> str:
    cmd = [nvcc(), *NVCC_FLAGS, *extra, "-c", str(src), "-o", str(obj)]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src.name}:\n{' '.join(cmd)}\n{r.stdout}\n{r.stderr}")
    return r.stderr


def build(force: bool = False, verbose: bool = False, extra: list[str] | None = None) -> pathlib.Path:
    """Compiles every csrc/*.cu for sm_100a and links libncm_cuda.so."""
    extra = list(extra or [])
    BUILD.mkdir(parents=True, exist_ok=True)
    hdr = _newest_header()
    srcs = sorted(CSRC.glob("*.cu"))
    jobs = []
    for src in srcs:
        obj = BUILD / (src.stem + ".o")
        if force or not obj.exists() or obj.stat().st_mtime < max(src.stat().st_mtime, hdr):
            jobs.append((src, obj))
    if jobs:
        with cf.ThreadPoolExecutor(max_workers=min(len(jobs), os.cpu_count() or 4)) as ex:
            futs = {ex.submit(_compile, s, o, extra): s for s, o in jobs}
            for f in cf.as_completed(futs):
                msg = f.result()
                if verbose and msg.strip():
                    print(f"[{futs[f].name}]\n{msg}", file=sys.stderr)
    objs = [BUILD / (s.stem + ".o") for s in srcs]
    if force or jobs or not LIB.exists() or LIB.stat().st_mtime < max(o.stat().st_mtime for o in objs):
        tmp = LIB.with_suffix(".so.tmp")
        cmd = [nvcc(), *ARCH, "-shared", "-o", str(tmp), *map(str, objs), "-lcudart_static", "-lrt", "-ldl",
               "-lpthread"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{' '.join(cmd)}\n{r.stdout}\n{r.stderr}")
        os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    args = sys.argv[1:]
    extra = []
    if "--ptxas-v" in args:
        extra += ["-Xptxas", "-v"]
    path = build(force="--force" in args or bool(extra), verbose=True, extra=extra)
    print(path)
