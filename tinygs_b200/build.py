"""Build recipe of the CUDA library ``tinygs_b200/libtgs_b200.so``.

Every translation unit under ``csrc/`` is compiled for sm_100a only
(``-gencode arch=compute_100a,code=sm_100a``) with ``--use_fast_math`` --
the reference rasterizer is built with fast math too
(tinygs/CMakeLists.txt:198-203), and the tile-overlap decisions depend on
the same approximate log/sqrt/division -- and linked into one shared library
with the CUDA runtime linked statically, so the library loads on any box with
a driver and needs no toolkit path.  nvcc cross-compiles without a GPU.

Run as ``python -m tinygs_b200.build`` or through ``__graft_entry__.build()``.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
CSRC = HERE / "csrc"
INCLUDE = HERE.parent / "include"
BUILD = HERE / "_build"
LIB = HERE / "libtgs_b200.so"
HOST_DIR = HERE / "host"
DRIVER = HERE / "tgs_train_step"
CUDA_HOME = Path("/usr/local/cuda")

SOURCES = ["abi.cu", "preprocess.cu", "binning.cu", "blend.cu", "loss.cu", "adam.cu", "densify.cu", "arena.cu", "metrics.cu", "image.cu", "checkpoint.cu", "noalloc.cu"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-lineinfo", "--use_fast_math", "-std=c++20", "-Xcompiler", "-fPIC",
              "-Xcompiler", "-fvisibility=hidden", "--expt-relaxed-constexpr", "-I", str(INCLUDE),
              "-I", str(CSRC)]


def nvcc() -> str:
    cand = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(cand).exists():
        raise RuntimeError("nvcc not found; the CUDA toolkit is required to build tinygs_b200")
    return cand


def _stale(target: Path, deps: list[Path]) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(d.stat().st_mtime > t for d in deps)


def build(verbose: bool = False, force: bool = False, extra_flags: list[str] | None = None) -> Path:
    """Compile the CUDA sources and link libtgs_b200.so; returns the path."""
    BUILD.mkdir(exist_ok=True)
    headers = sorted(CSRC.glob("*.cuh")) + sorted(CSRC.glob("*.h")) + [INCLUDE / "tgs_abi.h"]
    flags = NVCC_FLAGS + (extra_flags or [])
    procs = []
    objs = []
    for src in SOURCES:
        s = CSRC / src
        o = BUILD / (Path(src).stem + ".o")
        objs.append(o)
        if force or _stale(o, [s, *headers, Path(__file__)]):
            cmd = [nvcc(), *ARCH, *flags, "-c", str(s), "-o", str(o)]
            if verbose:
                print(" ".join(cmd), flush=True)
            procs.append((src, subprocess.Popen(cmd, stdout=subprocess.PIPE, stderr=subprocess.STDOUT)))
    failed = []
    for src, p in procs:
        out, _ = p.communicate()
        text = out.decode(errors="replace")
        if p.returncode != 0:
            failed.append(f"--- {src} ---\n{text}")
        elif verbose and text.strip():
            print(text)
    if failed:
        raise RuntimeError("nvcc failed:\n" + "\n".join(failed))
    if force or _stale(LIB, objs):
        cmd = [nvcc(), *ARCH, "-shared", "-cudart", "static", "-o", str(LIB), *map(str, objs)]
        if verbose:
            print(" ".join(cmd), flush=True)
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError("link failed:\n" + r.stdout + r.stderr)
    return LIB


def build_host(verbose: bool = False, force: bool = False) -> Path:
    """Compile the C++20 driver of the plugin adapters (host code only, g++),
    linked against libtgs_b200.so (found next to it at run time)."""
    src = HOST_DIR / "train_step_main.cpp"
    deps = [src, HOST_DIR / "tgs_plugins.hpp", INCLUDE / "tgs_abi.h", LIB]
    if not force and not _stale(DRIVER, deps):
        return DRIVER
    cmd = ["g++", "-std=c++20", "-O2", "-Wall", "-Wextra", "-I", str(INCLUDE), "-I", str(CUDA_HOME / "include"),
           str(src), "-o", str(DRIVER), "-L", str(HERE), "-ltgs_b200", "-L", str(CUDA_HOME / "lib64"),
           "-lcudart_static", "-ldl", "-lrt", "-lpthread", "-Wl,-rpath,$ORIGIN"]
    if verbose:
        print(" ".join(cmd), flush=True)
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError("host driver build failed:\n" + r.stdout + r.stderr)
    return DRIVER


if __name__ == "__main__":
    build(verbose=True, force="--force" in sys.argv)
    build_host(verbose=True, force="--force" in sys.argv)
    print(LIB)
