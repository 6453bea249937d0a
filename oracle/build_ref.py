"""Build recipe of ``oracle/_ref/libtgs_ref.so``: the reference's own CUDA
kernels, compiled unchanged from their sources where they lie.

TEST INFRASTRUCTURE ONLY.  The library holds the reference's fp32 and fp16
rasterizers (tinygs/src/rasterizer/fastgs_ours/{forward,backward}.cu,
fastgs_ours_fp16/{forward,backward}.cu), its L1 loss (tinygs/src/loss/l1.cu)
and fused SSIM (tinygs/src/loss/fused_ssim.cu), plus this repository's
harness (oracle/ref/) that drives them through their own raw entry points
(fastgs_ours/forward.h:13-45, backward.h:13-53, LossBase::evaluate) and reads
their scratch back.  The parity tests compare the product with it on the
same inputs, and bench.py's reference arm times the reference's training
step with it on the GPU.

The reference's CMake build fetches glm, nlohmann_json, spdlog, cxxopts and
google-benchmark over the network (cmake/dependencies.cmake:5-62); its
kernels need only a handful of names from the headers that pull those in, so
``oracle/refshim/`` stands in for exactly those headers.  The flags are the
reference's release flags for CUDA (tinygs/CMakeLists.txt: --use_fast_math,
C++20, NDEBUG), for sm_100a.  The reference's SimpleAdam
(tinygs/src/optim/simple_adam.cu) is built too, with stand-ins for the glm
vector types and the GPUGaussian3d container and the config plumbing of
optim/optim.cu restated in oracle/ref/ref_adam.cu; it needs nlohmann/json,
found vendored in an installed Python package (when none is, the optimizer
is left out).

Built only where the reference sources are present (this container); the
GPU box runs the prebuilt library, which travels with the repository.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
SHIM = HERE / "refshim"
HARNESS = HERE / "ref"
OUT = HERE / "_ref"
LIB = OUT / "libtgs_ref.so"
REFERENCE = Path(os.environ.get("TGS_REFERENCE_ROOT", "/root/reference")) / "tinygs"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "--use_fast_math", "-std=c++20", "-DNDEBUG", "--extended-lambda", "-Xcompiler", "-fPIC", "-w",
         "-I", str(SHIM), "-I", str(HARNESS)]


def json_include() -> list[str]:
    """nlohmann/json (a header-only third-party library the reference's
    optimizer configuration uses), from a copy vendored in an installed
    Python package; empty when none is found."""
    import glob
    import site

    roots = site.getsitepackages() + [site.getusersitepackages()]
    for root in roots:
        for hit in glob.glob(f"{root}/**/nlohmann/json.hpp", recursive=True):
            return ["-I", str(Path(hit).parents[1])]
    return []


def units() -> list[tuple[Path, list[str]]]:
    """(source, extra include dirs) of every translation unit."""
    raster = ["-I", str(REFERENCE / "src" / "rasterizer")]
    inc = ["-I", str(REFERENCE / "include")]
    src = REFERENCE / "src"
    js = json_include()
    adam = [(src / "optim" / "simple_adam.cu", inc + js), (HARNESS / "ref_adam.cu", inc + js)] if js else []
    return adam + [
        (src / "rasterizer" / "fastgs_ours" / "forward.cu", []),
        (src / "rasterizer" / "fastgs_ours" / "backward.cu", []),
        (src / "rasterizer" / "fastgs_ours_fp16" / "forward.cu", []),
        (src / "rasterizer" / "fastgs_ours_fp16" / "backward.cu", []),
        (src / "loss" / "l1.cu", inc),
        (src / "loss" / "fused_ssim.cu", inc),
        (HARNESS / "ref_raster_f32.cu", raster),
        (HARNESS / "ref_raster_f16.cu", raster),
        (HARNESS / "ref_api.cu", inc),
    ]


def available() -> bool:
    return (REFERENCE / "src" / "rasterizer" / "fastgs_ours" / "forward.cu").exists()


def build(force: bool = False, verbose: bool = False) -> Path | None:
    """Compile and link; returns the library path, or None when the reference
    sources are absent (the prebuilt library, if any, is left as it is)."""
    if not available():
        return LIB if LIB.exists() else None
    nvcc = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    OUT.mkdir(exist_ok=True)
    deps = [Path(__file__), *SHIM.rglob("*.h*"), *HARNESS.glob("*")]
    newest_dep = max(p.stat().st_mtime for p in deps)
    procs, objs = [], []
    for i, (src, extra) in enumerate(units()):
        obj = OUT / f"{i:02d}_{src.stem}.o"
        objs.append(obj)
        if not force and obj.exists() and obj.stat().st_mtime >= max(newest_dep, src.stat().st_mtime):
            continue
        cmd = [nvcc, *ARCH, *FLAGS, *extra, "-c", str(src), "-o", str(obj)]
        if verbose:
            print(" ".join(cmd), flush=True)
        procs.append((src, subprocess.Popen(cmd, stdout=subprocess.PIPE, stderr=subprocess.STDOUT)))
    failed = []
    for src, p in procs:
        out, _ = p.communicate()
        if p.returncode != 0:
            failed.append(f"--- {src} ---\n{out.decode(errors='replace')}")
    if failed:
        raise RuntimeError("reference build failed:\n" + "\n".join(failed))
    for stale in OUT.glob("*.o"):
        if stale not in objs:
            stale.unlink()
    if force or not LIB.exists() or LIB.stat().st_mtime < max(o.stat().st_mtime for o in objs):
        cmd = [nvcc, *ARCH, "-shared", "-cudart", "static", "-o", str(LIB), *map(str, objs)]
        if verbose:
            print(" ".join(cmd), flush=True)
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError("reference link failed:\n" + r.stdout + r.stderr)
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose=True))
