"""Build recipe of the CPU oracle ``oracle/_build/libtgs_oracle.so``.

TEST INFRASTRUCTURE ONLY: the oracle is the checker of the parity tests,
smoke() and bench.py's cpu_baseline leg; the product library never links or
loads it.  Plain C11 compiled with gcc, OpenMP for the tile/Gaussian loops
and no floating-point contraction (-ffp-contract=off) so the restatement
evaluates every float operation as written.
"""
from __future__ import annotations

import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
SRC = HERE / "tgs_oracle.c"
HDR = HERE / "tgs_oracle.h"
LIB = HERE / "_build" / "libtgs_oracle.so"


def build(force: bool = False, verbose: bool = False) -> Path:
    LIB.parent.mkdir(exist_ok=True)
    if not force and LIB.exists() and LIB.stat().st_mtime >= max(SRC.stat().st_mtime, HDR.stat().st_mtime,
                                                                   Path(__file__).stat().st_mtime):
        return LIB
    cmd = ["gcc", "-O2", "-std=c11", "-fopenmp", "-ffp-contract=off", "-fPIC", "-shared", "-Wall", "-Wextra",
           "-o", str(LIB), str(SRC), "-lm"]
    if verbose:
        print(" ".join(cmd))
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError("oracle build failed:\n" + r.stdout + r.stderr)
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose=True))
