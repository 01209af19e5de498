"""Compile libfa_b200.so (the sm_100a kernels + C ABI) in-tree.

Run as ``python -m frame_analytics_b200._build`` or through
``__graft_entry__.build()``.  The library is written next to this file under
``_lib/`` so it travels with the source tree; nothing is cached elsewhere.

Flags follow the reference's numerics contract (frame_analytics/_cabi.py:291-300):
IEEE division and square root, no flush-to-zero, no fast-math.
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
CSRC = HERE / "csrc"
LIBDIR = HERE / "_lib"
LIB = LIBDIR / "libfa_b200.so"
SOURCES = ["abi.cu", "pixel.cu", "ssim_fwd.cu", "ssim_bwd.cu", "gmsd.cu", "pool.cu", "grad_scale.cu",
           "ssim_compat.cu", "f64.cu",
           "ssimulacra2.cu"]

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "-prec-div=true", "-prec-sqrt=true", "-ftz=false",
    "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
    "--expt-relaxed-constexpr",
]


def _nvcc() -> str:
    cand = os.environ.get("NVCC") or shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(cand).exists():
        raise RuntimeError(f"nvcc not found (looked for {cand})")
    return cand


def sources() -> list:
    return [CSRC / s for s in SOURCES] + sorted(CSRC.glob("*.cuh")) + [
        HERE.parent / "include" / "fa_b200.h"]


def up_to_date() -> bool:
    if not LIB.exists():
        return False
    t = LIB.stat().st_mtime
    return all(p.stat().st_mtime <= t for p in sources() if p.exists())


def build(force: bool = False, verbose: bool = False, ptxas_info: bool = False) -> Path:
    """Compile every .cu into one shared library (atomic rename into place)."""
    if not force and up_to_date():
        return LIB
    LIBDIR.mkdir(exist_ok=True)
    objdir = LIBDIR / "obj"
    objdir.mkdir(exist_ok=True)
    nvcc = _nvcc()
    extra = ["-Xptxas", "-v"] if ptxas_info else []
    procs = []
    for src in SOURCES:  # one nvcc per translation unit, in parallel
        obj = objdir / (Path(src).stem + ".o")
        cmd = [nvcc, *extra, *NVCC_FLAGS, "-c", str(CSRC / src), "-o", str(obj)]
        if verbose:
            print(" ".join(cmd), flush=True)
        procs.append((src, obj, subprocess.Popen(cmd, stdout=subprocess.PIPE,
                                                 stderr=subprocess.PIPE, text=True)))
    errors = []
    for src, obj, pr in procs:
        out, err = pr.communicate()
        if pr.returncode != 0:
            errors.append(f"{src}: nvcc failed ({pr.returncode}):\n{err}\n{out}")
        elif ptxas_info or verbose:
            sys.stdout.write(err)
    if errors:
        raise RuntimeError("\n".join(errors))
    tmp = LIBDIR / f".libfa_b200.{os.getpid()}.so"
    cmd = [nvcc, "-gencode", "arch=compute_100a,code=sm_100a", "-shared", "-o", str(tmp),
           *[str(o) for _, o, _ in procs]]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        tmp.unlink(missing_ok=True)
        raise RuntimeError(f"link failed ({res.returncode}):\n{res.stderr}\n{res.stdout}")
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose=True, ptxas_info="-v" in sys.argv)
    print(LIB)
