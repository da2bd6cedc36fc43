"""Build ``qi_b200/libqi_b200.so`` (the C-ABI library) in-tree with nvcc for
sm_100a.  No torch headers are involved: the library is plain CUDA C++ with
an ``extern "C"`` surface declared in ``include/qi_b200.h``.

    python -m qi_b200.build [--verbose]
"""

from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
LIB = PKG / "libqi_b200.so"

SOURCES = [CSRC / "qi_b200.cu"]
DEPS = sorted(CSRC.glob("*.cu*")) + [ROOT / "include" / "qi_b200.h"]

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-std=c++17", "-lineinfo",
    "--shared", "-Xcompiler", "-fPIC",
    "-Xptxas", "-warn-spills",
    # IEEE division / reciprocal / rounding are part of the numerics contract:
    # never --use_fast_math.
    "-prec-div=true", "-prec-sqrt=true", "-ftz=false",
]


def nvcc_path() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found")


def needs_build() -> bool:
    if not LIB.exists():
        return True
    t = LIB.stat().st_mtime
    return any(p.stat().st_mtime > t for p in DEPS)


def build(force: bool = False, verbose: bool = False) -> Path:
    if not force and not needs_build():
        return LIB
    tmp = LIB.with_suffix(".so.tmp")
    cmd = [nvcc_path(), *NVCC_FLAGS, "-I", str(ROOT / "include"), "-o", str(tmp), *map(str, SOURCES)]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
        print(" ".join(cmd), flush=True)
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        sys.stderr.write(res.stdout + res.stderr)
        raise RuntimeError(f"nvcc failed ({res.returncode}) building {LIB.name}")
    if verbose:
        sys.stderr.write(res.stdout + res.stderr)
    os.replace(tmp, LIB)
    return LIB


TORCH_OPS_SRC = CSRC / "torch_ops.cpp"
TORCH_OPS_LIB = PKG / "libqi_b200_torch.so"


def build_torch_ops(force: bool = False, verbose: bool = False) -> Path:
    """Build ``libqi_b200_torch.so``: the torch operators (``qi_int8_w8a8::linear``
    with the reference's schema, ``qi_b200::*``) over the C ABI, linked to the
    in-tree ``libqi_b200.so`` (found next to it at run time).  Plain g++
    against torch's headers and libraries; load it with
    ``torch.ops.load_library``."""
    import torch
    from torch.utils import cpp_extension as ce

    deps = [TORCH_OPS_SRC, ROOT / "include" / "qi_b200.h", LIB]
    if not force and TORCH_OPS_LIB.exists() and all(p.stat().st_mtime <= TORCH_OPS_LIB.stat().st_mtime for p in deps):
        return TORCH_OPS_LIB
    build(force=False)
    cuda_home = Path(nvcc_path()).resolve().parent.parent
    cmd = ["g++", "-O2", "-std=c++17", "-fPIC", "-shared",
           f"-D_GLIBCXX_USE_CXX11_ABI={int(torch._C._GLIBCXX_USE_CXX11_ABI)}",
           *[f"-I{p}" for p in ce.include_paths()], f"-I{cuda_home / 'include'}", f"-I{ROOT / 'include'}",
           str(TORCH_OPS_SRC), "-o", str(TORCH_OPS_LIB.with_suffix(".so.tmp")),
           *[f"-L{p}" for p in ce.library_paths()], f"-L{PKG}", "-lqi_b200",
           "-ltorch", "-ltorch_cpu", "-ltorch_cuda", "-lc10", "-lc10_cuda",
           f"-L{cuda_home / 'lib64'}", "-lcudart", "-Wl,-rpath,$ORIGIN"]
    if verbose:
        print(" ".join(cmd), flush=True)
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        sys.stderr.write(res.stdout + res.stderr)
        raise RuntimeError(f"g++ failed ({res.returncode}) building {TORCH_OPS_LIB.name}")
    os.replace(TORCH_OPS_LIB.with_suffix(".so.tmp"), TORCH_OPS_LIB)
    return TORCH_OPS_LIB


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--verbose", action="store_true")
    ap.add_argument("--force", action="store_true")
    a = ap.parse_args()
    print(build(force=a.force or a.verbose, verbose=a.verbose))
    print(build_torch_ops(force=a.force, verbose=a.verbose))


if __name__ == "__main__":
    main()
