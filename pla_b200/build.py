"""Ahead-of-time build of the two in-tree libraries (next to this file).

    python -m pla_b200.build [--force]

* ``libpla_b200.so``: the sm_100a kernels behind the C ABI
  (include/pla_b200.h).  nvcc cross-compiles without a GPU; this is what the
  Python package and any C/C++ host load.
* ``libpla_b200_torch.so``: the torch custom ops (``torch.ops.pla_b200.*``,
  csrc/torch_ops.cpp), plain C++ over that C ABI, compiled with g++ against
  the installed torch's headers and linked to ``libpla_b200.so`` by rpath.
"""
from __future__ import annotations

import argparse
import glob
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
OUT = os.path.join(HERE, "libpla_b200.so")
TORCH_OUT = os.path.join(HERE, "libpla_b200_torch.so")

NVCC_FLAGS = [
    "-std=c++17", "-O3", "-lineinfo",
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
    "-shared", "-Xlinker", "-soname=libpla_b200.so",
]


def _nvcc() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def sources() -> list[str]:
    return sorted(glob.glob(os.path.join(CSRC, "*.cu")) + glob.glob(os.path.join(CSRC, "*.cuh"))
                  + [os.path.join(ROOT, "include", "pla_b200.h")])


def torch_sources() -> list[str]:
    return [os.path.join(CSRC, "torch_ops.cpp"), os.path.join(ROOT, "include", "pla_b200.h")]


def up_to_date(out: str = OUT, srcs: list[str] | None = None) -> bool:
    if not os.path.exists(out):
        return False
    t = os.path.getmtime(out)
    return all(os.path.getmtime(s) <= t for s in (sources() if srcs is None else srcs))


def _run(cmd: list[str], out: str, verbose: bool) -> None:
    if verbose:
        print(" ".join(cmd))
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"{os.path.basename(cmd[0])} failed:\n{r.stdout}\n{r.stderr}")
    os.replace(out + ".tmp", out)


def torch_cmd() -> list[str]:
    """g++ command for libpla_b200_torch.so (torch's headers, ABI flag and libraries)."""
    import torch
    from torch.utils import cpp_extension

    cuda_home = cpp_extension.CUDA_HOME or "/usr/local/cuda"
    cmd = [shutil.which("g++") or "g++", "-std=c++17", "-O2", "-fPIC", "-shared", "-fvisibility=hidden",
           f"-D_GLIBCXX_USE_CXX11_ABI={int(torch._C._GLIBCXX_USE_CXX11_ABI)}"]
    cmd += [f"-I{p}" for p in cpp_extension.include_paths()] + [f"-I{os.path.join(cuda_home, 'include')}"]
    cmd += ["-o", TORCH_OUT + ".tmp", os.path.join(CSRC, "torch_ops.cpp")]
    cmd += [f"-L{p}" for p in cpp_extension.library_paths()] + ["-lc10", "-lc10_cuda", "-ltorch_cpu", "-ltorch"]
    cmd += [f"-L{HERE}", "-lpla_b200", "-Wl,-rpath,$ORIGIN"]
    return cmd


def build(force: bool = False, verbose: bool = False) -> str:
    if force or not up_to_date():
        _run([_nvcc(), *NVCC_FLAGS, "-o", OUT + ".tmp", os.path.join(CSRC, "pla_capi.cu")], OUT, verbose)
    if force or not up_to_date(TORCH_OUT, torch_sources() + [OUT]):
        _run(torch_cmd(), TORCH_OUT, verbose)
    return OUT


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    args = ap.parse_args()
    print(build(force=args.force, verbose=True))
    sys.exit(0)
