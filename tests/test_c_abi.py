"""The C ABI from a C program (no Python, no torch): tests/c_abi/abi_example.c
compiled with gcc against include/pla_b200.h, linked to pla_b200/libpla_b200.so
(and libcudart for its allocations)."""
import os
import shutil
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
CUDA_LIB = "/usr/local/cuda/lib64"


@pytest.fixture(scope="module")
def exe(tmp_path_factory):
    if not shutil.which("gcc"):
        pytest.skip("no gcc")
    out = str(tmp_path_factory.mktemp("cabi") / "abi_example")
    libdir = os.path.join(ROOT, "pla_b200")
    cmd = ["gcc", "-O1", "-std=c11", "-I", os.path.join(ROOT, "include"),
           os.path.join(ROOT, "tests", "c_abi", "abi_example.c"), "-o", out,
           "-L", libdir, f"-Wl,-rpath,{libdir}", "-lpla_b200", "-L", CUDA_LIB, f"-Wl,-rpath,{CUDA_LIB}",
           "-lcudart", "-lm", "-ffp-contract=off"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    return out


def test_c_caller_cpu(exe):
    r = subprocess.run([exe, "cpu"], capture_output=True, text=True, timeout=120)
    assert r.returncode == 0 and "cpu ok" in r.stdout, r.stdout + r.stderr


@pytest.mark.gpu
def test_c_caller_gpu(exe):
    r = subprocess.run([exe, "gpu"], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0 and "gpu ok" in r.stdout, r.stdout + r.stderr
