"""The C++ host mirror (kvm::KvMemStore over the C ABI) against the reference
store's own test expectations, compiled with the system C++ compiler and run
on the GPU."""
import os
import subprocess
import tempfile

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "kvmem-llama.cpp_b200")

pytestmark = pytest.mark.gpu


def test_cpp_store_mirror_reference_cases(kvm_lib):
    cxx = os.environ.get("CXX", "g++")
    libdir = os.path.join(PKG, "kvm")
    with tempfile.TemporaryDirectory() as d:
        exe = os.path.join(d, "kvm_store_gpu_test")
        subprocess.run([cxx, "-std=c++17", "-O1", "-I", os.path.join(ROOT, "include"),
                        "-I", os.path.join(PKG, "host"),
                        os.path.join(ROOT, "tests", "cpp", "kvm_store_gpu_test.cpp"),
                        "-L", libdir, "-lkvm", f"-Wl,-rpath,{libdir}", "-o", exe], check=True)
        r = subprocess.run([exe], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "all checks passed" in r.stdout
