"""Shared pytest setup: import paths, the `gpu` marker, library fixtures."""
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "kvmem-llama.cpp_b200")
for p in (PKG, os.path.join(ROOT, "oracle"), ROOT):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200) and libkvm.so")


@pytest.fixture(scope="session")
def oracle():
    import oracle as O
    O.build()
    return O


@pytest.fixture(scope="session")
def kvm_lib():
    import torch
    if not torch.cuda.is_available():
        pytest.fail("GPU test collected without a CUDA device")
    import kvm
    kvm.build()
    kvm.lib()
    return kvm
