import os
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "kvmem-llama.cpp_b200")
for p in (PKG, os.path.join(ROOT, "oracle"), ROOT):
    if p not in sys.path:
        sys.path.insert(0, p)


def _ensure_built():
    lib = os.path.join(PKG, "kvmret", "libkvmret.so")
    orc = os.path.join(ROOT, "oracle", "liborc.so")
    if not os.path.exists(lib):
        subprocess.run(["make", "-C", os.path.join(PKG, "csrc")], check=True)
    if not os.path.exists(orc):
        subprocess.run(["make", "-C", os.path.join(ROOT, "oracle")], check=True)


_ensure_built()


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a)")


def pytest_collection_modifyitems(config, items):
    try:
        import torch
        has_gpu = torch.cuda.is_available()
    except Exception:
        has_gpu = False
    if has_gpu:
        return
    skip = pytest.mark.skip(reason="no CUDA GPU")
    for it in items:
        if "gpu" in it.keywords:
            it.add_marker(skip)
