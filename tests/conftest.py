"""Shared test set-up: the `gpu` marker, import paths, built artefacts."""
import os
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "php-gpu-tensors_b200")
for p in (PKG, os.path.join(ROOT, "tests")):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA B200 (sm_100a) device")


def _ensure_built():
    lib = os.path.join(PKG, "libgemm_sm100.so")
    oracle = os.path.join(ROOT, "oracle", "liboracle.so")
    if not (os.path.exists(lib) and os.path.exists(oracle)):
        subprocess.run([sys.executable, os.path.join(PKG, "build.py")], check=True)


_ensure_built()


@pytest.fixture(scope="session")
def golden():
    import json
    with open(os.path.join(ROOT, "tests", "golden", "matmul_golden.json")) as f:
        return json.load(f)
