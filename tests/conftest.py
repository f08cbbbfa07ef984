"""Shared test setup.

CPU tests (-m "not gpu") check the oracle against the golden vectors and the
reference's own sampler, the host logic, and that libt3b200.so loads and
exports every symbol of include/t3b200.h.  GPU tests (-m gpu) compare the
CUDA path, called through the C ABI, with the oracle.
"""
import importlib.util
import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG_DIR = os.path.join(ROOT, "chatterbox.cpp_b200")
sys.path.insert(0, os.path.join(ROOT, "oracle"))
sys.path.insert(0, ROOT)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200)")


def load_package():
    """Import chatterbox.cpp_b200/ (a directory name with a dot) as the
    module `chatterbox_cpp_b200`."""
    name = "chatterbox_cpp_b200"
    if name in sys.modules:
        return sys.modules[name]
    spec = importlib.util.spec_from_file_location(name, os.path.join(PKG_DIR, "__init__.py"),
                                                  submodule_search_locations=[PKG_DIR])
    mod = importlib.util.module_from_spec(spec)
    sys.modules[name] = mod
    spec.loader.exec_module(mod)
    return mod


@pytest.fixture(scope="session")
def pkg():
    return load_package()


@pytest.fixture(scope="session")
def orc():
    import oracle
    if not os.path.exists(oracle.LIB):
        oracle.build(ref=None)
    oracle.lib()
    return oracle


def rel_err(got, ref):
    """chatterbox.cpp's compare_f32 metric (src/npy.h:195-211): max |got-ref|
    divided by max |ref|."""
    got = np.asarray(got, np.float64)
    ref = np.asarray(ref, np.float64)
    return float(np.max(np.abs(got - ref)) / max(np.max(np.abs(ref)), 1e-30))


def synth_logits(seed, n=6563, scale=3.0, kind="normal"):
    """Deterministic synthetic logits (numpy PCG64, float64 -> float32)."""
    rng = np.random.default_rng(seed)
    x = rng.standard_normal(n) * scale
    if kind == "rounded":
        x = np.round(x, 1)
    return x.astype(np.float32)


def gpu_available():
    try:
        import torch
        return torch.cuda.is_available()
    except Exception:
        return False
