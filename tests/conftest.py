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


def nudged(tensors):
    """Copy of a T3 tensor dict with model/wpe moved by one ulp: the
    perturbation used to measure the quantized path's own sensitivity."""
    t = dict(tensors)
    ty, w = tensors["model/wpe"]
    t["model/wpe"] = (ty, np.nextafter(w, np.float32(np.inf)).astype(np.float32))
    return t


def noise_floor(orc, hp, tensors, text, tokens, max_ctx, kv_f16=1):
    """rel distance between the oracle and the oracle on 1-ulp-nudged
    positions, for the prefill logits and each step's logits.

    With Q8_0 re-quantised activations a 1-ulp input change flips a few
    rounding decisions, each moving a GEMV output by ~d_x * w, and the flips
    compound through GELU's f16 rounding and the following layers: on the
    random-init T3 this is ~1e-2 of max|logit| (F16 weights: ~5e-4).  Two
    implementations that do not sum in the same order cannot agree more
    closely than this."""
    a = orc.Model(hp, tensors, max_ctx=max_ctx, gemv_mode=1, gelu_f16=1, kv_f16=kv_f16)
    b = orc.Model(hp, nudged(tensors), max_ctx=max_ctx, gemv_mode=1, gelu_f16=1, kv_f16=kv_f16)
    P, la = a.prompt(text)
    _, lb = b.prompt(text)
    out = [rel_err(lb, la)]
    for i, tok in enumerate(tokens):
        out.append(rel_err(b.step(P + i, tok), a.step(P + i, tok)))
    return out
