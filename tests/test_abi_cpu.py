"""CPU tests of the C ABI library and the host-side Python: the library loads,
exports every symbol include/t3b200.h declares, reports errors without a GPU,
and the GGUF writer/reader keep the converter's layout."""
import ctypes as C
import os
import re

import numpy as np
import pytest

from conftest import ROOT, gpu_available

HEADER = os.path.join(ROOT, "include", "t3b200.h")


def header_functions():
    src = open(HEADER).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(t3b_[a-z0-9_]+)\s*\(", src)))


def test_library_exports_every_declared_symbol(pkg):
    L = pkg.lib()
    names = header_functions()
    assert len(names) >= 20
    for n in names:
        assert hasattr(L, n), n
    assert sorted(pkg.EXPORTS) == names


def test_row_bytes(pkg):
    L = pkg.lib()
    assert L.t3b_op_row_bytes(2, 1024) == 576
    assert L.t3b_op_row_bytes(2, 4096) == 2304
    assert L.t3b_op_row_bytes(8, 1024) == 1088
    assert L.t3b_op_row_bytes(1, 1024) == 2048
    for ty in (1, 2, 8):
        assert L.t3b_op_row_bytes(ty, 4096) % 16 == 0


def test_expf_fixup_list_small(pkg):
    # t3_expf_core restates glibc's expf (FMA build), so the build-time scan of
    # every float in [-104, 0] finds no or almost no arguments where the host
    # libm differs; those few would be served from the device fix-up table.
    n = pkg.lib().t3b_expf_fixup_count()
    assert 0 <= n < 1000


@pytest.mark.skipif(gpu_available(), reason="checks the no-device error path")
def test_create_without_device_reports_error(pkg):
    hp, t = pkg.t3_gguf.random_t3(dict(pkg.t3_gguf.T3_TURBO, n_layer=1, n_ctx=64, n_text_vocab=300), seed=1)
    with pytest.raises(pkg.T3BError) as e:
        pkg.T3Model(hp, t, device=0)
    assert "t3b_create" in str(e.value)


def test_bad_descriptor_is_rejected(pkg):
    L = pkg.lib()
    assert not L.t3b_create(0, None)
    assert "null" in pkg.last_error().lower()


@pytest.mark.parametrize("fn", ["t3b_op_attention", "t3b_op_attention_prompt", "t3b_op_attention_noalloc"])
def test_attention_ops_reject_unaligned_caches(pkg, fn):
    """The argument checks run before any device call: an unaligned K or V
    pointer (never dereferenced) is refused with T3B_ERR_ARG."""
    L = pkg.lib()
    f = getattr(L, fn)
    dummy = C.c_void_p(0x1000)
    for k, v in ((0x1008, 0x2000), (0x1000, 0x2002)):
        rc = f(dummy, C.c_void_p(k), C.c_void_p(v), 1, 16, 128, dummy, dummy, None)
        assert rc == -1                  # T3B_ERR_ARG
        assert "16-byte aligned" in pkg.last_error()


def test_gguf_roundtrip_keeps_converter_layout(pkg, tmp_path):
    g = pkg.t3_gguf
    hp = dict(g.T3_TURBO, n_layer=2, n_ctx=64, n_text_vocab=300)
    hp_, t = g.random_t3(hp, quant="q4_0", head_quant="f16", seed=3)
    path = tmp_path / "t3.gguf"
    g.write_gguf(path, hp_, t)
    hp2, t2 = g.read_gguf(path)
    assert hp2["eps"] == pytest.approx(hp_["eps"], rel=1e-7)   # stored as f32
    assert {k: v for k, v in hp2.items() if k != "eps"} == {k: v for k, v in hp_.items() if k != "eps"}
    assert set(t2) == set(t)
    for name, (ty, arr) in t.items():
        ty2, arr2 = t2[name]
        assert ty2 == int(ty), name
        np.testing.assert_array_equal(np.asarray(arr2).reshape(-1).view(np.uint8),
                                      np.ascontiguousarray(arr).reshape(-1).view(np.uint8))
    # GPT-2 Conv1D weights are stored transposed: ne0 = K (reduction axis)
    ty, arr = t2["model/h0/mlp/c_proj/w"]
    assert g.tensor_ne(ty, np.asarray(arr)) == [4096, 1024]
    ty, arr = t2["chatterbox/speech_head"]
    assert ty == 1 and g.tensor_ne(ty, np.asarray(arr)) == [1024, 6563]


def test_no_cpu_fallback_in_product():
    """The product package must not reach the oracle or any CPU compute
    path: it only talks to libt3b200.so."""
    pkg_dir = os.path.join(ROOT, "chatterbox.cpp_b200")
    for dirpath, _, files in os.walk(pkg_dir):
        for f in files:
            if f.endswith((".py", ".cu", ".cuh", ".cpp", ".h")):
                src = open(os.path.join(dirpath, f), errors="ignore").read()
                assert "oracle" not in src.replace("oracle/", "").lower() or f == "build.py", f
