"""The C++ mirror of chatterbox.cpp's T3 API (include/t3b200_dropin.hpp):
tests/cpp/t3_dropin_main.cpp runs Engine::Impl::run_t3's loop (eval_prompt,
then eval_step + sample_next_token_ex with a std::mt19937) against a GGUF
file written with the converter's layout."""
import os
import subprocess

import numpy as np
import pytest

from conftest import PKG_DIR, gpu_available, load_package

EXE = os.path.join(PKG_DIR, "_build", "t3_dropin_main")


@pytest.fixture(scope="module")
def gguf_path(tmp_path_factory):
    pkg = load_package()
    if not os.path.exists(EXE):
        import importlib.util
        spec = importlib.util.spec_from_file_location("t3b_build", os.path.join(PKG_DIR, "build.py"))
        b = importlib.util.module_from_spec(spec)
        spec.loader.exec_module(b)
        b.build_dropin()
    hp = dict(pkg.t3_gguf.T3_TURBO, n_layer=2)
    hp, t = pkg.t3_gguf.random_t3(hp, quant="q4_0", seed=4)
    path = tmp_path_factory.mktemp("gguf") / "t3_q4_0.gguf"
    pkg.t3_gguf.write_gguf(path, hp, t)
    return str(path)


TEXT = [int(x) for x in np.random.default_rng(3).integers(0, 50257, 24)]


def _run(path, seed, n_predict):
    return subprocess.run([EXE, path, str(seed), str(n_predict), str(len(TEXT))] + [str(x) for x in TEXT],
                          capture_output=True, text=True, timeout=300)


@pytest.mark.skipif(gpu_available(), reason="checks the no-device error path")
def test_dropin_parses_gguf_and_reports_missing_device(gguf_path):
    r = _run(gguf_path, 0, 4)
    assert r.returncode == 1
    assert "load_model_gguf: t3b_create" in r.stderr          # parsing succeeded, device creation failed
    assert "missing GGUF key" not in r.stderr


def test_dropin_rejects_non_gguf(tmp_path):
    if not os.path.exists(EXE):
        pytest.skip("drop-in test program not built")
    bad = tmp_path / "bad.gguf"
    bad.write_bytes(b"not a gguf file at all")
    r = subprocess.run([EXE, str(bad), "0", "1", "1", "5"], capture_output=True, text=True, timeout=60)
    assert r.returncode == 1 and "not a GGUF file" in r.stderr


@pytest.mark.gpu
def test_dropin_loop_matches_device_decode(gguf_path):
    """Same GGUF, seed and prompt: the C++ per-step loop (host logits, host
    std::mt19937 mirrored to the device) and t3b_decode (everything on the
    device) produce identical token streams."""
    pkg = load_package()
    for seed in (0, 7):
        r = _run(gguf_path, seed, 40)
        assert r.returncode == 0, r.stderr
        fields = r.stdout.split()
        P = int(fields[1])
        toks = [int(x) for x in fields[3:]]
        m = pkg.load_model_gguf(gguf_path)
        m.alloc_streams(1, 512)
        P2, _ = m.prefill(0, np.array(TEXT, np.int32))
        m.set_rng(0, pkg.T3B_RNG_MT19937, seed, 0)
        dev = m.decode([pkg.SampleParams.make()], 40)[0].tolist()
        if dev and dev[-1] == m.hp["stop_speech_token"]:
            dev.pop()
        m.close()
        assert P == P2 == 1 + 62 + len(TEXT) + 1
        assert toks == dev, seed
