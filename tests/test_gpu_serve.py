"""Continuous batching (t3b_serve_*) against one-utterance-at-a-time runs.

The scheduler steps every admitted stream in one batch and refills freed
slots from its queue.  Each utterance must come out exactly as chatterbox.cpp's
per-utterance loop would produce it: run_t3 (src/chatterbox_engine.cpp:
334-358) for plain requests, and the CLI's early-stop retry
(src/chatterbox_cli.cpp:1615-1674) when min_tokens is set.  The reference
run here is the device decode loop of one stream on the same kernels
(graph path), whose rows are computed independently of the batch size.
"""
import os

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")


def _text(seed, n):
    return np.random.default_rng(seed).integers(0, 50257, n).astype(np.int32)


def _single(pkg, m, text, params, seed, n_predict, discard=0):
    """run_t3 for one utterance on stream 0 (graph path); stop token popped."""
    os.environ["T3B_NO_MEGAKERNEL"] = "1"
    try:
        m.prefill(0, text)
        m.set_rng(0, pkg.T3B_RNG_MT19937, seed, discard)
        toks = m.decode([params], n_predict, streams=[0])[0].tolist()
    finally:
        os.environ.pop("T3B_NO_MEGAKERNEL", None)
    stopped = bool(toks) and toks[-1] == m.hp["stop_speech_token"]
    if stopped:
        toks.pop()
    return toks, stopped


def _drain(m, ids):
    for _ in range(10000):
        act, q = m.serve_run(64)
        if act == 0 and q == 0:
            break
    return [m.serve_result(i) for i in ids]


@pytest.mark.parametrize("cfg", [False, True])
def test_serve_matches_one_utterance_at_a_time(pkg, cfg):
    hp = dict(pkg.t3_gguf.T3_TURBO, n_layer=2)
    hp, t = pkg.t3_gguf.random_t3(hp, quant="q4_0", seed=51)
    m = pkg.T3Model(hp, t)
    try:
        reqs = [(_text(60 + i, 10 + 7 * i), 1000 + i, 12 + 5 * i) for i in range(5)]
        params = pkg.SampleParams.make(top_k=1000, top_p=0.95, temp=0.8, repeat_penalty=1.2,
                                       cfg_weight=0.5 if cfg else 0.0)
        m.alloc_streams(1, 256, cfg=cfg)
        want = [_single(pkg, m, txt, params, seed, n)[0] for txt, seed, n in reqs]
        m.alloc_streams(2, 256, cfg=cfg)                  # two slots for five requests
        ids = [m.serve_submit(txt, params, seed=seed, n_predict=n) for txt, seed, n in reqs]
        got = _drain(m, ids)
        for i, (toks, att) in enumerate(got):
            assert toks is not None and att == 1
            assert toks.tolist() == want[i], i
    finally:
        m.close()


def test_serve_early_stop_retry_as_the_cli(pkg):
    """A head bias that makes the stop token likely: short stop-token endings
    are replayed with the RNG advanced by attempt * 1009 draws, up to 3
    retries, keeping the longest attempt when all are short."""
    hp = dict(pkg.t3_gguf.T3_TURBO, n_layer=1)
    hp, t = pkg.t3_gguf.random_t3(hp, quant="q4_0", seed=52)
    ty, b = t["chatterbox/speech_head_bias"]
    b = b.copy()
    b[hp["stop_speech_token"]] += 5.0
    t["chatterbox/speech_head_bias"] = (ty, b)
    m = pkg.T3Model(hp, t)
    try:
        params = pkg.SampleParams.make(top_k=1000, top_p=0.95, temp=0.8, repeat_penalty=1.2)
        reqs = [(_text(70 + i, 6), 2000 + i) for i in range(8)]
        n_predict, min_tokens, retries = 40, 12, 3
        m.alloc_streams(1, 256)
        want = []
        for txt, seed in reqs:
            best = []
            for a in range(retries + 1):
                toks, stopped = _single(pkg, m, txt, params, seed, n_predict, discard=a * 1009)
                if len(toks) > len(best):
                    best = toks
                if not stopped or len(toks) >= min_tokens:
                    want.append((toks, a + 1))
                    break
            else:
                want.append((best, retries + 1))
        assert any(w[1] > 1 for w in want), "bias too weak: no retry exercised"
        m.alloc_streams(3, 256)
        ids = [m.serve_submit(txt, params, seed=seed, n_predict=n_predict, min_tokens=min_tokens,
                              max_retries=retries) for txt, seed in reqs]
        got = _drain(m, ids)
        for i, (toks, att) in enumerate(got):
            assert toks.tolist() == want[i][0], (i, att, want[i][1])
            assert att == want[i][1], i
    finally:
        m.close()


def test_serve_bad_request_does_not_stop_the_others(pkg):
    hp = dict(pkg.t3_gguf.T3_TURBO, n_layer=1)
    hp, t = pkg.t3_gguf.random_t3(hp, quant="q4_0", seed=53)
    m = pkg.T3Model(hp, t)
    try:
        m.alloc_streams(2, 128)
        params = pkg.SampleParams.make()
        ok = m.serve_submit(_text(1, 10), params, seed=1, n_predict=8)
        bad = m.serve_submit(_text(2, 200), params, seed=2, n_predict=8)   # prompt longer than the context
        ok2 = m.serve_submit(_text(3, 10), params, seed=3, n_predict=8)
        for _ in range(100):
            act, q = m.serve_run(16)
            if act == 0 and q == 0:
                break
        assert m.serve_result(ok)[0] is not None and m.serve_result(ok2)[0] is not None
        with pytest.raises(pkg.T3BError):
            m.serve_result(bad)
    finally:
        m.close()
