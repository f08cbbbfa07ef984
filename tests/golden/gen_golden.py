"""Generates the committed golden vectors in tests/golden/.

Run in a container that holds the chatterbox.cpp tree (the reference
sampler is compiled from it by `make -C oracle ref`):

    T3B_REFERENCE_TREE=<chatterbox.cpp tree> python tests/golden/gen_golden.py

sampler_ref.json   sample_next_token_ex (the reference's own code, compiled
                   from src/main.cpp) on seeded synthetic logits: token and
                   number of mt19937 outputs consumed per case, plus whole
                   decode-loop sequences.
quant_ref.npz      gguf-py Q4_0/Q8_0 blocks of a seeded matrix and their
                   dequantisation (gguf-py's Q8_0 is documented bit-exact
                   with ggml-quants.c).
"""
import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(ROOT, "oracle"))
sys.path.insert(0, os.path.join(ROOT, "tests"))

import oracle  # noqa: E402
from conftest import synth_logits  # noqa: E402


def sampler_cases():
    rng = np.random.default_rng(20261201)
    cases = []
    for i in range(240):
        scale = [3.0, 1.0, 0.3, 10.0, 30.0][i % 5]
        kind = "rounded" if i % 9 == 0 else "normal"
        p = dict(top_k=1000, top_p=0.95, temp=0.8, repeat_penalty=1.2)
        m = i % 12
        if m == 1: p["temp"] = 0.0                       # greedy
        if m == 2: p["top_k"] = 0                        # top-k off
        if m == 3: p["top_p"] = 1.0                      # top-p off
        if m == 4: p["repeat_penalty"] = 1.0             # penalty off
        if m == 5: p.update(top_k=50, top_p=0.5)
        if m == 6: p.update(temp=1.0)                    # no scaling
        if m == 7: p.update(top_k=6563)                  # k == n: off
        if m == 8: p.update(top_k=1, top_p=0.9)
        if m == 9: p.update(temp=1.3, repeat_penalty=1.5)
        if m == 10: p.update(top_p=0.0)                  # keep the first
        if m == 11: p.update(top_k=7000, top_p=0.99, repeat_penalty=0.8)
        hist_len = int(rng.integers(0, 400))
        hist_seed = int(rng.integers(0, 2**31))
        mt_seed = int(rng.integers(0, 2**32))
        skip = int(rng.integers(0, 5000))
        lseed = 1000 + i
        logits = synth_logits(lseed, scale=scale, kind=kind)
        hist = np.random.default_rng(hist_seed).integers(-2, 6565, hist_len).astype(np.int32)
        tok, used = oracle.ref_sample(logits, p, mt_seed, skip, hist)
        w = oracle.mt19937_words(mt_seed, skip, 2)
        _, aux = oracle.sample(logits, p, w[0], w[1], hist=hist)
        cases.append(dict(logit_seed=lseed, scale=scale, kind=kind, params=p, hist_seed=hist_seed,
                          hist_len=hist_len, mt_seed=mt_seed, skip=skip, token=int(tok), used=int(used),
                          tie_at_cut=int(aux[2]), survivors_topk=int(aux[0]), survivors_topp=int(aux[1])))
    return cases


def sequences():
    out = []
    R = oracle.ref_lib()
    for j, (scale, p) in enumerate([(3.0, dict(top_k=1000, top_p=0.95, temp=0.8, repeat_penalty=1.2)),
                                     (1.0, dict(top_k=100, top_p=0.8, temp=1.0, repeat_penalty=1.3)),
                                     (0.5, dict(top_k=1000, top_p=0.95, temp=0.8, repeat_penalty=1.2))]):
        steps = 64
        logits = np.stack([synth_logits(50000 + 100 * j + s, scale=scale) for s in range(steps)])
        toks = np.zeros(steps, np.int32)
        R.ref_sample_sequence(np.ascontiguousarray(logits.ravel()), 6563, steps, p["top_k"], p["top_p"], p["temp"],
                              p["repeat_penalty"], 42 + j, toks)
        out.append(dict(first_seed=50000 + 100 * j, scale=scale, steps=steps, params=p, mt_seed=42 + j,
                        tokens=toks.tolist()))
    return out


def quant():
    import gguf
    rng = np.random.default_rng(7)
    w = (rng.standard_normal((8, 256)) * 0.02).astype(np.float32)
    q4 = gguf.quants.quantize(w, gguf.GGMLQuantizationType.Q4_0)
    q8 = gguf.quants.quantize(w, gguf.GGMLQuantizationType.Q8_0)
    d4 = gguf.quants.dequantize(q4, gguf.GGMLQuantizationType.Q4_0).astype(np.float32)
    d8 = gguf.quants.dequantize(q8, gguf.GGMLQuantizationType.Q8_0).astype(np.float32)
    x = rng.standard_normal(256).astype(np.float32)
    xq8 = gguf.quants.quantize(x[None], gguf.GGMLQuantizationType.Q8_0)
    np.savez(os.path.join(HERE, "quant_ref.npz"), w=w, q4=q4, q8=q8, d4=d4, d8=d8, x=x, xq8=xq8)


if __name__ == "__main__":
    tree = os.environ.get("T3B_REFERENCE_TREE", "")
    if not tree:
        sys.exit("set T3B_REFERENCE_TREE to the chatterbox.cpp source tree")
    oracle.build(ref=tree)
    data = dict(generator="tests/golden/gen_golden.py", reference="chatterbox.cpp src/main.cpp:726-801 "
                "sample_next_token_ex compiled by oracle/Makefile (target ref)",
                cases=sampler_cases(), sequences=sequences())
    with open(os.path.join(HERE, "sampler_ref.json"), "w") as f:
        json.dump(data, f, indent=0)
    quant()
    print("cases:", len(data["cases"]), "tie-at-cut:", sum(c["tie_at_cut"] for c in data["cases"]))
