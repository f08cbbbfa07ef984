"""T3 GGUF files: random-init writer and reader.

The tensor names, shapes, dtypes and metadata keys follow chatterbox.cpp's
converter (scripts/convert-t3-turbo-to-gguf.py: constants :18-27,
map_tensor_name :147-194, metadata :209-241, builtin voice :259-264) and the
keys load_model_gguf reads (src/chatterbox_t3_internal.h:32-42).  2-D
projection weights are stored transposed (ne0 = K, the reduction axis,
contiguous), and quantized with gguf-py exactly as the converter's --quant
does (add_maybe_quantized, :90-104).  No checkpoint is available offline, so
weights are random: 2-D weights and biases ~N(0, 0.02^2), LayerNorm g = 1,
b = 0, embeddings ~N(0, 0.02^2), speaker embedding ~N(0, 1), cond speech
tokens ~U[0, 6561).
"""
import numpy as np

import gguf

GGML_F32, GGML_F16, GGML_Q4_0, GGML_Q8_0 = 0, 1, 2, 8
_QT = {"q4_0": gguf.GGMLQuantizationType.Q4_0, "q8_0": gguf.GGMLQuantizationType.Q8_0}
_TYPE_ID = {"f16": GGML_F16, "q4_0": GGML_Q4_0, "q8_0": GGML_Q8_0}

# convert-t3-turbo-to-gguf.py:18-27
T3_TURBO = dict(n_text_vocab=50276, n_speech_vocab=6563, start_speech_token=6561, stop_speech_token=6562,
                speaker_embed_size=256, n_ctx=8196, n_embd=1024, n_head=16, n_layer=24, eps=1e-5,
                cond_prompt_len=62)

HP_KEYS = {  # chatterbox_t3_internal.h:32-42
    "n_text_vocab": "chatterbox.text_vocab_size", "n_speech_vocab": "chatterbox.speech_vocab_size",
    "start_speech_token": "chatterbox.start_speech_token", "stop_speech_token": "chatterbox.stop_speech_token",
    "speaker_embed_size": "chatterbox.speaker_embed_size", "eps": "chatterbox.layer_norm_eps",
    "cond_prompt_len": "chatterbox.cond_prompt_length", "n_ctx": "chatterbox.n_ctx", "n_embd": "chatterbox.n_embd",
    "n_head": "chatterbox.n_head", "n_layer": "chatterbox.n_layer",
}


def _quant(arr, quant):
    """arr: [N, K] float32 -> (ggml type id, raw bytes [N, K/32*block])."""
    if quant == "f16":
        return GGML_F16, arr.astype(np.float16)
    return _TYPE_ID[quant], gguf.quants.quantize(arr.astype(np.float32), _QT[quant])


def random_t3(hp=None, quant="q4_0", head_quant=None, seed=0, text_emb=True):
    """Random-init T3 tensors in GGUF layout.

    Returns (hp, tensors) with tensors = {name: (ggml_type, ndarray)} where
    the ndarray is the row-major GGUF payload (numpy shape = reversed ne).
    head_quant defaults to `quant` (as convert --quant does); pass "f16" for
    a requantize-gguf.py style file that keeps speech_head in f16.
    """
    hp = dict(T3_TURBO if hp is None else hp)
    rng = np.random.default_rng(seed)
    D, V, TV, S = hp["n_embd"], hp["n_speech_vocab"], hp["n_text_vocab"], hp["speaker_embed_size"]
    head_quant = quant if head_quant is None else head_quant

    def nrm(*shape, s=0.02):
        return (rng.standard_normal(shape, dtype=np.float32) * np.float32(s)).astype(np.float32)

    t = {}
    t["model/wpe"] = (GGML_F32, nrm(hp["n_ctx"], D))
    t["model/ln_f/g"] = (GGML_F32, np.ones(D, np.float32))
    t["model/ln_f/b"] = (GGML_F32, np.zeros(D, np.float32))
    t["chatterbox/text_emb"] = (GGML_F16, (nrm(TV, D) if text_emb else np.zeros((TV, D), np.float32)).astype(np.float16))
    t["chatterbox/speech_emb"] = (GGML_F16, nrm(V, D).astype(np.float16))
    t["chatterbox/speech_head"] = _quant(nrm(V, D), head_quant)
    t["chatterbox/speech_head_bias"] = (GGML_F32, nrm(V))
    t["chatterbox/cond_spkr/w"] = (GGML_F32, nrm(D, S))
    t["chatterbox/cond_spkr/b"] = (GGML_F32, nrm(D))
    t["chatterbox/builtin/speaker_emb"] = (GGML_F32, rng.standard_normal((1, S), dtype=np.float32))
    t["chatterbox/builtin/cond_prompt_speech_tokens"] = (
        gguf.GGMLQuantizationType.I32, rng.integers(0, hp["start_speech_token"], hp["cond_prompt_len"]).astype(np.int32))
    for i in range(hp["n_layer"]):
        p = f"model/h{i}"
        t[f"{p}/ln_1/g"] = (GGML_F32, np.ones(D, np.float32))
        t[f"{p}/ln_1/b"] = (GGML_F32, np.zeros(D, np.float32))
        t[f"{p}/ln_2/g"] = (GGML_F32, np.ones(D, np.float32))
        t[f"{p}/ln_2/b"] = (GGML_F32, np.zeros(D, np.float32))
        t[f"{p}/attn/c_attn/w"] = _quant(nrm(3 * D, D), quant)
        t[f"{p}/attn/c_attn/b"] = (GGML_F32, nrm(3 * D))
        t[f"{p}/attn/c_proj/w"] = _quant(nrm(D, D), quant)
        t[f"{p}/attn/c_proj/b"] = (GGML_F32, nrm(D))
        t[f"{p}/mlp/c_fc/w"] = _quant(nrm(4 * D, D), quant)
        t[f"{p}/mlp/c_fc/b"] = (GGML_F32, nrm(4 * D))
        t[f"{p}/mlp/c_proj/w"] = _quant(nrm(D, 4 * D), quant)
        t[f"{p}/mlp/c_proj/b"] = (GGML_F32, nrm(D))
    return hp, t


def write_gguf(path, hp, tensors, quant_name="q4_0"):
    """Write a T3 GGUF with the converter's metadata keys."""
    w = gguf.GGUFWriter(str(path), "chatterbox")
    w.add_name("Chatterbox Turbo T3 (random init)")
    w.add_context_length(hp["n_ctx"])
    w.add_embedding_length(hp["n_embd"])
    w.add_block_count(hp["n_layer"])
    w.add_head_count(hp["n_head"])
    w.add_vocab_size(hp["n_text_vocab"])
    for k, key in HP_KEYS.items():
        if k == "eps":
            w.add_float32(key, float(hp[k]))
        else:
            w.add_uint32(key, int(hp[k]))
    w.add_string("chatterbox.variant", "t3_turbo")
    w.add_string("chatterbox.quantization", quant_name)
    for name, (ty, arr) in tensors.items():
        if ty in (GGML_Q4_0, GGML_Q8_0):
            qt = gguf.GGMLQuantizationType(ty)
            w.add_tensor(name, arr, raw_shape=arr.shape, raw_dtype=qt)
        else:
            w.add_tensor(name, arr)
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.write_tensors_to_file()
    w.close()


def read_gguf(path):
    """Read a T3 GGUF: (hp, tensors) like random_t3; arrays are memory maps."""
    r = gguf.GGUFReader(str(path))
    hp = {}
    for k, key in HP_KEYS.items():
        f = r.fields[key]
        v = f.parts[f.data[0]][0]
        hp[k] = float(v) if k == "eps" else int(v)
    tensors = {}
    for t in r.tensors:
        tensors[t.name] = (int(t.tensor_type), t.data)
    return hp, tensors


def tensor_ne(ty, arr):
    """ggml ne[] of a GGUF payload array (ne0 = innermost elements)."""
    shape = list(arr.shape)[::-1]
    if ty == GGML_Q4_0:
        shape[0] = shape[0] // 18 * 32
    elif ty == GGML_Q8_0:
        shape[0] = shape[0] // 34 * 32
    return shape
