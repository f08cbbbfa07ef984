"""ctypes access to the CPU oracle (liboracle.so) and the reference sampler
(_ref/libref_sampler.so).

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and
bench.py's cpu_baseline / --impl reference legs.  The product
(chatterbox.cpp_b200/) never imports this module.
"""
import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB = os.path.join(HERE, "liboracle.so")
REF_LIB = os.path.join(HERE, "_ref", "libref_sampler.so")
REF_TREE = os.environ.get("T3B_REFERENCE_TREE", "")

_lib = None
_ref = None

F32P = np.ctypeslib.ndpointer(np.float32, flags="C_CONTIGUOUS")
I32P = np.ctypeslib.ndpointer(np.int32, flags="C_CONTIGUOUS")
U32P = np.ctypeslib.ndpointer(np.uint32, flags="C_CONTIGUOUS")


def build(ref=None):
    """Compile liboracle.so, and the reference sampler when a reference tree
    is available: ref = the tree's path, None = $T3B_REFERENCE_TREE when it
    is set, False = never."""
    subprocess.check_call(["make", "-s", "-C", HERE, "liboracle.so"])
    tree = ref if isinstance(ref, str) else (REF_TREE if ref is not False else "")
    if tree and os.path.isfile(os.path.join(tree, "src", "main.cpp")):
        subprocess.check_call(["make", "-s", "-C", HERE, "ref", f"REF={tree}"])


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB):
            build(ref=False)
        L = C.CDLL(LIB)
        L.orc_set_threads.argtypes = [C.c_int]
        L.orc_expf_batch.argtypes = [F32P, F32P, C.c_int64]
        L.orc_f32_to_f16.restype = C.c_uint16
        L.orc_f32_to_f16.argtypes = [C.c_float]
        L.orc_dequant_rows.argtypes = [C.c_int, C.c_void_p, C.c_int, C.c_int, F32P]
        L.orc_quantize_q8_row.argtypes = [F32P, C.c_int, C.c_void_p, F32P]
        L.orc_matvec.argtypes = [C.c_int, C.c_void_p, C.c_int, C.c_int, F32P, C.c_int, C.c_void_p, F32P, C.c_int]
        L.orc_layernorm.argtypes = [F32P, C.c_int, F32P, F32P, C.c_float, F32P]
        L.orc_gelu.restype = C.c_float
        L.orc_gelu.argtypes = [C.c_float, C.c_int]
        L.orc_philox4x32_10.argtypes = [U32P, U32P, U32P]
        L.orc_canonical53.restype = C.c_double
        L.orc_canonical53.argtypes = [C.c_uint32, C.c_uint32]
        L.orc_mt19937_words.argtypes = [C.c_uint32, C.c_uint64, C.c_int, U32P]
        L.orc_sample.restype = C.c_int
        L.orc_sample.argtypes = [F32P, C.c_void_p, C.c_int, C.c_void_p, C.c_int, C.c_int32, C.c_float, C.c_float,
                                 C.c_float, C.c_float, C.c_float, C.c_uint32, C.c_uint32, I32P]
        L.orc_model_new.restype = C.c_void_p
        L.orc_model_new.argtypes = [C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, C.c_float]
        L.orc_model_free.argtypes = [C.c_void_p]
        L.orc_model_config.argtypes = [C.c_void_p, C.c_int, C.c_int, C.c_int]
        L.orc_model_set.restype = C.c_int
        L.orc_model_set.argtypes = [C.c_void_p, C.c_char_p, C.c_int, C.c_void_p, C.c_int64]
        L.orc_prompt.restype = C.c_int
        L.orc_prompt.argtypes = [C.c_void_p, C.c_void_p, C.c_int, C.c_void_p, C.c_int, C.c_void_p, C.c_int, C.c_int, F32P]
        L.orc_step.restype = C.c_int
        L.orc_step.argtypes = [C.c_void_p, C.c_int, C.c_int32, F32P]
        L.orc_step_trace.restype = C.c_int
        L.orc_step_trace.argtypes = [C.c_void_p, C.c_int, C.c_int32, F32P, F32P]
        L.orc_model_kv.argtypes = [C.c_void_p, C.c_int, C.c_int, C.c_int, F32P]
        _lib = L
    return _lib


def ref_lib():
    """The reference's own sampler, or None when it was not built here."""
    global _ref
    if _ref is None:
        if not os.path.exists(REF_LIB):
            return None
        R = C.CDLL(REF_LIB)
        R.ref_sample_next_token_ex.restype = C.c_int
        R.ref_sample_next_token_ex.argtypes = [F32P, C.c_int, C.c_void_p, C.c_int, C.c_int32, C.c_float, C.c_float,
                                               C.c_float, C.c_uint32, C.c_uint64, C.POINTER(C.c_int)]
        R.ref_sample_sequence.argtypes = [F32P, C.c_int, C.c_int, C.c_int32, C.c_float, C.c_float, C.c_float,
                                          C.c_uint32, I32P]
        _ref = R
    return _ref


def set_threads(n):
    lib().orc_set_threads(int(n))


def expf_batch(x):
    x = np.ascontiguousarray(x, np.float32)
    out = np.empty_like(x)
    lib().orc_expf_batch(x, out, x.size)
    return out


def mt19937_words(seed, skip, n):
    out = np.zeros(n, np.uint32)
    lib().orc_mt19937_words(seed, skip, n, out)
    return out


def philox(ctr, key):
    out = np.zeros(4, np.uint32)
    lib().orc_philox4x32_10(np.asarray(ctr, np.uint32), np.asarray(key, np.uint32), out)
    return out


def sample(cond, params, x1, x2, uncond=None, hist=None):
    """Oracle sampler.  params: dict(top_k, top_p, temp, repeat_penalty,
    min_p, cfg_weight).  Returns (token, aux[3])."""
    cond = np.ascontiguousarray(cond, np.float32)
    unc = None if uncond is None else np.ascontiguousarray(uncond, np.float32)
    h = np.zeros(0, np.int32) if hist is None else np.ascontiguousarray(hist, np.int32)
    aux = np.zeros(3, np.int32)
    t = lib().orc_sample(cond, unc.ctypes.data if unc is not None else None, cond.size,
                         h.ctypes.data if h.size else None, h.size,
                         int(params.get("top_k", 1000)), float(params.get("top_p", 0.95)), float(params.get("temp", 0.8)),
                         float(params.get("repeat_penalty", 1.2)), float(params.get("min_p", 0.0)),
                         float(params.get("cfg_weight", 0.0)), int(x1), int(x2), aux)
    return t, aux


def ref_sample(logits, params, seed, skip=0, hist=None):
    """Reference sample_next_token_ex; returns (token, engine outputs used)."""
    R = ref_lib()
    if R is None:
        raise RuntimeError("reference sampler not built (needs the reference tree)")
    l = np.ascontiguousarray(logits, np.float32)
    h = np.zeros(0, np.int32) if hist is None else np.ascontiguousarray(hist, np.int32)
    used = C.c_int(0)
    t = R.ref_sample_next_token_ex(l, l.size, h.ctypes.data if h.size else None, h.size, int(params.get("top_k", 1000)),
                                   float(params.get("top_p", 0.95)), float(params.get("temp", 0.8)),
                                   float(params.get("repeat_penalty", 1.2)), int(seed), int(skip), C.byref(used))
    return t, used.value


class Model:
    """Oracle T3 model bound to a dict of GGUF tensors {name: (type, ndarray)}."""

    def __init__(self, hp, tensors, max_ctx, gemv_mode=1, gelu_f16=1, kv_f16=0):
        L = lib()
        self.hp = hp
        self.h = L.orc_model_new(hp["n_layer"], hp["n_embd"], hp["n_head"], max_ctx, hp["n_speech_vocab"],
                                 hp["n_text_vocab"], hp["speaker_embed_size"], hp["eps"])
        self._keep = []
        for name, (ty, arr) in tensors.items():
            a = np.ascontiguousarray(arr)
            self._keep.append(a)
            L.orc_model_set(self.h, name.encode(), int(ty), a.ctypes.data, int(a.size))
        L.orc_model_config(self.h, gemv_mode, gelu_f16, kv_f16)

    def prompt(self, text, cond=None, spk=None, uncond=False):
        L = lib()
        V = self.hp["n_speech_vocab"]
        out = np.zeros(V, np.float32)
        t = np.ascontiguousarray(text, np.int32)
        c = None if cond is None else np.ascontiguousarray(cond, np.int32)
        s = None if spk is None else np.ascontiguousarray(spk, np.float32)
        P = L.orc_prompt(self.h, t.ctypes.data, t.size, c.ctypes.data if c is not None else None,
                         0 if c is None else c.size, s.ctypes.data if s is not None else None,
                         self.hp["start_speech_token"], 1 if uncond else 0, out)
        if P < 0:
            raise ValueError("prompt too long")
        return P, out

    def step(self, n_past, token):
        out = np.zeros(self.hp["n_speech_vocab"], np.float32)
        if lib().orc_step(self.h, n_past, token, out) != 0:
            raise ValueError("bad step")
        return out

    def step_trace(self, n_past, token):
        """step() plus the residual stream: (logits, hidden [n_layer + 1, n_embd])."""
        out = np.zeros(self.hp["n_speech_vocab"], np.float32)
        hid = np.zeros((self.hp["n_layer"] + 1, self.hp["n_embd"]), np.float32)
        if lib().orc_step_trace(self.h, n_past, token, out, hid) != 0:
            raise ValueError("bad step")
        return out, hid

    def kv(self, layer, which, n_pos):
        out = np.zeros(self.hp["n_head"] * n_pos * (self.hp["n_embd"] // self.hp["n_head"]), np.float32)
        lib().orc_model_kv(self.h, layer, which, n_pos, out)
        return out

    def __del__(self):
        try:
            lib().orc_model_free(self.h)
        except Exception:
            pass
