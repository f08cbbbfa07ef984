"""chatterbox.cpp_b200 — B200-native T3 decode step for chatterbox.cpp.

Python host side over the C ABI of libt3b200.so (include/t3b200.h).  The
names mirror chatterbox.cpp's T3 internal API (src/chatterbox_t3_internal.h:
120-148): load_model_gguf, eval_prompt, eval_step, sample_next_token_ex,
plus the batched / device-loop extensions of the C ABI.

There is no CPU fallback: importing works without a GPU (so the library can
be inspected and its symbols checked), but every compute call goes through
libt3b200.so and raises T3BError if the library or a device is missing.
"""
import ctypes as C
import os

import numpy as np

from . import sharding, t3_gguf

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libt3b200.so")

T3B_OK = 0
T3B_RNG_MT19937, T3B_RNG_PHILOX = 0, 1
ERRORS = {-1: "ARG", -2: "CUDA", -3: "OOM", -4: "STATE", -5: "DEVICE", -6: "CANCELLED", -7: "TIMEOUT"}

# every symbol include/t3b200.h declares
EXPORTS = [
    "t3b_create", "t3b_destroy", "t3b_last_error", "t3b_stream_alloc", "t3b_prefill", "t3b_step", "t3b_sample",
    "t3b_set_rng", "t3b_set_rng_state", "t3b_get_rng_state", "t3b_set_history", "t3b_decode", "t3b_cancel",
    "t3b_last_device_ms", "t3b_stream_handle", "t3b_trace_logits", "t3b_get_logits_trace", "t3b_op_row_bytes", "t3b_op_repack", "t3b_op_gemv", "t3b_op_attention",
    "t3b_op_sample_philox", "t3b_expf_fixup_count", "t3b_op_expf", "t3b_op_attention_noalloc",
    "t3b_trace_hidden", "t3b_get_hidden_trace", "t3b_set_wait_limit", "t3b_launch_count", "t3b_s3gen_tokens",
    "t3b_op_check", "t3b_op_attention_prompt", "t3b_serve_submit", "t3b_serve_run", "t3b_serve_result", "t3b_serve_stats",
]


class T3BError(RuntimeError):
    def __init__(self, code, msg):
        super().__init__(f"t3b error {code} ({ERRORS.get(code, '?')}): {msg}")
        self.code = code


class Tensor(C.Structure):
    _fields_ = [("name", C.c_char_p), ("type", C.c_int32), ("n_dims", C.c_int32), ("ne", C.c_int64 * 4),
                ("data", C.c_void_p)]


class HParams(C.Structure):
    _fields_ = [(k, C.c_int32) for k in ("n_text_vocab", "n_speech_vocab", "start_speech_token", "stop_speech_token",
                                          "n_ctx", "n_embd", "n_head", "n_layer", "speaker_embed_size",
                                          "cond_prompt_len")] + [("eps", C.c_float)]


class ModelDesc(C.Structure):
    _fields_ = [("hp", HParams), ("n_tensors", C.c_int32), ("tensors", C.POINTER(Tensor))]


class SampleParams(C.Structure):
    """chatterbox_sampling_params (+ min_p, cfg_weight extensions, 0 = off)."""
    _fields_ = [("top_k", C.c_int32), ("top_p", C.c_float), ("temp", C.c_float), ("repeat_penalty", C.c_float),
                ("min_p", C.c_float), ("cfg_weight", C.c_float)]

    @classmethod
    def make(cls, top_k=1000, top_p=0.95, temp=0.8, repeat_penalty=1.2, min_p=0.0, cfg_weight=0.0):
        return cls(int(top_k), float(top_p), float(temp), float(repeat_penalty), float(min_p), float(cfg_weight))


class Request(C.Structure):
    """t3b_request: one utterance for the continuous-batching scheduler."""
    _fields_ = [("text", C.c_void_p), ("n_text", C.c_int32), ("cond_tokens", C.c_void_p), ("n_cond", C.c_int32),
                ("spk_emb", C.c_void_p), ("params", SampleParams), ("rng_mode", C.c_int32), ("seed", C.c_uint64),
                ("n_predict", C.c_int32), ("min_tokens", C.c_int32), ("max_retries", C.c_int32)]


_lib = None


def lib():
    """Load libt3b200.so (raises if it was not built)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise T3BError(-4, f"{LIB_PATH} is missing: run chatterbox.cpp_b200/build.py")
        L = C.CDLL(LIB_PATH)
        vp, i32p = C.c_void_p, C.POINTER(C.c_int32)
        sig = {
            "t3b_create": (vp, [C.c_int, C.POINTER(ModelDesc)]),
            "t3b_destroy": (None, [vp]),
            "t3b_last_error": (C.c_char_p, [vp]),
            "t3b_stream_alloc": (C.c_int, [vp, C.c_int, C.c_int, C.c_int]),
            "t3b_prefill": (C.c_int, [vp, C.c_int, vp, C.c_int, vp, C.c_int, vp, vp, i32p]),
            "t3b_step": (C.c_int, [vp, C.c_int, vp, vp, vp, vp]),
            "t3b_sample": (C.c_int, [vp, C.c_int, vp, vp, vp, vp]),
            "t3b_set_rng": (C.c_int, [vp, C.c_int, C.c_int, C.c_uint64, C.c_uint64]),
            "t3b_set_rng_state": (C.c_int, [vp, C.c_int, vp]),
            "t3b_get_rng_state": (C.c_int, [vp, C.c_int, vp]),
            "t3b_set_history": (C.c_int, [vp, C.c_int, vp, C.c_int]),
            "t3b_decode": (C.c_int, [vp, C.c_int, vp, vp, C.c_int, C.c_int, vp, vp]),
            "t3b_cancel": (None, [vp]),
            "t3b_last_device_ms": (C.c_float, [vp]),
            "t3b_stream_handle": (vp, [vp]),
            "t3b_trace_logits": (C.c_int, [vp, C.c_int]),
            "t3b_get_logits_trace": (C.c_int, [vp, vp, C.c_int]),
            "t3b_op_row_bytes": (C.c_size_t, [C.c_int, C.c_int]),
            "t3b_op_repack": (C.c_int, [C.c_int, vp, C.c_int, C.c_int, vp]),
            "t3b_op_gemv": (C.c_int, [C.c_int, vp, C.c_int, C.c_int, vp, C.c_int, vp, vp, C.c_float, vp, vp, C.c_int,
                                      vp, vp]),
            "t3b_op_attention": (C.c_int, [vp, vp, vp, C.c_int, C.c_int, C.c_int, vp, vp, vp]),
            "t3b_op_attention_noalloc": (C.c_int, [vp, vp, vp, C.c_int, C.c_int, C.c_int, vp, vp, vp]),
            "t3b_op_sample_philox": (C.c_int, [vp, vp, C.c_int, C.c_int, vp, vp, C.c_int, vp, vp, vp, vp, vp]),
            "t3b_expf_fixup_count": (C.c_int, []),
            "t3b_op_expf": (C.c_int, [vp, vp, C.c_int, vp]),
            "t3b_trace_hidden": (C.c_int, [vp, C.c_int]),
            "t3b_get_hidden_trace": (C.c_int, [vp, vp]),
            "t3b_set_wait_limit": (C.c_int, [vp, C.c_uint]),
            "t3b_launch_count": (C.c_uint64, [vp]),
            "t3b_s3gen_tokens": (C.c_int, [vp, C.c_int, vp, C.c_int, vp, C.c_int, vp]),
            "t3b_op_check": (C.c_int, [vp]),
            "t3b_op_attention_prompt": (C.c_int, [vp, vp, vp, C.c_int, C.c_int, C.c_int, vp, vp, vp]),
            "t3b_serve_submit": (C.c_int, [vp, C.POINTER(Request)]),
            "t3b_serve_run": (C.c_int, [vp, C.c_int, i32p, i32p]),
            "t3b_serve_result": (C.c_int, [vp, C.c_int, vp, C.c_int, i32p, i32p]),
            "t3b_serve_stats": (C.c_int, [vp, C.POINTER(C.c_longlong), C.POINTER(C.c_double)]),
        }
        for name, (res, args) in sig.items():
            f = getattr(L, name)
            f.restype = res
            f.argtypes = args
        _lib = L
    return _lib


def last_error(ctx=None):
    m = lib().t3b_last_error(ctx)
    return m.decode() if m else ""


def check(rc, ctx=None):
    if rc != T3B_OK:
        raise T3BError(rc, last_error(ctx))
    return rc


def _ptr(a):
    return None if a is None else a.ctypes.data


class T3Model:
    """A T3 model on one GPU: the device side of chatterbox_model.

    tensors: {name: (ggml_type, ndarray)} as t3_gguf.random_t3 / read_gguf
    return them.  The host arrays may be released after construction.
    """

    def __init__(self, hp, tensors, device=0):
        self.hp = dict(hp)
        names, descs = [], []
        keep = []
        for name, (ty, arr) in tensors.items():
            a = np.ascontiguousarray(arr)
            keep.append(a)
            ne = t3_gguf.tensor_ne(ty, a) if ty in (0, 1, 2, 8) else list(a.shape)[::-1]
            t = Tensor()
            nb = name.encode()
            names.append(nb)
            t.name = nb
            t.type = int(ty)
            t.n_dims = len(ne)
            for i in range(4):
                t.ne[i] = ne[i] if i < len(ne) else 1
            t.data = a.ctypes.data
            descs.append(t)
        arr_t = (Tensor * len(descs))(*descs)
        hpc = HParams(*[int(self.hp[k]) for k in ("n_text_vocab", "n_speech_vocab", "start_speech_token",
                                                   "stop_speech_token", "n_ctx", "n_embd", "n_head", "n_layer",
                                                   "speaker_embed_size", "cond_prompt_len")], float(self.hp["eps"]))
        desc = ModelDesc(hpc, len(descs), arr_t)
        self.ctx = lib().t3b_create(int(device), C.byref(desc))
        if not self.ctx:
            raise T3BError(-1, last_error(None))
        self.V = self.hp["n_speech_vocab"]
        self.rps = 1
        self.n_streams = 0

    # ---------------- streams / reference-API mirror ----------------
    def alloc_streams(self, n_streams, max_ctx, cfg=False):
        check(lib().t3b_stream_alloc(self.ctx, n_streams, max_ctx, 1 if cfg else 0), self.ctx)
        self.rps = 2 if cfg else 1
        self.n_streams = n_streams

    def prefill(self, stream, text, cond=None, spk=None):
        """eval_prompt: returns (prompt_len, logits [rps, V])."""
        t = np.ascontiguousarray(text, np.int32)
        c = None if cond is None else np.ascontiguousarray(cond, np.int32)
        s = None if spk is None else np.ascontiguousarray(spk, np.float32)
        out = np.zeros((self.rps, self.V), np.float32)
        P = C.c_int32(0)
        check(lib().t3b_prefill(self.ctx, stream, _ptr(t), t.size, _ptr(c), 0 if c is None else c.size, _ptr(s),
                                _ptr(out), C.byref(P)), self.ctx)
        return P.value, out

    def step(self, tokens, streams=None, n_past=None, want_logits=True):
        """eval_step for len(tokens) streams: logits [n, rps, V] (or None)."""
        tok = np.ascontiguousarray(tokens, np.int32)
        n = tok.size
        st = None if streams is None else np.ascontiguousarray(streams, np.int32)
        np_ = None if n_past is None else np.ascontiguousarray(n_past, np.int32)
        out = np.zeros((n, self.rps, self.V), np.float32) if want_logits else None
        check(lib().t3b_step(self.ctx, n, _ptr(st), _ptr(tok), _ptr(np_), _ptr(out)), self.ctx)
        return out

    def sample(self, params, streams=None, logits=None, n=None):
        """sample_next_token_ex on the device; params: list of SampleParams."""
        if isinstance(params, SampleParams):
            params = [params]
        n = len(params) if n is None else n
        pa = (SampleParams * n)(*params)
        st = None if streams is None else np.ascontiguousarray(streams, np.int32)
        lg = None if logits is None else np.ascontiguousarray(logits, np.float32)
        out = np.zeros(n, np.int32)
        check(lib().t3b_sample(self.ctx, n, _ptr(st), C.cast(pa, C.c_void_p), _ptr(lg), _ptr(out)), self.ctx)
        return out

    def set_rng(self, stream, mode, seed, discard=0):
        check(lib().t3b_set_rng(self.ctx, stream, mode, seed, discard), self.ctx)

    def set_rng_state(self, stream, words625):
        w = np.ascontiguousarray(words625, np.uint32)
        check(lib().t3b_set_rng_state(self.ctx, stream, _ptr(w)), self.ctx)

    def get_rng_state(self, stream):
        w = np.zeros(625, np.uint32)
        check(lib().t3b_get_rng_state(self.ctx, stream, _ptr(w)), self.ctx)
        return w

    def set_history(self, stream, tokens):
        t = np.ascontiguousarray(tokens, np.int32)
        check(lib().t3b_set_history(self.ctx, stream, _ptr(t) if t.size else None, t.size), self.ctx)

    def decode(self, params, max_steps, streams=None, ignore_stop=False):
        """Device-side decode loop; returns a list of token arrays."""
        if isinstance(params, SampleParams):
            params = [params]
        n = len(params)
        pa = (SampleParams * n)(*params)
        st = None if streams is None else np.ascontiguousarray(streams, np.int32)
        out = np.zeros((n, max_steps + 1), np.int32)
        cnt = np.zeros(n, np.int32)
        check(lib().t3b_decode(self.ctx, n, _ptr(st), C.cast(pa, C.c_void_p), max_steps, 1 if ignore_stop else 0,
                               _ptr(out), _ptr(cnt)), self.ctx)
        return [out[i, :cnt[i]].copy() for i in range(n)]

    def trace_logits(self, max_steps):
        """Record the logits every decode step samples from (debug)."""
        check(lib().t3b_trace_logits(self.ctx, max_steps), self.ctx)

    def logits_trace(self, n):
        out = np.zeros((n, self.V), np.float32)
        check(lib().t3b_get_logits_trace(self.ctx, _ptr(out), n), self.ctx)
        return out

    def trace_hidden(self, on=True):
        """Record the residual stream of the next step's first row (embedding
        and every layer's output)."""
        check(lib().t3b_trace_hidden(self.ctx, 1 if on else 0), self.ctx)

    def hidden_trace(self):
        out = np.zeros((self.hp["n_layer"] + 1, self.hp["n_embd"]), np.float32)
        check(lib().t3b_get_hidden_trace(self.ctx, _ptr(out)), self.ctx)
        return out

    def set_wait_limit(self, polls):
        """Polls before a persistent-kernel wait gives up (0 = default)."""
        check(lib().t3b_set_wait_limit(self.ctx, int(polls)), self.ctx)

    def launch_count(self):
        return int(lib().t3b_launch_count(self.ctx))

    def s3gen_tokens(self, stream, tokens_dev_ptr, cap, n_dev_ptr, append_silence=True, consumer_stream=None):
        """S3Gen hand-off: the stream's speech tokens into a device buffer."""
        check(lib().t3b_s3gen_tokens(self.ctx, stream, tokens_dev_ptr, int(cap), n_dev_ptr,
                                     1 if append_silence else 0, consumer_stream), self.ctx)

    # ---------------- continuous batching ----------------
    def serve_submit(self, text, params, seed=0, n_predict=1000, min_tokens=0, max_retries=0,
                     rng_mode=T3B_RNG_MT19937, cond=None, spk=None):
        """Queue one utterance; returns its request id."""
        t = np.ascontiguousarray(text, np.int32)
        c = None if cond is None else np.ascontiguousarray(cond, np.int32)
        s = None if spk is None else np.ascontiguousarray(spk, np.float32)
        r = Request(_ptr(t), t.size, _ptr(c), 0 if c is None else c.size, _ptr(s), params, int(rng_mode), int(seed),
                    int(n_predict), int(min_tokens), int(max_retries))
        rid = lib().t3b_serve_submit(self.ctx, C.byref(r))
        if rid < 0:
            check(rid, self.ctx)
        return rid

    def serve_run(self, max_iters):
        """Run scheduler iterations; returns (n_active, n_queued)."""
        a, q = C.c_int32(0), C.c_int32(0)
        check(lib().t3b_serve_run(self.ctx, int(max_iters), C.byref(a), C.byref(q)), self.ctx)
        return a.value, q.value

    def serve_result(self, rid, cap=16384):
        """Tokens of a finished request (None while pending), and attempts."""
        out = np.zeros(cap, np.int32)
        n, att = C.c_int32(0), C.c_int32(0)
        rc = lib().t3b_serve_result(self.ctx, int(rid), _ptr(out), cap, C.byref(n), C.byref(att))
        if rc < 0:
            check(rc, self.ctx)
        return (out[:n.value].copy() if rc == 1 else None), att.value

    def serve_stats(self):
        """(tokens sampled by batched steps, their device ms) since alloc_streams."""
        n, ms = C.c_longlong(0), C.c_double(0)
        check(lib().t3b_serve_stats(self.ctx, C.byref(n), C.byref(ms)), self.ctx)
        return n.value, ms.value

    def stream_handle(self):
        """cudaStream_t of this context (int), e.g. for torch.cuda.ExternalStream."""
        return lib().t3b_stream_handle(self.ctx)

    def last_device_ms(self):
        return lib().t3b_last_device_ms(self.ctx)

    def cancel(self):
        lib().t3b_cancel(self.ctx)

    def close(self):
        if getattr(self, "ctx", None):
            lib().t3b_destroy(self.ctx)
            self.ctx = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def load_model_gguf(path, device=0):
    """load_model_gguf (main.cpp:348-463): parse the GGUF on the host, upload
    and repack on the device."""
    hp, tensors = t3_gguf.read_gguf(path)
    return T3Model(hp, tensors, device)


def sample_params_from(top_k=1000, top_p=0.95, temp=0.8, repeat_penalty=1.2, min_p=0.0, cfg_weight=0.0):
    return SampleParams.make(top_k, top_p, temp, repeat_penalty, min_p, cfg_weight)
