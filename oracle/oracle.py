"""ctypes wrapper of the CPU oracle (oracle/oracle.c).

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and
bench.py's cpu_baseline / reference leg, always as the checker or the CPU
baseline, never by the product library. The oracle restates the reference's
Go scalar path; oracle.c cites the Go source for every function.
"""
import ctypes as C
import os
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "build" / "liboracle.so"

OC = {"F32": 0, "F16": 1, "Q5_1": 7, "Q8_0": 8, "Q5_K": 13, "Q6_K": 14, "BF16": 30}


class Tensor(C.Structure):
    _fields_ = [("dtype", C.c_int), ("rows", C.c_int64), ("cols", C.c_int64), ("data", C.c_void_p)]


class Config(C.Structure):
    _fields_ = [("vocab_size", C.c_int), ("hidden_size", C.c_int), ("intermediate_size", C.c_int),
                ("num_hidden_layers", C.c_int), ("num_attention_heads", C.c_int), ("num_key_value_heads", C.c_int),
                ("max_position_embeddings", C.c_int), ("layer_norm_eps", C.c_double), ("rope_theta", C.c_double),
                ("partial_rotary_factor", C.c_double)]


_lib = None


def build():
    subprocess.run(["make", "-s", "-C", str(HERE)], check=True)


def lib():
    global _lib
    if _lib is not None:
        return _lib
    if not LIB_PATH.exists() or LIB_PATH.stat().st_mtime < (HERE / "oracle.c").stat().st_mtime:
        build()
    L = C.CDLL(str(LIB_PATH))
    f32p, i32p, f64p, P = C.POINTER(C.c_float), C.POINTER(C.c_int), C.POINTER(C.c_double), C.c_void_p
    sig = {
        "oc_half_to_float": ([C.c_uint16], C.c_float),
        "oc_float_to_half": ([C.c_float], C.c_uint16),
        "oc_decode_kblock": ([f32p, P, C.c_int], None),
        "oc_read_values": ([f32p, C.POINTER(Tensor), C.c_int64, C.c_int64], None),
        "oc_mul_rows": ([f32p, f32p, C.POINTER(Tensor)], None),
        "oc_mul_batch": ([f32p, f32p, C.c_int, C.POINTER(Tensor)], None),
        "oc_stable_rotate": ([f32p, C.c_int, C.c_int, C.c_int, C.c_int, C.c_double], None),
        "oc_argmax": ([f32p, C.c_int], C.c_int),
        "oc_stablelm_new": ([C.POINTER(Config), C.POINTER(Tensor), C.c_int, C.c_int, C.c_int], P),
        "oc_stablelm_free": ([P], None),
        "oc_stablelm_forward": ([P, C.c_int, C.c_int, C.c_int, f32p], C.c_int),
        "oc_stablelm_prefill": ([P, i32p, C.c_int, C.c_int, C.c_int, f32p], C.c_int),
        "oc_stablelm_greedy": ([P, i32p, C.c_int, C.c_int, C.c_int, i32p, f32p], C.c_int),
        "oc_llama_new": ([P, C.c_size_t], P),
        "oc_llama_free": ([P], None),
        "oc_llama_config": ([P, i32p], C.c_int),
        "oc_llama_transformer": ([P, C.c_int, C.c_int, f32p], C.c_int),
        "oc_summarize_logits": ([f32p, C.c_int, C.c_int, C.c_int, i32p, f64p, i32p], C.c_double),
        "oc_sampling_candidates": ([f32p, C.c_int, C.c_int, i32p, f64p], C.c_int),
        "oc_repetition_weight": ([C.c_int, C.c_int, C.c_double], C.c_double),
        "oc_penalized_logits": ([f32p, C.c_int, i32p, C.c_int, C.c_double, C.c_int, C.c_double, C.c_double, C.c_double, f64p],
                                None),
        "oc_sampling_candidates_f64": ([f64p, C.c_int, C.c_int, i32p, f64p], C.c_int),
        "oc_set_threads": ([C.c_int], None),
        "oc_get_threads": ([], C.c_int),
    }
    for name, (args, res) in sig.items():
        fn = getattr(L, name)
        fn.argtypes = args
        fn.restype = res
    _lib = L
    return L


def _f32(a):
    a = np.ascontiguousarray(a, dtype=np.float32)
    return a, a.ctypes.data_as(C.POINTER(C.c_float))


def _u8(payload):
    if isinstance(payload, np.ndarray):
        return np.ascontiguousarray(payload).view(np.uint8).reshape(-1)
    return np.frombuffer(bytes(payload), dtype=np.uint8)


def set_threads(n):
    lib().oc_set_threads(int(n))


def threads():
    return lib().oc_get_threads()


def half_to_float(h):
    return lib().oc_half_to_float(int(h))


def float_to_half(v):
    return lib().oc_float_to_half(float(v))


def tensor(dtype, rows, cols, payload):
    buf = _u8(payload)
    return Tensor(OC[dtype], rows, cols, buf.ctypes.data), buf


def read_values(dtype, payload, rows, cols, offset=0, n=None):
    t, buf = tensor(dtype, rows, cols, payload)
    n = rows * cols - offset if n is None else n
    out = np.empty(n, np.float32)
    lib().oc_read_values(out.ctypes.data_as(C.POINTER(C.c_float)), C.byref(t), offset, n)
    return out


def mul_rows(dtype, payload, rows, cols, x):
    t, buf = tensor(dtype, rows, cols, payload)
    x, xp = _f32(x)
    out = np.empty(rows, np.float32)
    lib().oc_mul_rows(out.ctypes.data_as(C.POINTER(C.c_float)), xp, C.byref(t))
    return out


def mul_batch(dtype, payload, rows, cols, x):
    """x: [n, cols] -> [n, rows] (matmul.go:55-95)."""
    t, buf = tensor(dtype, rows, cols, payload)
    x, xp = _f32(x)
    n = x.shape[0]
    out = np.empty((n, rows), np.float32)
    lib().oc_mul_batch(out.ctypes.data_as(C.POINTER(C.c_float)), xp, n, C.byref(t))
    return out


def stable_rotate(x, head_size, rotary, pos, theta):
    x = np.array(x, dtype=np.float32)
    lib().oc_stable_rotate(x.ctypes.data_as(C.POINTER(C.c_float)), len(x), head_size, rotary, pos, theta)
    return x


def summarize_logits(logits, chosen, count):
    logits, lp = _f32(logits)
    ids = np.empty(max(count, 1), np.int32)
    vals = np.empty(max(count, 1), np.float64)
    n = C.c_int()
    ch = lib().oc_summarize_logits(lp, len(logits), chosen, count, ids.ctypes.data_as(C.POINTER(C.c_int)),
                                   vals.ctypes.data_as(C.POINTER(C.c_double)), C.byref(n))
    return ch, ids[:n.value], vals[:n.value]


def sampling_candidates(logits, k):
    logits, lp = _f32(logits)
    ids = np.empty(k, np.int32)
    vals = np.empty(k, np.float64)
    n = lib().oc_sampling_candidates(lp, len(logits), k, ids.ctypes.data_as(C.POINTER(C.c_int)),
                                     vals.ctypes.data_as(C.POINTER(C.c_double)))
    return ids[:n], vals[:n]


def repetition_weight(age, window, slope):
    return lib().oc_repetition_weight(int(age), int(window), float(slope))


def penalized_logits(logits, history, repetition_penalty=1.0, repetition_range=0, repetition_slope=0.0,
                     presence_penalty=0.0, frequency_penalty=0.0):
    """sampling.go:76-101 penalizedLogits -> float64 scores."""
    logits, lp = _f32(logits)
    h = np.ascontiguousarray(history, dtype=np.int32)
    out = np.empty(len(logits), np.float64)
    lib().oc_penalized_logits(lp, len(logits), h.ctypes.data_as(C.POINTER(C.c_int)), len(h), float(repetition_penalty),
                              int(repetition_range), float(repetition_slope), float(presence_penalty),
                              float(frequency_penalty), out.ctypes.data_as(C.POINTER(C.c_double)))
    return out


def sampling_candidates_f64(scores, k):
    scores = np.ascontiguousarray(scores, dtype=np.float64)
    ids = np.empty(k, np.int32)
    vals = np.empty(k, np.float64)
    n = lib().oc_sampling_candidates_f64(scores.ctypes.data_as(C.POINTER(C.c_double)), len(scores), k,
                                         ids.ctypes.data_as(C.POINTER(C.c_int)), vals.ctypes.data_as(C.POINTER(C.c_double)))
    return ids[:n], vals[:n]


class StableLM:
    """The Go CPU StableLM engine (stablelm.go, prefill.go) with one KV state."""

    def __init__(self, config, tensors, half_kv=False, capacity=None):
        from tinyoai_b200.checkpoint import stablelm_layer_names
        self.c = config
        capacity = capacity or config["max_position_embeddings"]
        names = stablelm_layer_names(config)
        arr = (Tensor * len(names))()
        self._keep = []
        for i, name in enumerate(names):
            dt, shape, payload = tensors[name]
            rows, cols = (shape[0], shape[1]) if len(shape) == 2 else (1, shape[0])
            t, buf = tensor(dt, rows, cols, payload)
            self._keep.append(buf)
            arr[i] = t
        cfg = Config(config["vocab_size"], config["hidden_size"], config["intermediate_size"],
                     config["num_hidden_layers"], config["num_attention_heads"], config["num_key_value_heads"],
                     config["max_position_embeddings"], float(config["layer_norm_eps"]), float(config["rope_theta"]),
                     float(config["partial_rotary_factor"]))
        self._h = lib().oc_stablelm_new(C.byref(cfg), arr, len(names), int(half_kv), capacity)
        if not self._h:
            raise ValueError("oracle: invalid model")
        self.V = config["vocab_size"]

    def forward(self, token, pos, want_logits=True):
        out = np.empty(self.V, np.float32)
        rc = lib().oc_stablelm_forward(self._h, int(token), int(pos), int(want_logits), out.ctypes.data_as(C.POINTER(C.c_float)))
        if rc:
            raise ValueError("oracle forward failed")
        return out if want_logits else None

    def prefill(self, ids, start=0, chunk=128):
        ids = np.ascontiguousarray(ids, dtype=np.int32)
        out = np.empty(self.V, np.float32)
        rc = lib().oc_stablelm_prefill(self._h, ids.ctypes.data_as(C.POINTER(C.c_int)), len(ids), start, chunk,
                                       out.ctypes.data_as(C.POINTER(C.c_float)))
        if rc:
            raise ValueError("oracle prefill failed")
        return out

    def greedy(self, prompt, steps, chunk=128):
        prompt = np.ascontiguousarray(prompt, dtype=np.int32)
        out = np.empty(steps, np.int32)
        margins = np.empty(steps, np.float32)
        rc = lib().oc_stablelm_greedy(self._h, prompt.ctypes.data_as(C.POINTER(C.c_int)), len(prompt), steps, chunk,
                                      out.ctypes.data_as(C.POINTER(C.c_int)), margins.ctypes.data_as(C.POINTER(C.c_float)))
        if rc:
            raise ValueError("oracle greedy failed")
        return out, margins

    def close(self):
        if self._h:
            lib().oc_stablelm_free(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class Llama:
    """The Go legacy llama2.c engine (model.go:407-481)."""

    def __init__(self, checkpoint):
        self._buf = C.create_string_buffer(bytes(checkpoint), len(checkpoint))
        self._h = lib().oc_llama_new(self._buf, len(checkpoint))
        if not self._h:
            raise ValueError("oracle: invalid llama2.c checkpoint")
        cfg = (C.c_int * 7)()
        lib().oc_llama_config(self._h, cfg)
        self.dim, self.hidden, self.layers, self.heads, self.kv_heads, self.vocab, self.seq = list(cfg)

    def transformer(self, token, pos):
        out = np.empty(self.vocab, np.float32)
        if lib().oc_llama_transformer(self._h, int(token), int(pos), out.ctypes.data_as(C.POINTER(C.c_float))):
            raise ValueError("oracle transformer failed")
        return out

    def greedy(self, prompt, steps):
        """Forced prompt then argmax tokens (model.go:314-340 with Temperature 0)."""
        logits = None
        for pos, tok in enumerate(prompt):
            logits = self.transformer(tok, pos)
        out, pos = [], len(prompt)
        for i in range(steps):
            t = int(np.argmax(logits))
            out.append(t)
            if i + 1 < steps:
                logits = self.transformer(t, pos)
                pos += 1
        return np.array(out, np.int32)

    def close(self):
        if self._h:
            lib().oc_llama_free(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
