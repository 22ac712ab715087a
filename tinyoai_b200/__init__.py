"""tinyoai_b200: a B200 (sm_100a) backend for tinyoai's StableLM and llama2.c
forward path, reached through the C ABI of include/tinyoai_cuda.h.

This module is the host-side mirror of the reference's native forwarder
interfaces, as a cgo wrapper would expose them to Go:

  Session.forward          mlxForwarder.Forward            (mlx.go:45-51)
  Session.forward_all      llamaMLXForwarder.Forward(all)  (mlx_llama.go:27-35)
  Session.fork             mlxForker.Fork                  (sessions.go:26-30)
  Session.new_branches     mlxBrancher.NewBranches         (branches.go:55-59)
  Branches.forward / close mlxBranches                     (branches.go:49-54)
  Session.limit_cache      LimitCache                      (mlx_native.go:231-244)
  Session.set_kv_bits      SetKVBits                       (mlx_kv.go:78-91)
  Session.reset            llamaMLXForwarder.Reset

All computation runs in libtinyoai_cuda.so on the GPU; there is no CPU path.
Errors raise BackendError carrying the library's status and message.
"""
import ctypes as C

import numpy as np

from . import _lib
from ._lib import BackendError, check, lib
from .checkpoint import as_bytes, dtype_code

__all__ = ["Model", "Session", "Branches", "BackendError", "GGUF", "device_count", "read_values", "tp_unique_id", "tp_plan"]


def _i32(a):
    a = np.ascontiguousarray(np.asarray(a, dtype=np.int32))
    return a, a.ctypes.data_as(C.POINTER(C.c_int32))


def device_count():
    n = C.c_int32()
    check(lib().tcu_device_count(C.byref(n)))
    return n.value


_DECODERS = {"element": _lib.DECODE_ELEMENT, "group8": _lib.DECODE_GROUP8, "tc": _lib.DECODE_TC}


def read_values(dtype, payload, rows, cols, offset=0, n=None, decoder="element", device=0):
    """weightTensor.readValues (matmul.go:12-50) through one of the device
    decoders: "element" (matrix-vector kernels), "group8" (batched products,
    Q6_K/Q5_K) or "tc" (the tcgen05 GEMM operand, Q8_0/Q6_K/Q5_K). payload is
    the tensor in its file encoding; returns n float32 values."""
    buf = np.ascontiguousarray(np.frombuffer(bytes(as_bytes(payload)), dtype=np.uint8))
    n = rows * cols - offset if n is None else n
    out = np.empty(max(n, 1), np.float32)
    check(lib().tcu_read_values(device, dtype_code(dtype), buf.ctypes.data_as(C.c_void_p), buf.nbytes, rows, cols, offset, n,
                                _DECODERS[decoder], out.ctypes.data_as(C.POINTER(C.c_float))))
    return out[:n]


def penalties_struct(repetition_penalty=1.0, presence_penalty=0.0, frequency_penalty=0.0, repetition_slope=0.0,
                     repetition_range=0):
    return _lib.Penalties(repetition_penalty, presence_penalty, frequency_penalty, repetition_slope, repetition_range)


def _config_struct(config):
    return _lib.StableLMConfig(
        config["vocab_size"], config["hidden_size"], config["intermediate_size"], config["num_hidden_layers"],
        config["num_attention_heads"], config["num_key_value_heads"], config["max_position_embeddings"],
        int(config.get("bos_token_id", 0)), int(config.get("eos_token_id", 0)), float(config["layer_norm_eps"]),
        float(config["rope_theta"]), float(config["partial_rotary_factor"]))


class GGUF:
    """A memory-mapped GGUF StableLM checkpoint (tcu_gguf_open: readGGUF and
    loadStableGGUF's checks, gguf.go:139-357). .config is the derived
    configuration; .tensors() lists (name, dtype, shape, nbytes) under the
    Hugging Face names; .load() uploads the model from the mapping."""

    def __init__(self, path):
        h = C.c_void_p()
        check(lib().tcu_gguf_open(str(path).encode(), C.byref(h)))
        self._h = h
        c = _lib.StableLMConfig()
        check(lib().tcu_gguf_config(self._h, C.byref(c)))
        self.config = dict(model_type="stablelm", vocab_size=c.vocab_size, hidden_size=c.hidden_size,
                           intermediate_size=c.intermediate_size, num_hidden_layers=c.num_hidden_layers,
                           num_attention_heads=c.num_attention_heads, num_key_value_heads=c.num_key_value_heads,
                           max_position_embeddings=c.max_position_embeddings, bos_token_id=c.bos_token_id,
                           eos_token_id=c.eos_token_id, layer_norm_eps=c.layer_norm_eps, rope_theta=c.rope_theta,
                           partial_rotary_factor=c.partial_rotary_factor, use_parallel_residual=True)

    def tensors(self):
        n = C.c_int32()
        check(lib().tcu_gguf_tensor_count(self._h, C.byref(n)))
        out = []
        for i in range(n.value):
            t = _lib.Tensor()
            check(lib().tcu_gguf_tensor(self._h, i, C.byref(t)))
            shape = tuple(t.shape[j] for j in range(t.ndim))
            out.append((t.name.decode(), t.dtype, shape, C.string_at(t.data, t.nbytes)))
        return out

    def load(self, device=0, kv_page_tokens=0, kv_pool_bytes=0):
        out = C.c_void_p()
        opts = _options(device, kv_page_tokens, kv_pool_bytes)
        check(lib().tcu_gguf_load_stablelm(self._h, C.byref(opts), None, C.byref(out)))
        m = Model(out.value, "stablelm")
        m.config = dict(self.config)
        m.tp = None
        return m

    def close(self):
        if self._h:
            check(lib().tcu_gguf_close(self._h))
            self._h = None

    def __enter__(self):
        return self

    def __exit__(self, *a):
        self.close()


def tp_unique_id():
    """128 bytes naming a new NCCL communicator (rank 0 makes it; every rank
    passes the same bytes to Model.load_stablelm(..., tp=...))."""
    buf = (C.c_uint8 * 128)()
    check(lib().tcu_tp_unique_id(buf))
    return bytes(buf)


def tp_plan(config, world, rank):
    """Rank `rank`'s share of a head-parallel model (needs no GPU):
    (first query head, query heads, first KV head, KV heads, first MLP row,
    MLP rows)."""
    out = (C.c_int32 * 6)()
    check(lib().tcu_tp_plan(C.byref(_config_struct(config)), world, rank, out))
    return tuple(out)


def _options(device, kv_page_tokens, kv_pool_bytes):
    return _lib.LoadOptions(device, kv_page_tokens, kv_pool_bytes)


class Model:
    """Weights resident on one GPU plus the model's paged KV pool."""

    def __init__(self, handle, arch):
        self._h = C.c_void_p(handle)
        self.arch = arch
        v, d, L, H, KVH, P = (C.c_int32() for _ in range(6))
        check(lib().tcu_model_info(self._h, C.byref(v), C.byref(d), C.byref(L), C.byref(H), C.byref(KVH), C.byref(P)))
        self.vocab_size, self.hidden_size, self.num_layers = v.value, d.value, L.value
        self.num_heads, self.num_kv_heads, self.max_positions = H.value, KVH.value, P.value

    @classmethod
    def load_stablelm(cls, config, tensors, device=0, kv_page_tokens=0, kv_pool_bytes=0, tp=None):
        """config: validated dict (checkpoint.stablelm_config); tensors: {name:
        (dtype name, shape, payload)} in file encoding (LoadStableLM). tp:
        (world, rank, nccl_id bytes) loads this rank's share of a
        head-parallel model (tcu_stablelm_load_tp)."""
        cfg = _config_struct(config)
        arr = (_lib.Tensor * len(tensors))()
        keep = []
        for i, (name, (dt, shape, payload)) in enumerate(tensors.items()):
            buf = as_bytes(payload)
            if isinstance(buf, np.ndarray):
                ptr, n = buf.ctypes.data, buf.nbytes
            else:
                cb = C.create_string_buffer(bytes(buf), len(buf))
                ptr, n = C.addressof(cb), len(buf)
                buf = cb
            keep.append(buf)
            nm = name.encode()
            keep.append(nm)
            sh = (C.c_int64 * 2)(*(list(shape) + [0] * (2 - len(shape))))
            arr[i] = _lib.Tensor(nm, dtype_code(dt), len(shape), sh, ptr, n)
        out = C.c_void_p()
        opts = _options(device, kv_page_tokens, kv_pool_bytes)
        if tp is None:
            check(lib().tcu_stablelm_load(C.byref(cfg), arr, len(tensors), C.byref(opts), C.byref(out)))
        else:
            world, rank, nccl_id = tp
            t = _lib.TpOptions(world, rank)
            C.memmove(t.nccl_id, bytes(nccl_id), 128)
            check(lib().tcu_stablelm_load_tp(C.byref(cfg), arr, len(tensors), C.byref(opts), C.byref(t), C.byref(out)))
        m = cls(out.value, "stablelm")
        m.config = dict(config)
        m.tp = tp
        return m

    def tp_exchange_handle(self):
        """This rank's CUDA IPC handle of its exchange buffer (64 bytes;
        tcu_tp_exchange_handle). Share it with the other ranks, then call
        tp_exchange_open with every rank's handle in rank order."""
        buf = (C.c_uint8 * 64)()
        check(lib().tcu_tp_exchange_handle(self._h, buf))
        return bytes(buf)

    def tp_exchange_open(self, handles):
        """Opens the other ranks' exchange buffers; from then on the per-layer
        exchange runs over NVLink peer memory (tcu_tp_exchange_open)."""
        raw = b"".join(bytes(h) for h in handles)
        buf = (C.c_uint8 * len(raw)).from_buffer_copy(raw)
        check(lib().tcu_tp_exchange_open(self._h, buf))

    @classmethod
    def load_llama(cls, checkpoint, device=0, kv_page_tokens=0, kv_pool_bytes=0):
        """llama2.c checkpoint bytes (LoadModel, model.go:90-122)."""
        buf = C.create_string_buffer(bytes(checkpoint), len(checkpoint))
        out = C.c_void_p()
        opts = _options(device, kv_page_tokens, kv_pool_bytes)
        check(lib().tcu_llama_load(buf, len(checkpoint), C.byref(opts), C.byref(out)))
        return cls(out.value, "llama")

    def memory(self):
        w, p, u = C.c_uint64(), C.c_uint64(), C.c_uint64()
        check(lib().tcu_model_memory(self._h, C.byref(w), C.byref(p), C.byref(u)))
        return {"weights": w.value, "kv_pool": p.value, "kv_used": u.value}

    def batch(self, max_rows):
        """A continuous-batching step runner for up to max_rows sessions."""
        h = C.c_void_p()
        check(lib().tcu_batch_open(self._h, int(max_rows), C.byref(h)))
        return Batch(self, h.value, int(max_rows))

    def session(self, kv="f32"):
        return Session(self, kv)

    def close(self):
        if self._h:
            check(lib().tcu_model_free(self._h))
            self._h = None


class Session:
    """One resident token stream with paged KV (the native forwarder)."""

    def __init__(self, model, kv="f32", handle=None):
        self.model = model
        if kv not in ("f32", "f16"):
            raise ValueError(f"unsupported KV cache precision {kv!r}: use f32 or f16")
        self.kv = kv
        if handle is None:
            h = C.c_void_p()
            check(lib().tcu_session_new(model._h, _lib.F32 if kv == "f32" else _lib.F16, C.byref(h)))
            handle = h.value
        self._h = C.c_void_p(handle)

    @property
    def length(self):
        n = C.c_int32()
        check(lib().tcu_session_length(self._h, C.byref(n)))
        return n.value

    def forward(self, prefix, tokens, want_logits=True):
        t, tp = _i32(tokens)
        if want_logits:
            out = np.empty(self.model.vocab_size, np.float32)
            check(lib().tcu_session_forward(self._h, prefix, tp, len(t), 1, out.ctypes.data_as(C.POINTER(C.c_float))))
            return out
        check(lib().tcu_session_forward(self._h, prefix, tp, len(t), 0, None))
        return None

    def forward_all(self, prefix, tokens):
        t, tp = _i32(tokens)
        out = np.empty((len(t), self.model.vocab_size), np.float32)
        check(lib().tcu_session_forward_all(self._h, prefix, tp, len(t), out.ctypes.data_as(C.POINTER(C.c_float))))
        return out

    def generate_greedy(self, prefix, tokens, steps):
        t, tp = _i32(tokens)
        out = np.empty(steps, np.int32)
        check(lib().tcu_session_generate_greedy(self._h, prefix, tp, len(t), steps, out.ctypes.data_as(C.POINTER(C.c_int32))))
        return out

    def forward_logprobs(self, prefix, tokens, targets, count, want_logits=True):
        """mlxProbabilityForwarder.ForwardWithLogprobs (mlx.go:53-57): per
        input position the target's log probability and `count` top (id,
        log probability) pairs (summarizeLogits, logprobs.go:64-95). Returns
        (chosen [n], top_ids [n, count], top_logprobs [n, count], final logits
        or None)."""
        t, tp = _i32(tokens)
        g, gp = _i32(targets)
        n = len(t)
        chosen = np.empty(n, np.float64)
        ids = np.empty((n, count), np.int32)
        vals = np.empty((n, count), np.float64)
        logits = np.empty(self.model.vocab_size, np.float32) if want_logits else None
        check(lib().tcu_session_forward_logprobs(
            self._h, prefix, tp, gp, n, count, chosen.ctypes.data_as(C.POINTER(C.c_double)),
            ids.ctypes.data_as(C.POINTER(C.c_int32)), vals.ctypes.data_as(C.POINTER(C.c_double)),
            logits.ctypes.data_as(C.POINTER(C.c_float)) if want_logits else None))
        return chosen, ids, vals, logits

    def sample_candidates(self, history, k, **penalties):
        """samplingCandidates(penalizedLogits(...), k) (sampling.go:76-143)
        over the last forward's logits: (ids, float64 scores); ids[0] is the
        greedy choice. penalties: repetition_penalty, presence_penalty,
        frequency_penalty, repetition_slope, repetition_range."""
        h, hp = _i32(history)
        ids = np.empty(k, np.int32)
        scores = np.empty(k, np.float64)
        n = C.c_int32()
        check(lib().tcu_session_sample_candidates(self._h, hp, len(h), C.byref(penalties_struct(**penalties)), k,
                                                  ids.ctypes.data_as(C.POINTER(C.c_int32)),
                                                  scores.ctypes.data_as(C.POINTER(C.c_double)), C.byref(n)))
        return ids[:n.value], scores[:n.value]

    def shortlist(self, k):
        ids = np.empty(k, np.int32)
        vals = np.empty(k, np.float32)
        lse = C.c_double()
        n = C.c_int32()
        check(lib().tcu_session_shortlist(self._h, k, ids.ctypes.data_as(C.POINTER(C.c_int32)),
                                          vals.ctypes.data_as(C.POINTER(C.c_float)), C.byref(lse), C.byref(n)))
        return ids[:n.value], vals[:n.value], lse.value

    def save_cache(self, path, model_sha256, tokens):
        """SaveCache (cache_file.go:55-104): the resident positions' KV to a
        TNYKV001 file; tokens are the session's resident token ids."""
        t, tp = _i32(tokens)
        ident = (C.c_uint8 * 32).from_buffer_copy(bytes(model_sha256))
        check(lib().tcu_session_save_cache(self._h, str(path).encode(), ident, tp, len(t)))

    def load_cache(self, path, model_sha256):
        """LoadCache (cache_file.go:108-176): restores a TNYKV001 file's
        positions as this session's context; returns their token ids."""
        ident = (C.c_uint8 * 32).from_buffer_copy(bytes(model_sha256))
        cap = self.model.max_positions
        out = np.empty(max(cap, 1), np.int32)
        n = C.c_int32()
        check(lib().tcu_session_load_cache(self._h, str(path).encode(), ident, out.ctypes.data_as(C.POINTER(C.c_int32)), cap,
                                           C.byref(n)))
        return out[:n.value]

    def fork(self):
        h = C.c_void_p()
        check(lib().tcu_session_fork(self._h, C.byref(h)))
        return Session(self.model, self.kv, handle=h.value)

    def limit_cache(self, window):
        c = C.c_int32()
        check(lib().tcu_session_limit(self._h, window, C.byref(c)))
        return bool(c.value)

    def set_kv_bits(self, bits):
        """16 -> binary16 KV, 32 -> float32 KV; reports whether KV was cleared."""
        if bits not in (16, 32):
            raise ValueError("kv bits must be 16 or 32")
        c = C.c_int32()
        check(lib().tcu_session_set_kv_dtype(self._h, _lib.F16 if bits == 16 else _lib.F32, C.byref(c)))
        self.kv = "f16" if bits == 16 else "f32"
        return bool(c.value)

    def reset(self):
        check(lib().tcu_session_reset(self._h))

    def set_stream(self, stream):
        """Run on a caller-owned CUDA stream handle (int), or None for the
        session's own stream."""
        check(lib().tcu_session_set_stream(self._h, C.c_void_p(stream) if stream else None))

    STAGES = ("embed", "norm_qkv_gate_up", "attention", "out_down_residual", "head", "prefill_projection",
              "prefill_attention", "other", "decode_step", "allreduce")

    def profile(self, enable=True):
        check(lib().tcu_session_profile(self._h, int(bool(enable))))

    def profile_read(self, reset=False):
        """{stage: (launches, milliseconds)} accumulated while profiling."""
        n = len(self.STAGES)
        launches = (C.c_int64 * n)()
        ms = (C.c_double * n)()
        rc = lib().tcu_session_profile_read(self._h, n, launches, ms, int(bool(reset)))
        if rc < 0:
            check(rc)
        return {name: (launches[i], ms[i]) for i, name in enumerate(self.STAGES)}

    def new_branches(self, prefix, count):
        h = C.c_void_p()
        check(lib().tcu_branches_open(self._h, prefix, count, C.byref(h)))
        return Branches(self, h.value, count)

    def close(self):
        if self._h:
            check(lib().tcu_session_free(self._h))
            self._h = None


class Branches:
    """count suffixes sharing a session's resident prefix read-only."""

    def __init__(self, session, handle, count):
        self.session = session
        self.count = count
        self._h = C.c_void_p(handle)

    def forward(self, tokens, want_rows=True):
        t, tp = _i32(tokens)
        if len(t) != self.count:
            raise ValueError("invalid branch batch")
        if want_rows:
            out = np.empty((self.count, self.session.model.vocab_size), np.float32)
            check(lib().tcu_branches_forward(self._h, tp, out.ctypes.data_as(C.POINTER(C.c_float))))
            return out
        check(lib().tcu_branches_forward(self._h, tp, None))
        return None

    def argmax(self):
        ids = np.empty(self.count, np.int32)
        check(lib().tcu_branches_argmax(self._h, ids.ctypes.data_as(C.POINTER(C.c_int32))))
        return ids

    def close(self):
        if self._h:
            check(lib().tcu_branches_close(self._h))
            self._h = None


class Batch:
    """One decode step for several sessions of one model at their own
    positions (tcu_batch_forward): a batching server's step."""

    def __init__(self, model, handle, max_rows):
        self.model = model
        self.max_rows = max_rows
        self._h = C.c_void_p(handle)

    def forward(self, sessions, tokens, want_rows=True):
        """Appends tokens[i] to sessions[i]; returns (rows or None, argmax ids)."""
        t, tp = _i32(tokens)
        n = len(sessions)
        if len(t) != n:
            raise ValueError("one token per session")
        hs = (C.c_void_p * n)(*[s._h.value for s in sessions])
        ids = np.empty(n, np.int32)
        rows = np.empty((n, self.model.vocab_size), np.float32) if want_rows else None
        check(lib().tcu_batch_forward(self._h, hs, tp, n, rows.ctypes.data_as(C.POINTER(C.c_float)) if want_rows else None,
                                      ids.ctypes.data_as(C.POINTER(C.c_int32))))
        return rows, ids

    def sample_candidates(self, histories, k, penalties=None):
        """tcu_batch_sample_candidates over the last step's rows: histories is
        one id list per row, penalties one dict per row (or None: neutral).
        Returns (ids [n, k], scores [n, k])."""
        n = len(histories)
        lens = np.array([len(h) for h in histories], np.int32)
        flat = np.concatenate([np.asarray(h, np.int32) for h in histories]) if lens.sum() else np.zeros(1, np.int32)
        flat = np.ascontiguousarray(flat, np.int32)
        ps = (_lib.Penalties * n)(*[penalties_struct(**(penalties[i] if penalties else {})) for i in range(n)])
        ids = np.empty((n, k), np.int32)
        scores = np.empty((n, k), np.float64)
        check(lib().tcu_batch_sample_candidates(self._h, n, flat.ctypes.data_as(C.POINTER(C.c_int32)),
                                                lens.ctypes.data_as(C.POINTER(C.c_int32)), ps, k,
                                                ids.ctypes.data_as(C.POINTER(C.c_int32)),
                                                scores.ctypes.data_as(C.POINTER(C.c_double))))
        return ids, scores

    def close(self):
        if self._h:
            check(lib().tcu_batch_close(self._h))
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
