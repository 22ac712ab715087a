"""ctypes binding of include/tinyoai_cuda.h (the same entry points a cgo
binding declares). Loading never falls back to another implementation: if
the in-tree libtinyoai_cuda.so is missing, import of the backend fails."""
import ctypes as C
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libtinyoai_cuda.so"

DECODE_ELEMENT, DECODE_GROUP8, DECODE_TC = 0, 1, 2
TCU_OK, TCU_EINVAL, TCU_ENODEV, TCU_ENOMEM, TCU_ECUDA, TCU_ECLOSED, TCU_EUNSUP, TCU_ETIMEOUT = 0, -1, -2, -3, -4, -5, -6, -7
F32, F16, Q5_1, Q8_0, Q5_K, Q6_K, BF16 = 0, 1, 7, 8, 13, 14, 30
DTYPE_CODES = {"F32": F32, "F16": F16, "Q5_1": Q5_1, "Q8_0": Q8_0, "Q5_K": Q5_K, "Q6_K": Q6_K, "BF16": BF16}

# Every symbol declared in include/tinyoai_cuda.h.
EXPORTS = [
    "tcu_abi_version", "tcu_last_error", "tcu_device_count", "tcu_stablelm_load", "tcu_llama_load",
    "tcu_model_info", "tcu_model_memory", "tcu_model_free", "tcu_session_new", "tcu_session_free",
    "tcu_session_length", "tcu_session_forward", "tcu_session_forward_all", "tcu_session_generate_greedy",
    "tcu_session_shortlist", "tcu_session_fork", "tcu_session_limit", "tcu_session_set_kv_dtype",
    "tcu_session_reset", "tcu_session_set_stream", "tcu_session_profile", "tcu_session_profile_read", "tcu_branches_open", "tcu_branches_forward", "tcu_branches_argmax", "tcu_branches_close",
    "tcu_batch_open", "tcu_batch_forward", "tcu_batch_close", "tcu_shortlist_static", "tcu_read_values",
    "tcu_session_forward_logprobs", "tcu_session_sample_candidates", "tcu_batch_sample_candidates",
    "tcu_tp_unique_id", "tcu_stablelm_load_tp", "tcu_tp_plan", "tcu_tp_exchange_handle", "tcu_tp_exchange_open",
    "tcu_gguf_open", "tcu_gguf_config", "tcu_gguf_tensor_count", "tcu_gguf_tensor", "tcu_gguf_load_stablelm", "tcu_gguf_close",
    "tcu_session_save_cache", "tcu_session_load_cache",
]


class Tensor(C.Structure):
    _fields_ = [("name", C.c_char_p), ("dtype", C.c_int32), ("ndim", C.c_int32), ("shape", C.c_int64 * 2),
                ("data", C.c_void_p), ("nbytes", C.c_uint64)]


class StableLMConfig(C.Structure):
    _fields_ = [("vocab_size", C.c_int32), ("hidden_size", C.c_int32), ("intermediate_size", C.c_int32),
                ("num_hidden_layers", C.c_int32), ("num_attention_heads", C.c_int32),
                ("num_key_value_heads", C.c_int32), ("max_position_embeddings", C.c_int32),
                ("bos_token_id", C.c_int32), ("eos_token_id", C.c_int32), ("layer_norm_eps", C.c_double),
                ("rope_theta", C.c_double), ("partial_rotary_factor", C.c_double)]


class Penalties(C.Structure):
    """tcu_penalties: SamplingOptions' penalty fields (sampling.go:12-58)."""
    _fields_ = [("repetition_penalty", C.c_double), ("presence_penalty", C.c_double), ("frequency_penalty", C.c_double),
                ("repetition_slope", C.c_double), ("repetition_range", C.c_int32)]


class TpOptions(C.Structure):
    """tcu_tp_options: this process's rank of `world` and the NCCL id bytes."""
    _fields_ = [("world", C.c_int32), ("rank", C.c_int32), ("nccl_id", C.c_uint8 * 128)]


class LoadOptions(C.Structure):
    _fields_ = [("device", C.c_int32), ("kv_page_tokens", C.c_int32), ("kv_pool_bytes", C.c_int64)]


_lib = None


def lib():
    """Loads the in-tree library (once) and declares its signatures."""
    global _lib
    if _lib is not None:
        return _lib
    if not LIB_PATH.exists():
        raise ImportError(f"{LIB_PATH} is missing: run `python -m tinyoai_b200.build` (nvcc, sm_100a)")
    L = C.CDLL(str(LIB_PATH))
    P = C.c_void_p
    i32p = C.POINTER(C.c_int32)
    f32p = C.POINTER(C.c_float)
    f64p = C.POINTER(C.c_double)
    sig = {
        "tcu_abi_version": ([], C.c_int),
        "tcu_last_error": ([], C.c_char_p),
        "tcu_device_count": ([i32p], C.c_int),
        "tcu_stablelm_load": ([C.POINTER(StableLMConfig), C.POINTER(Tensor), C.c_int32, C.POINTER(LoadOptions), C.POINTER(P)], C.c_int),
        "tcu_llama_load": ([P, C.c_uint64, C.POINTER(LoadOptions), C.POINTER(P)], C.c_int),
        "tcu_model_info": ([P, i32p, i32p, i32p, i32p, i32p, i32p], C.c_int),
        "tcu_model_memory": ([P, C.POINTER(C.c_uint64), C.POINTER(C.c_uint64), C.POINTER(C.c_uint64)], C.c_int),
        "tcu_model_free": ([P], C.c_int),
        "tcu_session_new": ([P, C.c_int32, C.POINTER(P)], C.c_int),
        "tcu_session_free": ([P], C.c_int),
        "tcu_session_length": ([P, i32p], C.c_int),
        "tcu_session_forward": ([P, C.c_int32, i32p, C.c_int32, C.c_int32, f32p], C.c_int),
        "tcu_session_forward_all": ([P, C.c_int32, i32p, C.c_int32, f32p], C.c_int),
        "tcu_session_generate_greedy": ([P, C.c_int32, i32p, C.c_int32, C.c_int32, i32p], C.c_int),
        "tcu_session_shortlist": ([P, C.c_int32, i32p, f32p, C.POINTER(C.c_double), i32p], C.c_int),
        "tcu_session_fork": ([P, C.POINTER(P)], C.c_int),
        "tcu_session_limit": ([P, C.c_int32, i32p], C.c_int),
        "tcu_session_set_kv_dtype": ([P, C.c_int32, i32p], C.c_int),
        "tcu_session_reset": ([P], C.c_int),
        "tcu_session_set_stream": ([P, P], C.c_int),
        "tcu_session_profile": ([P, C.c_int32], C.c_int),
        "tcu_session_profile_read": ([P, C.c_int32, C.POINTER(C.c_int64), C.POINTER(C.c_double), C.c_int32], C.c_int),
        "tcu_branches_open": ([P, C.c_int32, C.c_int32, C.POINTER(P)], C.c_int),
        "tcu_branches_forward": ([P, i32p, f32p], C.c_int),
        "tcu_branches_argmax": ([P, i32p], C.c_int),
        "tcu_branches_close": ([P], C.c_int),
        "tcu_batch_open": ([P, C.c_int32, C.POINTER(P)], C.c_int),
        "tcu_batch_forward": ([P, C.POINTER(P), i32p, C.c_int32, f32p, i32p], C.c_int),
        "tcu_batch_close": ([P], C.c_int),
        "tcu_shortlist_static": ([C.c_int32, P, C.c_int32, C.c_int32, P, i32p, f32p, C.POINTER(C.c_double), i32p], C.c_int),
        "tcu_read_values": ([C.c_int32, C.c_int32, P, C.c_uint64, C.c_int32, C.c_int32, C.c_int64, C.c_int64, C.c_int32, f32p],
                            C.c_int),
        "tcu_session_forward_logprobs": ([P, C.c_int32, i32p, i32p, C.c_int32, C.c_int32, f64p, i32p, f64p, f32p], C.c_int),
        "tcu_session_sample_candidates": ([P, i32p, C.c_int32, C.POINTER(Penalties), C.c_int32, i32p, f64p, i32p], C.c_int),
        "tcu_batch_sample_candidates": ([P, C.c_int32, i32p, i32p, C.POINTER(Penalties), C.c_int32, i32p, f64p], C.c_int),
        "tcu_tp_unique_id": ([C.POINTER(C.c_uint8)], C.c_int),
        "tcu_stablelm_load_tp": ([C.POINTER(StableLMConfig), C.POINTER(Tensor), C.c_int32, C.POINTER(LoadOptions),
                                  C.POINTER(TpOptions), C.POINTER(P)], C.c_int),
        "tcu_tp_plan": ([C.POINTER(StableLMConfig), C.c_int32, C.c_int32, i32p], C.c_int),
        "tcu_tp_exchange_handle": ([C.c_void_p, C.POINTER(C.c_uint8)], C.c_int),
        "tcu_tp_exchange_open": ([C.c_void_p, C.POINTER(C.c_uint8)], C.c_int),
        "tcu_gguf_open": ([C.c_char_p, C.POINTER(P)], C.c_int),
        "tcu_gguf_config": ([P, C.POINTER(StableLMConfig)], C.c_int),
        "tcu_gguf_tensor_count": ([P, i32p], C.c_int),
        "tcu_gguf_tensor": ([P, C.c_int32, C.POINTER(Tensor)], C.c_int),
        "tcu_gguf_load_stablelm": ([P, C.POINTER(LoadOptions), C.POINTER(TpOptions), C.POINTER(P)], C.c_int),
        "tcu_gguf_close": ([P], C.c_int),
        "tcu_session_save_cache": ([P, C.c_char_p, C.POINTER(C.c_uint8), i32p, C.c_int32], C.c_int),
        "tcu_session_load_cache": ([P, C.c_char_p, C.POINTER(C.c_uint8), i32p, C.c_int32, i32p], C.c_int),
    }
    for name, (args, res) in sig.items():
        fn = getattr(L, name)
        fn.argtypes = args
        fn.restype = res
    _lib = L
    return L


class BackendError(RuntimeError):
    """A failed C call: .code is the TCU_E* status, the message is tcu_last_error()."""

    def __init__(self, code, message):
        super().__init__(f"{message} (status {code})")
        self.code = code


def check(rc):
    if rc != TCU_OK:
        raise BackendError(rc, lib().tcu_last_error().decode(errors="replace"))
    return rc
