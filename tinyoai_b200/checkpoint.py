"""Checkpoint readers feeding the C ABI: a Hugging Face safetensors directory
(LoadStableLM, stablelm.go:136-161; openTensorStore, safetensors.go:130-225)
and StableLM config validation (stablelm.go:85-111)."""
import json
import math
import struct
from pathlib import Path

import numpy as np

from ._lib import DTYPE_CODES

_ST_DTYPES = {"F32": "F32", "F16": "F16", "BF16": "BF16"}


def read_safetensors(path):
    """Returns {name: (dtype, shape, bytes)} for one safetensors file."""
    data = Path(path).read_bytes()
    (n,) = struct.unpack_from("<Q", data, 0)
    header = json.loads(data[8:8 + n])
    base = 8 + n
    out = {}
    for name, info in header.items():
        if name == "__metadata__":
            continue
        if info["dtype"] not in _ST_DTYPES:
            raise ValueError(f"tensor {name}: unsupported safetensors dtype {info['dtype']}")
        a, b = info["data_offsets"]
        out[name] = (_ST_DTYPES[info["dtype"]], tuple(info["shape"]), data[base + a:base + b])
    return out


def read_safetensors_dir(directory):
    """Single-file or sharded safetensors in a directory."""
    d = Path(directory)
    files = sorted(d.glob("*.safetensors"))
    if not files:
        raise FileNotFoundError(f"no safetensors weights in {d}")
    tensors = {}
    for f in files:
        for name, t in read_safetensors(f).items():
            if name in tensors:
                raise ValueError(f"duplicate tensor {name}")
            tensors[name] = t
    return tensors


def stablelm_config(raw):
    """Applies LoadStableLM's defaults (stablelm.go:144) and validate()
    (stablelm.go:85-111); returns a plain dict of the fields the backend uses."""
    c = {"layer_norm_eps": 1e-5, "rope_theta": 10000.0, "partial_rotary_factor": 0.25, "hidden_act": "silu"}
    c.update(raw)
    rp = c.get("rope_parameters")
    if rp is not None:
        if rp.get("rope_type") != "default":
            raise ValueError(f"unsupported RoPE type {rp.get('rope_type')!r}")
        c["rope_theta"] = rp.get("rope_theta")
        c["partial_rotary_factor"] = rp.get("partial_rotary_factor")
    if (c.get("model_type") != "stablelm" or not c.get("use_parallel_residual") or c.get("use_qkv_bias")
            or c.get("qk_layernorm") or c.get("tie_word_embeddings") or c.get("hidden_act") != "silu"):
        raise ValueError("unsupported StableLM variant: require parallel residuals, no QKV bias/QK norm, untied embeddings, and silu")
    if c.get("rope_scaling") is not None:
        raise ValueError("RoPE scaling is not supported")
    ints = ["vocab_size", "hidden_size", "intermediate_size", "num_hidden_layers", "num_attention_heads",
            "num_key_value_heads", "max_position_embeddings"]
    if any(int(c.get(k, 0)) <= 0 for k in ints) or c["hidden_size"] % c["num_attention_heads"] \
            or c["num_attention_heads"] % c["num_key_value_heads"]:
        raise ValueError("invalid StableLM dimensions")
    rotary = c["hidden_size"] // c["num_attention_heads"] * c["partial_rotary_factor"]
    if not (c["layer_norm_eps"] > 0 and math.isfinite(c["layer_norm_eps"]) and c["rope_theta"] > 0
            and math.isfinite(c["rope_theta"]) and 0 < c["partial_rotary_factor"] <= 1
            and rotary == int(rotary) and int(rotary) % 2 == 0 and rotary >= 2):
        raise ValueError("invalid LayerNorm or partial RoPE settings")
    for k in ("bos_token_id", "eos_token_id"):
        if not 0 <= int(c.get(k, 0)) < c["vocab_size"]:
            raise ValueError("invalid BOS/EOS token IDs")
    c.setdefault("bos_token_id", 0)
    c.setdefault("eos_token_id", 0)
    return c


def load_stablelm_dir(directory):
    """(config, tensors) from a Hugging Face StableLM directory."""
    d = Path(directory)
    cfg = stablelm_config(json.loads((d / "config.json").read_text()))
    return cfg, read_safetensors_dir(d)


def stablelm_layer_names(c):
    """Tensor names in the order the oracle expects: per layer norm, bias, q,
    k, v, o, gate, up, down; then embed, head, final norm, final bias."""
    names = []
    for l in range(c["num_hidden_layers"]):
        p = f"model.layers.{l}."
        names += [p + "input_layernorm.weight", p + "input_layernorm.bias", p + "self_attn.q_proj.weight",
                  p + "self_attn.k_proj.weight", p + "self_attn.v_proj.weight", p + "self_attn.o_proj.weight",
                  p + "mlp.gate_proj.weight", p + "mlp.up_proj.weight", p + "mlp.down_proj.weight"]
    return names + ["model.embed_tokens.weight", "lm_head.weight", "model.norm.weight", "model.norm.bias"]


def dtype_code(name):
    return DTYPE_CODES[name]


def as_bytes(buf):
    """bytes-like view of a tensor payload (bytes, bytearray or numpy array)."""
    if isinstance(buf, np.ndarray):
        return np.ascontiguousarray(buf).view(np.uint8).reshape(-1)
    return buf
