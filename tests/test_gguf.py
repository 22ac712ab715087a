"""GGUF StableLM checkpoints through the library's reader (tcu_gguf_open),
mirroring gguf_test.go: the tiny reference checkpoint is written as GGUF by an
independent writer (reversed dimensions, 32-byte alignment), read back with
the same configuration and bytes, and the malformed variants of
TestGGUFRejects (gguf_test.go:179-230) are refused. The CPU tests need no GPU
(the reader only maps and parses); the GPU test loads the model from the
mapping and compares its logits bit for bit with the safetensors load
(TestGGUFRoundTrip, gguf_test.go:143-177).
"""
import json
import math
import struct

import numpy as np
import pytest

from tinyoai_b200 import GGUF, BackendError, Model
from tinyoai_b200.checkpoint import load_stablelm_dir

CODES = {"F32": 0, "F16": 1, "BF16": 30, "Q8_0": 8, "Q5_K": 13, "Q6_K": 14, "Q5_1": 7}
NAMES = [("model.embed_tokens", "token_embd"), ("lm_head", "output"), ("model.norm", "output_norm"), ("model.layers.", "blk."),
         ("input_layernorm", "attn_norm"), ("self_attn.q_proj", "attn_q"), ("self_attn.k_proj", "attn_k"),
         ("self_attn.v_proj", "attn_v"), ("self_attn.o_proj", "attn_output"), ("mlp.gate_proj", "ffn_gate"),
         ("mlp.up_proj", "ffn_up"), ("mlp.down_proj", "ffn_down")]


def gguf_name(hf):
    out, i = [], 0
    while i < len(hf):
        for a, b in NAMES:
            if hf.startswith(a, i):
                out.append(b)
                i += len(a)
                break
        else:
            out.append(hf[i])
            i += 1
    return "".join(out)


def tiny(golden):
    cfg, tensors = load_stablelm_dir(golden / "stablelm_tiny")
    meta = {
        "general.architecture": ("str", "stablelm"), "stablelm.embedding_length": ("u32", cfg["hidden_size"]),
        "stablelm.feed_forward_length": ("u32", cfg["intermediate_size"]), "stablelm.block_count": ("u32", cfg["num_hidden_layers"]),
        "stablelm.attention.head_count": ("u32", cfg["num_attention_heads"]),
        "stablelm.attention.head_count_kv": ("u32", cfg["num_key_value_heads"]),
        "stablelm.context_length": ("u32", cfg["max_position_embeddings"]),
        "stablelm.rope.dimension_count": ("u32", int(cfg["hidden_size"] // cfg["num_attention_heads"] * cfg["partial_rotary_factor"])),
        "stablelm.use_parallel_residual": ("bool", True), "stablelm.attention.layer_norm_epsilon": ("f64", cfg["layer_norm_eps"]),
        "tokenizer.ggml.bos_token_id": ("u32", cfg["bos_token_id"]), "tokenizer.ggml.eos_token_id": ("u32", cfg["eos_token_id"]),
        "tokenizer.ggml.tokens": ("strs", [f"t{i}" for i in range(cfg["vocab_size"])]),
    }
    tens = {gguf_name(n): [dt, list(shape), bytes(payload)] for n, (dt, shape, payload) in tensors.items()}
    return cfg, tensors, meta, tens


def write_gguf(path, meta, tensors, align=32):
    head, body = bytearray(), bytearray()

    def s(x):
        b = x.encode()
        head.extend(struct.pack("<Q", len(b)) + b)

    head.extend(struct.pack("<IIQQ", 0x46554747, 3, len(tensors), len(meta)))
    for key in sorted(meta):
        kind, v = meta[key]
        s(key)
        if kind == "str":
            head.extend(struct.pack("<I", 8))
            s(v)
        elif kind == "u32":
            head.extend(struct.pack("<II", 4, v))
        elif kind == "i32":
            head.extend(struct.pack("<Ii", 5, v))
        elif kind == "f64":
            head.extend(struct.pack("<Id", 12, v))
        elif kind == "bool":
            head.extend(struct.pack("<IB", 7, int(v)))
        elif kind == "strs":
            head.extend(struct.pack("<IIQ", 9, 8, len(v)))
            for x in v:
                s(x)
        else:
            raise ValueError(kind)
    for name in sorted(tensors):
        dt, shape, data = tensors[name]
        s(name)
        head.extend(struct.pack("<I", len(shape)))
        for d in reversed(shape):
            head.extend(struct.pack("<Q", d))
        head.extend(struct.pack("<IQ", CODES.get(dt, 99), len(body)))
        body.extend(data)
        while len(body) % align:
            body.append(0)
    while len(head) % align:
        head.append(0)
    path.write_bytes(bytes(head + body))
    return path


def test_gguf_round_trip(golden, tmp_path):
    cfg, tensors, meta, tens = tiny(golden)
    with GGUF(write_gguf(tmp_path / "model.gguf", meta, tens)) as g:
        for k in ("vocab_size", "hidden_size", "intermediate_size", "num_hidden_layers", "num_attention_heads",
                  "num_key_value_heads", "max_position_embeddings", "bos_token_id", "eos_token_id"):
            assert g.config[k] == cfg[k], k
        assert g.config["layer_norm_eps"] == cfg["layer_norm_eps"]
        assert g.config["rope_theta"] == 10000.0 and g.config["partial_rotary_factor"] == cfg["partial_rotary_factor"]
        got = {name: (dt, shape, data) for name, dt, shape, data in g.tensors()}
        assert sorted(got) == sorted(tensors)
        for name, (dt, shape, payload) in tensors.items():
            assert got[name][0] == CODES[dt] and got[name][1] == tuple(shape) and got[name][2] == bytes(payload), name


def edit_arch(m, t): m["general.architecture"] = ("str", "llama")
def edit_nan(m, t): m["stablelm.attention.layer_norm_epsilon"] = ("f64", math.nan)
def edit_inf(m, t): m["stablelm.rope.freq_base"] = ("f64", math.inf)
def edit_align(m, t): m["general.alignment"] = ("u32", 3)
def edit_missing(m, t): del t["output.weight"]
def edit_shape(m, t): t["output.weight"][1] = t["output.weight"][1][::-1]
def edit_type(m, t): t["output.weight"][0] = "Q4_K"
def edit_q8(m, t): t["output.weight"][0] = "Q8_0"
def edit_scaling(m, t): m["stablelm.rope.scaling.type"] = ("str", "linear")


@pytest.mark.parametrize("edit,message", [(edit_arch, "StableLM"), (edit_nan, "LayerNorm"), (edit_inf, "RoPE"),
                                          (edit_align, "alignment"), (edit_missing, "tensor count"), (edit_shape, "shape"),
                                          (edit_type, "unsupported type"), (edit_q8, "divisible by 32"),
                                          (edit_scaling, "scaling")])
def test_gguf_rejects(golden, tmp_path, edit, message):
    _, _, meta, tens = tiny(golden)
    edit(meta, tens)
    path = write_gguf(tmp_path / "model.gguf", meta, tens)
    with pytest.raises(BackendError) as e:
        GGUF(path)
    assert message in str(e.value)


def test_gguf_rejects_truncated_and_overlapping(golden, tmp_path):
    _, _, meta, tens = tiny(golden)
    path = write_gguf(tmp_path / "model.gguf", meta, tens)
    raw = path.read_bytes()
    (tmp_path / "cut.gguf").write_bytes(raw[:-100])
    with pytest.raises(BackendError):
        GGUF(tmp_path / "cut.gguf")
    # Point the second tensor's offset at the first's data.
    body = bytearray(raw)
    first = sorted(tens)[1]
    key = struct.pack("<Q", len(first)) + first.encode()
    at = body.index(key) + len(key)
    rank = struct.unpack_from("<I", body, at)[0]
    struct.pack_into("<Q", body, at + 4 + 8 * rank + 4, 0)
    (tmp_path / "overlap.gguf").write_bytes(bytes(body))
    with pytest.raises(BackendError) as e:
        GGUF(tmp_path / "overlap.gguf")
    assert "overlapping" in str(e.value)


@pytest.mark.gpu
def test_gguf_load_matches_safetensors_bitwise(golden, tmp_path):
    """TestGGUFRoundTrip: identical logits from the GGUF and safetensors loads."""
    cfg, tensors, meta, tens = tiny(golden)
    ids = json.loads((golden / "stablelm_tiny" / "expected.json").read_text())["input_ids"]
    with GGUF(write_gguf(tmp_path / "model.gguf", meta, tens)) as g:
        a = g.load()
    b = Model.load_stablelm(cfg, tensors)
    try:
        sa, sb = a.session(), b.session()
        try:
            assert np.array_equal(sa.forward(0, ids), sb.forward(0, ids))
            assert np.array_equal(sa.generate_greedy(0, ids, 8), sb.generate_greedy(0, ids, 8))
        finally:
            sa.close()
            sb.close()
    finally:
        a.close()
        b.close()
