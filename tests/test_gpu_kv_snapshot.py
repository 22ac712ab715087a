"""KV snapshots in the reference's TNYKV001 format (cache_file.go:16-258).

A session's resident positions are saved, the file is read back by an
independent reader of the format (magic, length-prefixed JSON header as Go's
encoding/json writes it, payload in layer -> KV head -> keys, values order,
SHA-256 trailer), restored into a fresh session whose next forward must equal
the original's bit for bit, and the damaged or mismatched files LoadCache
refuses are refused here too, leaving the session as it was.
"""
import hashlib
import json
import struct

import numpy as np
import pytest

from tinyoai_b200 import BackendError, Model
from tinyoai_b200.synth import prompt_ids, synth_stablelm

pytestmark = pytest.mark.gpu

SMALL = dict(model_type="stablelm", vocab_size=2048, hidden_size=320, intermediate_size=864, num_hidden_layers=3,
             num_attention_heads=4, num_key_value_heads=2, max_position_embeddings=1024, layer_norm_eps=1e-5,
             rope_theta=10000.0, partial_rotary_factor=0.25, use_parallel_residual=True, use_qkv_bias=False,
             qk_layernorm=False, tie_word_embeddings=False, hidden_act="silu", bos_token_id=0, eos_token_id=0)
IDENT = hashlib.sha256(b"model identity of the test checkpoint").digest()


@pytest.fixture(scope="module")
def model():
    cfg, tensors = synth_stablelm(SMALL, "Q8_0", seed=83)
    m = Model.load_stablelm(cfg, tensors)
    yield cfg, m
    m.close()


def read_snapshot(path):
    raw = path.read_bytes()
    assert raw[:8] == b"TNYKV001"
    (n,) = struct.unpack_from("<I", raw, 8)
    header = json.loads(raw[12:12 + n])
    assert hashlib.sha256(raw[:-32]).digest() == raw[-32:]
    return header, raw[12 + n:-32]


@pytest.mark.parametrize("kv", ["f32", "f16"])
def test_snapshot_round_trip(model, tmp_path, kv):
    cfg, m = model
    ids = prompt_ids(150, cfg["vocab_size"], seed=89)
    a = m.session(kv)
    b = m.session(kv)
    try:
        a.forward(0, ids, want_logits=False)
        path = tmp_path / "kv.bin"
        a.save_cache(path, IDENT, ids)
        header, payload = read_snapshot(path)
        assert header == {"model_sha256": list(IDENT), "float16": kv == "f16", "tokens": [int(x) for x in ids]}
        hd = cfg["hidden_size"] // cfg["num_attention_heads"]
        es = 2 if kv == "f16" else 4
        assert len(payload) == cfg["num_hidden_layers"] * 2 * cfg["num_key_value_heads"] * hd * len(ids) * es
        b.forward(0, prompt_ids(40, cfg["vocab_size"], seed=97), want_logits=False)  # some other context first
        got = b.load_cache(path, IDENT)
        assert list(got) == list(ids) and b.length == len(ids)
        nxt = [int(ids[0])]
        assert np.array_equal(b.forward(len(ids), nxt), a.forward(len(ids), nxt))
        # A save of the restored session (one position longer) holds the same
        # KV for the first positions: the payload survived the round trip.
        b2 = tmp_path / "kv2.bin"
        b.save_cache(b2, IDENT, np.concatenate([ids, nxt]))
        T, L, KVH = len(ids), cfg["num_hidden_layers"], cfg["num_key_value_heads"]
        dt = np.uint16 if kv == "f16" else np.uint32
        first = np.frombuffer(payload, dt).reshape(L, KVH, 2, T, hd)
        second = np.frombuffer(read_snapshot(b2)[1], dt).reshape(L, KVH, 2, T + 1, hd)
        assert np.array_equal(second[:, :, :, :T], first)
    finally:
        a.close()
        b.close()


def test_snapshot_rejects(model, tmp_path):
    cfg, m = model
    ids = prompt_ids(70, cfg["vocab_size"], seed=101)
    a = m.session("f32")
    b = m.session("f32")
    h = m.session("f16")
    try:
        a.forward(0, ids, want_logits=False)
        path = tmp_path / "kv.bin"
        a.save_cache(path, IDENT, ids)
        raw = path.read_bytes()
        b.forward(0, ids[:10], want_logits=False)
        cases = {
            "does not match checkpoint": (raw, hashlib.sha256(b"another model").digest(), b),
            "precision": (raw, IDENT, h),
            "checksum mismatch": (raw[:-40] + bytes([raw[-40] ^ 1]) + raw[-39:], IDENT, b),  # a payload byte
            "size": (raw[:-10], IDENT, b),
            "unsupported KV cache format": (b"TNYKV002" + raw[8:], IDENT, b),
        }
        for message, (data, ident, sess) in cases.items():
            p = tmp_path / "bad.bin"
            p.write_bytes(data)
            before = sess.length
            with pytest.raises(BackendError) as e:
                sess.load_cache(p, ident)
            assert message in str(e.value), (message, str(e.value))
            assert sess.length == before
        with pytest.raises(BackendError):
            a.save_cache(tmp_path / "x.bin", IDENT, ids[:-1])  # tokens must cover the resident positions
        # An empty context saves with null tokens and restores to length 0.
        e0 = m.session("f32")
        try:
            e0.save_cache(tmp_path / "empty.bin", IDENT, [])
            assert read_snapshot(tmp_path / "empty.bin")[0]["tokens"] is None
            assert len(b.load_cache(tmp_path / "empty.bin", IDENT)) == 0 and b.length == 0
        finally:
            e0.close()
    finally:
        a.close()
        b.close()
        h.close()
