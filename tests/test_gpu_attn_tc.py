"""Shared-prefix attention on the tensor cores (k_attn_shared_tc) against the
float32 CUDA-core kernel it replaces (k_attn_shared, TCU_ATTN=simt) and
against sessions that evaluated prefix + their own suffix
(mlx_branches.go:98-184). Binary16 KV: the keys and values are exact
tensor-core operands, the queries and softmax weights exact binary16 pairs
to 22 bits, so the two kernels agree to float32 accumulation-order noise.

Shapes: 64 branches over a 1,100-token prefix (one 128-row tile of query
rows with or without grouped heads, 17 shared splits of 64 positions), and
70 branches with two query heads per KV head (140 rows: a full and a ragged
tile).
"""
import numpy as np
import pytest

from tinyoai_b200 import Model
from tinyoai_b200.synth import prompt_ids, synth_stablelm

pytestmark = pytest.mark.gpu

SMALL = dict(model_type="stablelm", vocab_size=2048, hidden_size=320, intermediate_size=864, num_hidden_layers=3,
             num_attention_heads=4, num_key_value_heads=4, max_position_embeddings=2048, layer_norm_eps=1e-5,
             rope_theta=10000.0, partial_rotary_factor=0.25, use_parallel_residual=True, use_qkv_bias=False,
             qk_layernorm=False, tie_word_embeddings=False, hidden_act="silu", bos_token_id=0, eos_token_id=0)
PREFIX = 1100


def rel_err(got, want):
    return float(np.max(np.abs(got - want)) / max(1e-30, float(np.max(want) - np.min(want))))


def run_branches(m, ids, steps, count):
    s = m.session("f16")
    try:
        s.forward(0, ids, want_logits=False)
        br = s.new_branches(len(ids), count)
        try:
            rows = [br.forward(t) for t in steps]
            am = br.argmax()
        finally:
            br.close()
    finally:
        s.close()
    return rows, am


@pytest.mark.parametrize("kvh,count", [(4, 64), (2, 64), (2, 70)])
def test_shared_attention_tc_matches_cuda_cores(monkeypatch, kvh, count):
    cfg, tensors = synth_stablelm(dict(SMALL, num_key_value_heads=kvh), "Q8_0", seed=211 + kvh)
    ids = prompt_ids(PREFIX, cfg["vocab_size"], seed=223)
    rng = np.random.default_rng(count)
    steps = [rng.integers(3, cfg["vocab_size"], count).astype(np.int32) for _ in range(3)]
    monkeypatch.setenv("TCU_ATTN", "simt")
    ms = Model.load_stablelm(cfg, tensors)
    monkeypatch.delenv("TCU_ATTN")
    mt = Model.load_stablelm(cfg, tensors)
    try:
        rows_s, am_s = run_branches(ms, ids, steps, count)
        rows_t, am_t = run_branches(mt, ids, steps, count)
        worst = max(rel_err(t, s) for t, s in zip(rows_t, rows_s))
        print(f"KV heads {kvh}, {count} branches: worst rel err tensor cores vs CUDA cores {worst:.3g}")
        assert worst <= 2e-5
        for b in (0, count // 2, count - 1):
            ref = mt.session("f16")
            try:
                want = ref.forward(0, np.concatenate([ids, [st[b] for st in steps]]))
            finally:
                ref.close()
            assert rel_err(rows_t[-1][b], want) <= 1e-4
            srt = np.sort(want)
            if srt[-1] - srt[-2] > 1e-3 * (srt[-1] - srt[0]):
                assert am_t[b] == int(np.argmax(want))
    finally:
        ms.close()
        mt.close()


@pytest.mark.parametrize("kvh", [4, 2])
def test_prefill_attention_tc_matches_cuda_cores(monkeypatch, kvh):
    """Causal prefill attention (k_attn_prefill_tc vs k_attn_prefill): a
    700-token prompt (a 512-token chunk and a ragged one starting at 512),
    then 77 more tokens at position 700; every row's logits."""
    cfg, tensors = synth_stablelm(dict(SMALL, num_key_value_heads=kvh), "Q8_0", seed=227 + kvh)
    ids = prompt_ids(777, cfg["vocab_size"], seed=229)
    monkeypatch.setenv("TCU_ATTN", "simt")
    ms = Model.load_stablelm(cfg, tensors)
    monkeypatch.delenv("TCU_ATTN")
    mt = Model.load_stablelm(cfg, tensors)
    try:
        got = {}
        for name, m in (("simt", ms), ("tc", mt)):
            s = m.session("f16")
            try:
                got[name] = (s.forward_all(0, ids[:700]), s.forward_all(700, ids[700:]))
            finally:
                s.close()
        for part in (0, 1):
            t, c = got["tc"][part], got["simt"][part]
            worst = max(rel_err(t[i], c[i]) for i in range(len(t)))
            print(f"KV heads {kvh}, part {part}: worst row rel err tensor cores vs CUDA cores {worst:.3g}")
            assert worst <= 2e-5
    finally:
        ms.close()
        mt.close()
