"""Pins the CPU oracle to the reference's own golden vectors (CPU only).

Each test names the reference test it mirrors (path:line in wbrown/tinyoai).
"""
import json
import math
import struct

import numpy as np
import pytest

from oracle import oracle as oc
from tinyoai_b200.checkpoint import load_stablelm_dir


@pytest.mark.parametrize("name,dtype", [("q5_k", "Q5_K"), ("q6_k", "Q6_K"), ("q5_1", "Q5_1")])
def test_kquant_decode_bitwise(golden, name, dtype):
    """quant_k_test.go:14-48: decode of 4x2048 weights is bitwise equal to the
    gguf fixture, including partial-block reads."""
    raw = (golden / "kquant" / f"{name}.bin").read_bytes()
    want = np.frombuffer((golden / "kquant" / f"{name}-f32.bin").read_bytes(), dtype="<u4")
    got = oc.read_values(dtype, raw, 4, 2048)
    assert np.array_equal(got.view(np.uint32), want)
    for start, n in [(0, 1), (255, 3), (257, 511), (1000, 777)]:
        part = oc.read_values(dtype, raw, 4, 2048, start, n)
        assert np.array_equal(part.view(np.uint32), got[start:start + n].view(np.uint32))


@pytest.mark.parametrize("name,dtype", [("q5_k", "Q5_K"), ("q6_k", "Q6_K"), ("q5_1", "Q5_1"), ("q8_0", "Q8_0")])
def test_quant_products(golden, name, dtype):
    """quant_k_test.go:49-71: batched and single products vs a float64 sum of
    the decoded weights, within 2e-4 relative.

    The reference bound assumes the fused multiply-add its arm64 build emits.
    This oracle keeps every float32 operation separately rounded (the amd64
    code generation), and a float32 partial over a 512-wide tile then carries
    an error proportional to sum|x*w| rather than to the result, so one
    cancelling element of the K-quant fixture (|w| up to 4096) exceeds 2e-4 of
    |result|. The bound below adds 1e-6 * sum|x*w| (16 ulp of the magnitude)."""
    raw = (golden / "kquant" / f"{name}.bin").read_bytes()
    dec = np.frombuffer((golden / "kquant" / f"{name}-f32.bin").read_bytes(), dtype="<f4").reshape(4, 2048)
    for n in [1, 7, 128]:
        x = np.sin(np.arange(n * 2048) * 0.17).astype(np.float32).reshape(n, 2048)
        want = x.astype(np.float64) @ dec.astype(np.float64).T
        mag = np.abs(x.astype(np.float64)) @ np.abs(dec.astype(np.float64)).T
        got = oc.mul_batch(dtype, raw, 4, 2048, x)
        assert np.all(np.abs(got - want) <= 2e-4 * np.maximum(1, np.abs(want)) + 1e-6 * mag)
    got1 = oc.mul_rows(dtype, raw, 4, 2048, x[0])
    assert np.all(np.abs(got1 - want[0]) <= 2e-4 * np.maximum(1, np.abs(want[0])))


def test_q8_0_decode_matches_gguf(golden):
    """Q8_0 decode (matmul.go:24-34) is bitwise equal to gguf's dequantizer."""
    raw = (golden / "kquant" / "q8_0.bin").read_bytes()
    want = np.frombuffer((golden / "kquant" / "q8_0-f32.bin").read_bytes(), dtype="<u4")
    got = oc.read_values("Q8_0", raw, 4, 2048)
    assert np.array_equal(got.view(np.uint32), want)


def test_half_rounding_exhaustive():
    """kv_cache_test.go:12-41: every binary16 round trips; every midpoint
    rounds to even; the overflow boundary."""
    for h in range(65536):
        v = oc.half_to_float(h)
        got = oc.float_to_half(v)
        if math.isnan(v):
            assert got & 0x7FFF == 0x7E00
        else:
            assert got == h, hex(h)
    for h in range(0, 0x7BFF, 7):  # a spread of midpoints (the full sweep is in the GPU f16 test)
        mid = np.float32((np.float64(oc.half_to_float(h)) + np.float64(oc.half_to_float(h + 1))) / 2)
        want = h + (h & 1)
        assert oc.float_to_half(float(mid)) == want
        assert oc.float_to_half(float(-mid)) == want | 0x8000
    assert oc.float_to_half(65520) == 0x7C00 and oc.float_to_half(-65520) == 0xFC00 and oc.float_to_half(65504) == 0x7BFF


def test_rope_split_half_equation():
    """stablelm_test.go:168-179"""
    x = oc.stable_rotate([1, 2, 3, 4, 5, 6, 7, 8], 8, 4, 1, 10000)
    want = [math.cos(1) - 3 * math.sin(1), 2 * math.cos(.01) - 4 * math.sin(.01), 3 * math.cos(1) + math.sin(1),
            4 * math.cos(.01) + 2 * math.sin(.01), 5, 6, 7, 8]
    assert np.max(np.abs(x - np.array(want))) <= 1e-6


def test_rope_context_boundary(golden):
    """stablelm_test.go:181-205: rope.json at positions up to 8191, 5e-7."""
    ref = json.loads((golden / "stablelm_tiny" / "rope.json").read_text())
    for case in ref["cases"]:
        got = oc.stable_rotate(ref["input"], 128, 32, case["position"], 10000)
        assert np.max(np.abs(got - np.array(case["output"], np.float32))) <= 5e-7, case["position"]


@pytest.fixture(scope="module")
def tiny(golden):
    return load_stablelm_dir(golden / "stablelm_tiny")


def test_stablelm_reference_logits(tiny, golden):
    """stablelm_test.go:50-72: sequential forward logits within 3e-5 of the
    Transformers float32 reference."""
    cfg, tensors = tiny
    ref = json.loads((golden / "stablelm_tiny" / "expected.json").read_text())
    m = oc.StableLM(cfg, tensors, capacity=len(ref["input_ids"]))
    for pos, tok in enumerate(ref["input_ids"]):
        got = m.forward(tok, pos)
        assert np.max(np.abs(got - np.array(ref["logits"][pos], np.float32))) <= 3e-5


@pytest.mark.parametrize("half", [False, True])
def test_stablelm_prefill_matches_forward(tiny, half):
    """prefill_test.go:217-277: a batched prefill equals sequential forwards."""
    cfg, tensors = tiny
    ids = np.random.default_rng(1).integers(0, cfg["vocab_size"], 40).astype(np.int32)
    a = oc.StableLM(cfg, tensors, half_kv=half, capacity=64)
    for pos, t in enumerate(ids):
        want = a.forward(t, pos)
    b = oc.StableLM(cfg, tensors, half_kv=half, capacity=64)
    got = b.prefill(ids, chunk=16)
    assert np.max(np.abs(got - want)) <= 3e-5


def test_stablelm_greedy_generation_ids(tiny, golden):
    """stablelm_test.go:73-82: greedy generation from the fixture prompt
    reproduces the Transformers token ids."""
    cfg, tensors = tiny
    gen = json.loads((golden / "stablelm_tiny" / "generation.json").read_text())
    m = oc.StableLM(cfg, tensors, capacity=64)
    got, _ = m.greedy(np.array(gen["prompt_ids"], np.int32), len(gen["ids"]))
    assert list(got) == gen["ids"]


def test_llama_checkpoint_layout(golden):
    """load_test.go:40-72: stories260K consumes the checkpoint exactly; the
    forward yields finite logits."""
    raw = (golden / "llama" / "stories260K.bin").read_bytes()
    dim, hidden, layers, heads, kv_heads, vocab, seq = struct.unpack_from("<7i", raw)
    assert (dim, hidden, layers, heads, kv_heads, vocab, seq) == (64, 172, 5, 8, 4, 512, 512)
    m = oc.Llama(raw)
    logits = m.transformer(1, 0)
    assert logits.shape == (512,) and np.all(np.isfinite(logits))
    with pytest.raises(ValueError):
        oc.Llama(raw[:-4])


def test_sampling_candidates_order():
    """sampling.go:112-143: descending scores, ties by ascending id."""
    logits = np.array([0.5, 2.0, 2.0, -1.0, 0.5, 3.0, 2.0], np.float32)
    ids, vals = oc.sampling_candidates(logits, 4)
    assert list(ids) == [5, 1, 2, 6]
    ids, vals = oc.sampling_candidates(logits, 7)
    assert list(ids) == [5, 1, 2, 6, 0, 4, 3]


def test_summarize_logits():
    """logprobs.go:64-95: full-vocabulary normalisation, top entries with
    ties by lower id."""
    rng = np.random.default_rng(3)
    logits = rng.standard_normal(1000).astype(np.float32)
    logits[10] = logits[20] = 5.0
    ch, ids, vals = oc.summarize_logits(logits, 7, 5)
    z = np.log(np.sum(np.exp(logits.astype(np.float64) - 5.0))) + 5.0
    assert abs(ch - (float(logits[7]) - z)) < 1e-12
    assert list(ids[:2]) == [10, 20]
    order = np.lexsort((np.arange(1000), -logits.astype(np.float64)))[:5]
    assert list(ids) == list(order)


def test_penalties_known_answers():
    """sampling_test.go:14-31 TestProbabilityPenalties: repetition 2, presence
    0.1, frequency 0.2 over a 3-token window, and invariance to a constant
    logit offset."""
    kw = dict(repetition_penalty=2.0, presence_penalty=0.1, frequency_penalty=0.2, repetition_range=3)
    got = oc.penalized_logits(np.zeros(4, np.float32), [3, 1, 2, 1], **kw)
    want = [0.0, -math.log(2) - 0.1 - 0.4, -math.log(2) - 0.1 - 0.2, 0.0]
    assert np.all(np.abs(got - want) <= 1e-12)
    shifted = oc.penalized_logits(np.full(4, 20, np.float32), [3, 1, 2, 1], **kw)
    assert np.all(np.abs(shifted - got - 20) <= 1e-12)


def test_repetition_slope_and_range_known_answers():
    """sampling_test.go:35-57 TestRepetitionSlopeAndRange."""
    assert oc.repetition_weight(0, 5, 1) == 2 and oc.repetition_weight(2, 5, 1) == 1 and oc.repetition_weight(4, 5, 1) == 0
    assert oc.repetition_weight(1, 5, 3.33) > oc.repetition_weight(1, 5, 1)
    kw = dict(repetition_penalty=math.e, repetition_slope=1.0, repetition_range=5)
    got = oc.penalized_logits(np.zeros(5, np.float32), [4, 3, 2, 1, 0], **kw)
    assert np.all(np.abs(got - [-2, -1.5, -1, -0.5, 0]) <= 1e-12)
    got = oc.penalized_logits(np.zeros(5, np.float32), [1, 0], **kw)
    assert abs(got[1] + 1.5) <= 1e-12


def test_float64_candidates_match_full_sort():
    """sampling_test.go:105-149: the bounded shortlist equals the full sort
    (descending, ties by ascending id) for random, tied and monotone scores."""
    rng = np.random.default_rng(42)
    for size in (1, 300, 4096):
        for pattern in ("random", "ties", "ascending", "descending"):
            i = np.arange(size)
            v = {"random": rng.standard_normal(size), "ties": (i % 7).astype(np.float64),
                 "ascending": i.astype(np.float64), "descending": -i.astype(np.float64)}[pattern]
            order = sorted(range(size), key=lambda j: (-v[j], j))
            for k in (1, 12, 25, 64, 256):
                ids, vals = oc.sampling_candidates_f64(v, k)
                assert list(ids) == order[:k]
                assert np.array_equal(vals, v[order[:k]])
