"""CUDA path vs the CPU oracle and the reference's golden vectors (B200).

Tolerances (north star): logits within max-abs 2e-3 of the oracle relative to
the logit range for float32 KV (1e-2 for float16 KV); greedy token streams
identical; the tiny Transformers fixture within 3e-5 absolute
(stablelm_test.go:65). Every call goes through the C ABI.
"""
import json

import numpy as np
import pytest

from oracle import oracle as oc
from tinyoai_b200 import BackendError, Model, _lib
from tinyoai_b200.checkpoint import load_stablelm_dir
from tinyoai_b200.synth import prompt_ids, synth_stablelm

pytestmark = pytest.mark.gpu

SMALL = dict(model_type="stablelm", vocab_size=2048, hidden_size=320, intermediate_size=864, num_hidden_layers=3,
             num_attention_heads=4, num_key_value_heads=4, max_position_embeddings=1024, layer_norm_eps=1e-5,
             rope_theta=10000.0, partial_rotary_factor=0.25, use_parallel_residual=True, use_qkv_bias=False,
             qk_layernorm=False, tie_word_embeddings=False, hidden_act="silu", bos_token_id=0, eos_token_id=0)
SMALL_GQA = dict(SMALL, num_key_value_heads=2)


def rel_err(got, want):
    return float(np.max(np.abs(got - want)) / max(1e-30, float(np.max(want) - np.min(want))))


@pytest.fixture(scope="module")
def tiny(golden):
    cfg, tensors = load_stablelm_dir(golden / "stablelm_tiny")
    m = Model.load_stablelm(cfg, tensors)
    yield cfg, tensors, m
    m.close()


@pytest.fixture(scope="module")
def small():
    cfg, tensors = synth_stablelm(SMALL, "Q8_0", seed=7)
    m = Model.load_stablelm(cfg, tensors)
    yield cfg, tensors, m
    m.close()


def test_tiny_reference_logits_decode(tiny, golden):
    """stablelm_test.go:50-72 on the GPU: one-token forwards (decode kernels)."""
    cfg, tensors, m = tiny
    ref = json.loads((golden / "stablelm_tiny" / "expected.json").read_text())
    s = m.session()
    try:
        for pos, tok in enumerate(ref["input_ids"]):
            got = s.forward(pos, [tok])
            assert np.max(np.abs(got - np.array(ref["logits"][pos], np.float32))) <= 3e-5
    finally:
        s.close()


def test_tiny_reference_logits_prefill(tiny, golden):
    """The same logits through the chunked prefill kernels, for every prefix length."""
    cfg, tensors, m = tiny
    ref = json.loads((golden / "stablelm_tiny" / "expected.json").read_text())
    ids = ref["input_ids"]
    for n in range(2, len(ids) + 1):
        s = m.session()
        try:
            got = s.forward(0, ids[:n])
            assert np.max(np.abs(got - np.array(ref["logits"][n - 1], np.float32))) <= 3e-5, n
        finally:
            s.close()


def test_tiny_greedy_generation(tiny, golden):
    """stablelm_test.go:73-82: the device greedy loop reproduces the fixture ids."""
    cfg, tensors, m = tiny
    gen = json.loads((golden / "stablelm_tiny" / "generation.json").read_text())
    s = m.session()
    try:
        got = s.generate_greedy(0, gen["prompt_ids"], len(gen["ids"]))
        assert list(got) == gen["ids"]
        assert s.length == len(gen["prompt_ids"]) + len(gen["ids"]) - 1
    finally:
        s.close()


@pytest.mark.parametrize("kv", ["f32", "f16"])
def test_small_q8_forward_vs_oracle(small, kv):
    """Prefill (GEMM path) then one-token forwards (GEMV path) vs the oracle's
    prefill + forward (prefill.go / stablelm.go) with the same KV precision."""
    cfg, tensors, m = small
    ids = prompt_ids(300, cfg["vocab_size"], seed=11)
    ora = oc.StableLM(cfg, tensors, half_kv=(kv == "f16"), capacity=cfg["max_position_embeddings"])
    want = ora.prefill(ids[:200])
    s = m.session(kv)
    tol = 2e-3 if kv == "f32" else 1e-2
    try:
        got = s.forward(0, ids[:200])
        assert rel_err(got, want) <= tol
        for pos in range(200, 260):
            want = ora.forward(ids[pos], pos)
            got = s.forward(pos, [ids[pos]])
            assert rel_err(got, want) <= tol, pos
        assert rel_err(got, want) <= 1e-4  # float32 accumulation, far inside the bound
    finally:
        s.close()
        ora.close()


def test_small_greedy_64_tokens(small):
    """Greedy streams identical for 64 tokens (north star), device loop vs oracle."""
    cfg, tensors, m = small
    ids = prompt_ids(96, cfg["vocab_size"], seed=5)
    ora = oc.StableLM(cfg, tensors, capacity=cfg["max_position_embeddings"])
    want, margins = ora.greedy(ids, 64, chunk=128)
    s = m.session()
    try:
        got = s.generate_greedy(0, ids, 64)
    finally:
        s.close()
        ora.close()
    bad = np.nonzero(got != want)[0]
    assert bad.size == 0, f"first divergence at step {bad[0]} (oracle top-2 margin {margins[bad[0]]:.3g})"


def test_gqa_model(golden):
    """Grouped-query attention (2 query heads per KV head) vs the oracle."""
    cfg, tensors = synth_stablelm(SMALL_GQA, "Q8_0", seed=3)
    m = Model.load_stablelm(cfg, tensors)
    ids = prompt_ids(70, cfg["vocab_size"], seed=2)
    ora = oc.StableLM(cfg, tensors, capacity=cfg["max_position_embeddings"])
    s = m.session()
    try:
        assert rel_err(s.forward(0, ids[:64]), ora.prefill(ids[:64])) <= 2e-3
        for pos in range(64, 70):
            assert rel_err(s.forward(pos, [ids[pos]]), ora.forward(ids[pos], pos)) <= 2e-3
    finally:
        s.close()
        m.close()
        ora.close()


def test_bf16_model():
    """BF16 weights (config 3's format) through the same kernels."""
    cfg, tensors = synth_stablelm(SMALL, "BF16", seed=4)
    m = Model.load_stablelm(cfg, tensors)
    ids = prompt_ids(40, cfg["vocab_size"], seed=9)
    ora = oc.StableLM(cfg, tensors, capacity=cfg["max_position_embeddings"])
    s = m.session("f16")
    ora16 = oc.StableLM(cfg, tensors, half_kv=True, capacity=cfg["max_position_embeddings"])
    try:
        assert rel_err(s.forward(0, ids[:32]), ora16.prefill(ids[:32])) <= 1e-2
        for pos in range(32, 40):
            assert rel_err(s.forward(pos, [ids[pos]]), ora16.forward(ids[pos], pos)) <= 1e-2
    finally:
        s.close()
        m.close()
        ora.close()
        ora16.close()


# K-quant super-blocks span 256 columns: hidden and MLP widths are multiples.
KQ_SMALL = dict(SMALL, hidden_size=256, intermediate_size=768)


@pytest.mark.parametrize("fmt", ["Q6_K", "Q5_K"])
@pytest.mark.parametrize("kv", ["f32", "f16"])
def test_kquant_model_vs_oracle(fmt, kv):
    """Q6_K / Q5_K weights (config 4's formats, quant_k.go:47-85) through the
    prefill GEMM and the per-token GEMV: logits against the oracle's
    decode-then-multiply at the north-star tolerance, then identical greedy
    streams."""
    cfg, tensors = synth_stablelm(KQ_SMALL, fmt, seed=31)
    m = Model.load_stablelm(cfg, tensors)
    ids = prompt_ids(120, cfg["vocab_size"], seed=13)
    ora = oc.StableLM(cfg, tensors, half_kv=(kv == "f16"), capacity=cfg["max_position_embeddings"])
    tol = 2e-3 if kv == "f32" else 1e-2
    s = m.session(kv)
    try:
        assert rel_err(s.forward(0, ids[:96]), ora.prefill(ids[:96])) <= tol
        for pos in range(96, 120):
            assert rel_err(s.forward(pos, [ids[pos]]), ora.forward(ids[pos], pos)) <= tol, pos
    finally:
        s.close()
        ora.close()
    ora = oc.StableLM(cfg, tensors, half_kv=(kv == "f16"), capacity=cfg["max_position_embeddings"])
    s = m.session(kv)
    try:
        want, margins = ora.greedy(ids[:64], 24, chunk=128)
        got = s.generate_greedy(0, ids[:64], 24)
    finally:
        s.close()
        ora.close()
        m.close()
    bad = np.nonzero(got != want)[0]
    assert bad.size == 0, f"first divergence at step {bad[0]} (oracle top-2 margin {margins[bad[0]]:.3g})"


@pytest.mark.parametrize("fmt", ["Q6_K", "Q5_K"])
def test_kquant_branches_match_sequential(fmt):
    """Config 4's shape in small: branches over a shared prefix with K-quant
    weights and f16 KV (batched rows) equal sessions that evaluated prefix +
    their own suffix."""
    cfg, tensors = synth_stablelm(KQ_SMALL, fmt, seed=37)
    m = Model.load_stablelm(cfg, tensors)
    count = 8
    ids = prompt_ids(70, cfg["vocab_size"], seed=43)
    rng = np.random.default_rng(7)
    steps = [rng.integers(3, cfg["vocab_size"], count).astype(np.int32) for _ in range(5)]
    s = m.session("f16")
    try:
        s.forward(0, ids, want_logits=False)
        br = s.new_branches(70, count)
        try:
            rows = [br.forward(t) for t in steps]
        finally:
            br.close()
        for b in range(count):
            ref = m.session("f16")
            try:
                want = ref.forward(0, np.concatenate([ids, [st[b] for st in steps]]))
            finally:
                ref.close()
            assert rel_err(rows[-1][b], want) <= 1e-4
    finally:
        s.close()
        m.close()


WIDE = dict(SMALL, hidden_size=512, intermediate_size=1024, num_hidden_layers=2)


@pytest.mark.parametrize("fmt", ["Q8_0", "Q6_K"])
def test_split_k_products_vs_oracle(fmt):
    """Tensor-core products with too few tiles for the GPU split K into slices
    summed in order (W1 with the GLU epilogue, the lm_head with the store
    epilogue; K = 512 is 8 stages): prefill and branch-step rows against the
    oracle at the north-star tolerance."""
    cfg, tensors = synth_stablelm(WIDE, fmt, seed=41)
    m = Model.load_stablelm(cfg, tensors)
    ids = prompt_ids(96, cfg["vocab_size"], seed=47)
    rng = np.random.default_rng(11)
    count = 24
    steps = [rng.integers(3, cfg["vocab_size"], count).astype(np.int32) for _ in range(2)]
    cap = cfg["max_position_embeddings"]
    s = m.session()
    try:
        ora = oc.StableLM(cfg, tensors, half_kv=False, capacity=cap)
        try:
            assert rel_err(s.forward(0, ids), ora.prefill(ids)) <= 2e-3
        finally:
            ora.close()
        br = s.new_branches(96, count)
        try:
            rows = [br.forward(t) for t in steps]
        finally:
            br.close()
        for b in (0, 11, 23):
            ora = oc.StableLM(cfg, tensors, half_kv=False, capacity=cap)
            try:
                want = ora.prefill(np.concatenate([ids, [st[b] for st in steps]]).astype(np.int32))
            finally:
                ora.close()
            assert rel_err(rows[-1][b], want) <= 2e-3, b
    finally:
        s.close()
        m.close()


def test_prefix_reuse_matches_cold(small):
    """prefill_test.go:68-109: extending or replacing a resident suffix gives
    the same logits as a cold evaluation."""
    cfg, tensors, m = small
    ids = prompt_ids(150, cfg["vocab_size"], seed=21)
    other = prompt_ids(50, cfg["vocab_size"], seed=22)
    warm = m.session()
    cold = m.session()
    try:
        warm.forward(0, ids[:100], want_logits=False)
        warm.forward(60, other, want_logits=False)  # replace the suffix after 60
        a = warm.forward(110, ids[110:120])
        b = cold.forward(0, np.concatenate([ids[:60], other, ids[110:120]]))
        assert np.max(np.abs(a - b)) <= 1e-5
        assert warm.length == 120
    finally:
        warm.close()
        cold.close()


def test_fork_diverges_independently(small):
    """sessions.go:36-72: the child shares the prefix; parent and child then
    generate independently and match cold sessions."""
    cfg, tensors, m = small
    ids = prompt_ids(77, cfg["vocab_size"], seed=31)  # 77 = 2 full pages + a partial tail
    parent = m.session()
    try:
        parent.forward(0, ids[:70], want_logits=False)
        child = parent.fork()
        try:
            a = child.forward(70, ids[70:77])
            b = parent.forward(70, ids[70:73][::-1])
            cold = m.session()
            try:
                ca = cold.forward(0, ids[:77])
                cb = cold.forward(70, ids[70:73][::-1])
            finally:
                cold.close()
            assert np.max(np.abs(a - ca)) <= 1e-5
            assert np.max(np.abs(b - cb)) <= 1e-5
            # after the parent wrote its tail, the child's history is unchanged
            assert np.max(np.abs(child.forward(76, [ids[76]]) - ca)) <= 1e-5
        finally:
            child.close()
    finally:
        parent.close()


@pytest.mark.parametrize("count", [3, 6])
def test_branches_match_sequential(small, count):
    """branches.go / mlx_branches.go:98-184: each branch equals a session that
    evaluated prefix + its own suffix (GEMV path for <= 4 branches, batched
    path above)."""
    cfg, tensors, m = small
    ids = prompt_ids(45, cfg["vocab_size"], seed=41)
    rng = np.random.default_rng(count)
    steps = [rng.integers(3, cfg["vocab_size"], count).astype(np.int32) for _ in range(4)]
    s = m.session()
    try:
        s.forward(0, ids, want_logits=False)
        br = s.new_branches(45, count)
        try:
            rows = [br.forward(t) for t in steps]
            am = br.argmax()
        finally:
            br.close()
        assert s.length == 45
        for b in range(count):
            ref = m.session()
            try:
                want = ref.forward(0, np.concatenate([ids, [st[b] for st in steps]]))
            finally:
                ref.close()
            assert np.max(np.abs(rows[-1][b] - want)) <= 1e-4
            assert am[b] == int(np.argmax(want))
        # the shared prefix is intact
        again = s.forward(44, [ids[44]])
        fresh = m.session()
        try:
            assert np.max(np.abs(again - fresh.forward(0, ids))) <= 1e-5
        finally:
            fresh.close()
    finally:
        s.close()


@pytest.mark.parametrize("kv", ["f32", "f16"])
@pytest.mark.parametrize("gqa", [False, True])
def test_branches_long_prefix(kv, gqa):
    """Branches over a 300-token prefix: the whole 64-position splits inside
    the shared pages are attended once for all branches (k_attn_shared), the
    rest per branch; each branch still equals a session that evaluated
    prefix + its own suffix."""
    cfg, tensors = synth_stablelm(SMALL_GQA if gqa else SMALL, "Q8_0", seed=19)
    m = Model.load_stablelm(cfg, tensors)
    count = 12
    ids = prompt_ids(300, cfg["vocab_size"], seed=47)
    rng = np.random.default_rng(3)
    steps = [rng.integers(3, cfg["vocab_size"], count).astype(np.int32) for _ in range(40)]
    s = m.session(kv)
    try:
        s.forward(0, ids, want_logits=False)
        br = s.new_branches(300, count)
        try:
            rows = [br.forward(t) for t in steps]
        finally:
            br.close()
        for b in (0, 5, count - 1):
            ref = m.session(kv)
            try:
                want = ref.forward(0, np.concatenate([ids, [st[b] for st in steps]]))
            finally:
                ref.close()
            assert rel_err(rows[-1][b], want) <= 1e-4
    finally:
        s.close()
        m.close()


@pytest.mark.parametrize("kv", ["f32", "f16"])
def test_batch_step_matches_single_sessions(small, kv):
    """Continuous batching: sessions at different positions (one a fork
    sharing its parent's pages) advance together through tcu_batch_forward;
    every row equals the same session stepped alone, for 6 greedy steps."""
    cfg, tensors, m = small
    lens = [9, 37, 64, 100, 131]
    prompts = [prompt_ids(n, cfg["vocab_size"], seed=60 + i) for i, n in enumerate(lens)]
    batch_s, alone = [], []
    try:
        for p in prompts:
            a, b = m.session(kv), m.session(kv)
            a.forward(0, p, want_logits=False)
            b.forward(0, p, want_logits=False)
            batch_s.append(a)
            alone.append(b)
        batch_s.append(batch_s[3].fork())  # shares the parent's pages until written
        alone_f = m.session(kv)
        alone_f.forward(0, prompts[3], want_logits=False)
        alone.append(alone_f)
        toks = np.array([p[-1] for p in prompts] + [prompts[3][-1]], np.int32)
        bt = m.batch(8)
        try:
            for step in range(6):
                rows, ids = bt.forward(batch_s, toks)
                for i, s in enumerate(alone):
                    want = s.forward(s.length, [toks[i]])
                    assert rel_err(rows[i], want) <= 1e-4, (step, i)
                    assert ids[i] == int(np.argmax(want))
                assert [s.length for s in batch_s] == [s.length for s in alone]
                toks = ids.astype(np.int32)
        finally:
            bt.close()
    finally:
        for s in batch_s + alone:
            s.close()


def test_shortlist_matches_oracle(small):
    """sampling.go:112-143 ordering and logprobs.go:64-95 normaliser on device."""
    cfg, tensors, m = small
    s = m.session()
    try:
        logits = s.forward(0, prompt_ids(20, cfg["vocab_size"], seed=51))
        ids, vals, lse = s.shortlist(40)
        want_ids, want_vals = oc.sampling_candidates(logits, 40)
        assert list(ids) == list(want_ids)
        assert np.array_equal(vals, want_vals.astype(np.float32))
        ch, _, _ = oc.summarize_logits(logits, 0, 1)
        assert abs((float(logits[0]) - lse) - ch) <= 1e-9
    finally:
        s.close()


def test_invalid_requests(small):
    """mlx_native.go:328-335: bad tokens and prefixes are rejected before
    dispatch; a failed forward leaves the session usable."""
    cfg, tensors, m = small
    s = m.session()
    try:
        with pytest.raises(BackendError) as e:
            s.forward(0, [cfg["vocab_size"]])
        assert e.value.code == _lib.TCU_EINVAL
        s.forward(0, [5, 6, 7], want_logits=False)
        with pytest.raises(BackendError):
            s.forward(4, [1])
        with pytest.raises(BackendError):
            s.forward(0, np.zeros(cfg["max_position_embeddings"] + 1, np.int32))
        assert s.length == 3
        assert s.limit_cache(2) is True and s.length == 0
        s.forward(0, [5, 6, 7], want_logits=False)
        assert s.set_kv_bits(16) is True and s.length == 0
    finally:
        s.close()


@pytest.fixture(scope="module")
def stories(golden):
    raw = (golden / "llama" / "stories260K.bin").read_bytes()
    m = Model.load_llama(raw)
    yield raw, m
    m.close()


def test_llama_logits_vs_oracle(stories):
    """model.go:407-481 (config 1): every position's logits, decode path and
    the all-logits prefill path."""
    raw, m = stories
    ora = oc.Llama(raw)
    ids = prompt_ids(32, 512, seed=0)
    s = m.session()
    try:
        rows = s.forward_all(0, ids)
        s2 = m.session()
        try:
            for pos, t in enumerate(ids):
                want = ora.transformer(t, pos)
                assert rel_err(rows[pos], want) <= 2e-3, pos
                got = s2.forward(pos, [t])
                assert rel_err(got, want) <= 2e-3, pos
                assert np.max(np.abs(got - want)) <= 1e-4
        finally:
            s2.close()
    finally:
        s.close()
        ora.close()


def test_llama_greedy_128(stories):
    """Config 1: 32 seeded prompt ids, greedy 128 tokens, identical to the oracle."""
    raw, m = stories
    ora = oc.Llama(raw)
    ids = prompt_ids(32, 512, seed=0)
    want = ora.greedy(ids, 128)
    s = m.session()
    try:
        got = s.generate_greedy(0, ids, 128)
    finally:
        s.close()
        ora.close()
    assert list(got) == list(want)


def test_stage_profile(small):
    """Stage timing (stableProfile, stablelm.go:229-250): every stage of a
    prefill + greedy decode is counted once per launch; results are unchanged."""
    cfg, tensors, m = small
    ids = prompt_ids(40, cfg["vocab_size"], seed=61)
    s = m.session()
    try:
        want = s.generate_greedy(0, ids, 6)
        s.profile(True)
        got = s.generate_greedy(0, ids, 6)
        prof = s.profile_read(reset=True)
        s.profile(False)
        assert list(got) == list(want)
        L = cfg["num_hidden_layers"]
        assert prof["prefill_projection"][0] == 2 * L
        assert prof["prefill_attention"][0] == L
        if prof["decode_step"][0]:
            # Persistent decode: one launch per decoded token (steps - 1),
            # with layers and head inside it.
            assert prof["decode_step"][0] == 5 and prof["decode_step"][1] > 0
            assert prof["norm_qkv_gate_up"][0] == 0 and prof["attention"][0] == 0
            assert prof["head"][0] == 1  # the prefill's head
        else:
            assert prof["norm_qkv_gate_up"][0] == 5 * L  # five decode forwards (steps - 1)
            assert prof["attention"][0] == 5 * L and prof["out_down_residual"][0] == 5 * L
            assert prof["head"][0] == 6  # prefill head + five decode heads
        assert all(ms >= 0 for _, ms in prof.values())

        # A single-token forward takes the per-layer kernels.
        s.profile(True)
        s.forward(len(ids) + 4, [int(got[-1])])
        prof = s.profile_read(reset=True)
        s.profile(False)
        assert prof["norm_qkv_gate_up"][0] == L and prof["attention"][0] == L
        assert prof["out_down_residual"][0] == L and prof["head"][0] == 1
        assert prof["norm_qkv_gate_up"][1] > 0 and prof["decode_step"][0] == 0
    finally:
        s.close()


@pytest.mark.parametrize("fmt", ["Q8_0", "BF16", "Q6_K", "Q5_K"])
def test_tensor_core_prefill_matches_cuda_core_prefill(monkeypatch, fmt):
    """The tcgen05 prefill GEMM against the CUDA-core GEMM on the same model:
    Q8_0 weights as an exact binary16 pair, BF16 weights against a
    three-piece bfloat16 split of the activations, K-quant weights decoded in
    float32 and split into a binary16 pair (22 significant bits); float32
    accumulation. Logits of a 96-token prefill within 1e-4 of the logit
    range, identical greedy continuations."""
    cfg, tensors = synth_stablelm(KQ_SMALL if fmt in ("Q6_K", "Q5_K") else SMALL, fmt, seed=23)
    ids = prompt_ids(96, cfg["vocab_size"], seed=5)
    out = {}
    for mode in ("simt", "tc"):
        if mode == "simt":
            monkeypatch.setenv("TCU_GEMM", "simt")
        else:
            monkeypatch.delenv("TCU_GEMM", raising=False)
        m = Model.load_stablelm(cfg, tensors)
        s = m.session()
        try:
            out[mode] = (s.forward_all(0, ids), s.generate_greedy(0, ids, 16))
        finally:
            s.close()
            m.close()
    (a, ga), (b, gb) = out["simt"], out["tc"]
    assert rel_err(b, a) <= 1e-4
    assert list(ga) == list(gb)
