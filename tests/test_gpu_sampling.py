"""Device probability rows and penalised sampling candidates against the
oracle's restatement of the reference (logprobs.go:64-95 summarizeLogits,
sampling.go:76-143 penalizedLogits + samplingCandidates).

- ForwardWithLogprobs (mlx.go:53-57): every position's chosen log probability
  and top alternatives equal summarizeLogits over the same device logits
  (ids exactly, values within 1e-9 absolute: float64 sums in another order),
  and the oracle's rows within the north-star logit tolerance.
- Penalised candidates: the same float32 logits row in, float64 scores out;
  the device applies the same chain of float64 subtractions per id, so ids
  and scores are bitwise equal to the oracle's.
"""
import numpy as np
import pytest

from oracle import oracle as oc
from tinyoai_b200 import BackendError, Model, _lib
from tinyoai_b200.synth import prompt_ids, synth_stablelm

pytestmark = pytest.mark.gpu

SMALL = dict(model_type="stablelm", vocab_size=2048, hidden_size=320, intermediate_size=864, num_hidden_layers=3,
             num_attention_heads=4, num_key_value_heads=4, max_position_embeddings=1024, layer_norm_eps=1e-5,
             rope_theta=10000.0, partial_rotary_factor=0.25, use_parallel_residual=True, use_qkv_bias=False,
             qk_layernorm=False, tie_word_embeddings=False, hidden_act="silu", bos_token_id=0, eos_token_id=0)


@pytest.fixture(scope="module")
def small():
    cfg, tensors = synth_stablelm(SMALL, "Q8_0", seed=29)
    m = Model.load_stablelm(cfg, tensors)
    yield cfg, tensors, m
    m.close()


def check_rows(chosen, ids, vals, logits_rows, targets, count):
    for i, row in enumerate(logits_rows):
        want_c, want_ids, want_vals = oc.summarize_logits(row, int(targets[i]), count)
        assert abs(chosen[i] - want_c) <= 1e-9, i
        # Equal ids wherever the order is not decided by a float64 sum's last bits.
        assert np.all(np.abs(vals[i] - want_vals) <= 1e-9), i
        gaps = np.abs(np.diff(want_vals)) > 1e-9
        same = ids[i] == want_ids
        assert np.all(same | ~np.concatenate([gaps, [True]]) | ~np.concatenate([[True], gaps])), i


def test_forward_logprobs_matches_summarize(small):
    cfg, tensors, m = small
    V = cfg["vocab_size"]
    ids = prompt_ids(600, V, seed=31)  # two prefill chunks: 512 + 88
    targets = np.concatenate([ids[1:], [7]]).astype(np.int32)
    count = 12
    s, ref = m.session(), m.session()
    try:
        chosen, top, vals, last = s.forward_logprobs(0, ids, targets, count)
        rows = ref.forward_all(0, ids)  # the same prefill, every position's logits row
        assert np.max(np.abs(last - rows[-1])) <= 1e-5
        # Log-probabilities over the same rows up to the head's summation order.
        for i in (0, 1, 255, 511, 512, 599):
            want_c, want_ids, want_vals = oc.summarize_logits(rows[i], int(targets[i]), count)
            assert abs(chosen[i] - want_c) <= 1e-4, i
            assert np.all(np.abs(vals[i] - want_vals) <= 1e-4), i
        # A one-token forward takes the decode path; its row is exact.
        c1, t1, v1, l1 = s.forward_logprobs(600, [5], [9], count)
        check_rows(c1, t1, v1, [l1], [9], count)
        assert s.length == 601
        # Against the oracle's own logits (decode forwards) at the f32 tolerance.
        ora = oc.StableLM(cfg, tensors, capacity=1024)
        try:
            for i in range(40):
                want = ora.forward(int(ids[i]), i)
                wc, _, _ = oc.summarize_logits(want, int(targets[i]), count)
                assert abs(chosen[i] - wc) <= 2 * 2e-3 * float(want.max() - want.min()), i
        finally:
            ora.close()
    finally:
        s.close()
        ref.close()


def test_forward_logprobs_rejects_bad_requests(small):
    cfg, tensors, m = small
    s = m.session()
    try:
        for targets, count in (([cfg["vocab_size"]], 4), ([1], 0), ([1], 257)):
            with pytest.raises(BackendError) as e:
                s.forward_logprobs(0, [3], targets, count)
            assert e.value.code == _lib.TCU_EINVAL
    finally:
        s.close()


PENALTIES = [
    dict(),
    dict(repetition_penalty=2.0, presence_penalty=0.1, frequency_penalty=0.2, repetition_range=3),
    dict(repetition_penalty=1.3, presence_penalty=-0.4, frequency_penalty=0.35, repetition_slope=3.33, repetition_range=64),
    dict(repetition_penalty=1.1, frequency_penalty=0.05, repetition_slope=1.0),  # whole history
]


@pytest.mark.parametrize("pen", PENALTIES)
def test_sample_candidates_bitwise(small, pen):
    cfg, tensors, m = small
    V = cfg["vocab_size"]
    rng = np.random.default_rng(37)
    s = m.session()
    try:
        logits = s.forward(0, prompt_ids(50, V, seed=41))
        # A history with repeats, ids out of range (skipped), and the top ids.
        top = np.argsort(-logits)[:20]
        hist = np.concatenate([rng.integers(0, V, 300), top, rng.choice(top, 40), [-1, V + 5]]).astype(np.int32)
        for k in (1, 40, 256):
            ids, scores = s.sample_candidates(hist, k, **pen)
            want_ids, want_scores = oc.sampling_candidates_f64(oc.penalized_logits(logits, hist, **pen), k)
            assert list(ids) == list(want_ids), k
            assert np.array_equal(scores, want_scores), k
    finally:
        s.close()


def test_batch_sample_candidates_bitwise(small):
    cfg, tensors, m = small
    V = cfg["vocab_size"]
    sessions = [m.session() for _ in range(5)]
    try:
        for i, ss in enumerate(sessions):
            ss.forward(0, prompt_ids(20 + 7 * i, V, seed=50 + i), want_logits=False)
        toks = np.array([3, 4, 5, 6, 7], np.int32)
        bt = m.batch(8)
        try:
            rows, _ = bt.forward(sessions, toks)
            rng = np.random.default_rng(43)
            hists = [rng.integers(0, V, n).astype(np.int32) for n in (0, 5, 50, 200, 700)]
            pens = [PENALTIES[i % len(PENALTIES)] for i in range(5)]
            ids, scores = bt.sample_candidates(hists, 40, pens)
            for i in range(5):
                want_ids, want_scores = oc.sampling_candidates_f64(oc.penalized_logits(rows[i], hists[i], **pens[i]), 40)
                assert list(ids[i]) == list(want_ids), i
                assert np.array_equal(scores[i], want_scores), i
        finally:
            bt.close()
    finally:
        for ss in sessions:
            ss.close()
