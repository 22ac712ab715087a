"""Failure detection on the GPU without a fault: a bounded device wait that
runs out is reported as TCU_ETIMEOUT, and the session's resident KV is
discarded (mlx.go:171-176 invalidates the prefix after a native failure).

TCU_TEST_HOLD_ARRIVAL=<layer> makes the first launch of the persistent decode
step (k_decode_mega) hold back one merged-head arrival in that layer, so the
out-projection wait of every CTA polls a count that never completes until its
limit (about one second of %globaltimer). The kernel then sets its error word
and runs to its end: the call returns, the host reads the word, and the same
session (and the context) keep working afterwards.
"""
import numpy as np
import pytest

from tinyoai_b200 import BackendError, Model, _lib
from tinyoai_b200.synth import prompt_ids, synth_stablelm

pytestmark = pytest.mark.gpu

SMALL = dict(model_type="stablelm", vocab_size=2048, hidden_size=320, intermediate_size=864, num_hidden_layers=3,
             num_attention_heads=4, num_key_value_heads=4, max_position_embeddings=1024, layer_norm_eps=1e-5,
             rope_theta=10000.0, partial_rotary_factor=0.25, use_parallel_residual=True, use_qkv_bias=False,
             qk_layernorm=False, tie_word_embeddings=False, hidden_act="silu", bos_token_id=0, eos_token_id=0)


def test_expired_device_wait_reports_timeout_and_invalidates_kv(monkeypatch):
    cfg, tensors = synth_stablelm(SMALL, "Q8_0", seed=13)
    m = Model.load_stablelm(cfg, tensors)
    ids = prompt_ids(40, cfg["vocab_size"], seed=17)
    s = m.session()
    try:
        # The persistent step serves this model (one launch per decoded token).
        s.profile(True)
        want = s.generate_greedy(0, ids, 8)
        prof = s.profile_read(reset=True)
        s.profile(False)
        assert prof["decode_step"][0] == 7
        assert s.length == len(ids) + 7

        monkeypatch.setenv("TCU_TEST_HOLD_ARRIVAL", "1")
        with pytest.raises(BackendError) as e:
            s.generate_greedy(0, ids, 8)
        assert e.value.code == _lib.TCU_ETIMEOUT
        assert "bounded device wait" in str(e.value)
        assert s.length == 0  # resident KV discarded
        monkeypatch.delenv("TCU_TEST_HOLD_ARRIVAL")

        # The kernel ended normally: the same session evaluates again, with
        # the results of the first run.
        got = s.generate_greedy(0, ids, 8)
        assert list(got) == list(want)
        other = m.session()
        try:
            assert np.array_equal(other.generate_greedy(0, ids, 8), want)
        finally:
            other.close()
    finally:
        s.close()
        m.close()
