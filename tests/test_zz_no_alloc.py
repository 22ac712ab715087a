"""tcu_shortlist_static, the shortlist entry point that allocates no device
memory, against tcu_session_shortlist on the same logits rows.

Both run the same kernel, so ids and values must match exactly and the
float64 log-sum-exp within 1e-9 (the tolerance of the shortlist parity test).
This file is named to be collected last: the entry point must also work
after every other GPU test has run in the same process.
"""
import ctypes as C

import numpy as np
import pytest

from tinyoai_b200 import BackendError, Model, _lib
from tinyoai_b200.synth import prompt_ids, synth_stablelm

pytestmark = pytest.mark.gpu

SMALL = dict(model_type="stablelm", vocab_size=2048, hidden_size=320, intermediate_size=864, num_hidden_layers=3,
             num_attention_heads=4, num_key_value_heads=4, max_position_embeddings=1024, layer_norm_eps=1e-5,
             rope_theta=10000.0, partial_rotary_factor=0.25, use_parallel_residual=True, use_qkv_bias=False,
             qk_layernorm=False, tie_word_embeddings=False, hidden_act="silu", bos_token_id=0, eos_token_id=0)


def shortlist_static(dev_logits, vocab, k, device=0):
    ids = np.full(k, -1, np.int32)
    vals = np.full(k, np.nan, np.float32)
    lse = C.c_double()
    n = C.c_int32()
    _lib.check(_lib.lib().tcu_shortlist_static(device, C.c_void_p(dev_logits.data_ptr()), vocab, k, None,
                                               ids.ctypes.data_as(C.POINTER(C.c_int32)),
                                               vals.ctypes.data_as(C.POINTER(C.c_float)), C.byref(lse), C.byref(n)))
    return ids[:n.value], vals[:n.value], lse.value


def test_static_shortlist_matches_session_shortlist():
    import torch

    cfg, tensors = synth_stablelm(SMALL, "Q8_0", seed=11)
    m = Model.load_stablelm(cfg, tensors)
    s = m.session()
    try:
        V = cfg["vocab_size"]
        ids_a = prompt_ids(24, V, seed=3)
        logits_a = s.forward(0, ids_a)
        want_a = s.shortlist(40)
        logits_b = s.forward(len(ids_a), prompt_ids(5, V, seed=4))
        want_b = s.shortlist(17)
        assert not np.array_equal(logits_a, logits_b)

        dev_a = torch.from_numpy(logits_a).to("cuda:0")
        dev_b = torch.from_numpy(logits_b).to("cuda:0")
        torch.cuda.synchronize()
        # Two calls in a row (the first does the per-device set-up), then the
        # first row again: each result must be that row's own.
        for dev, k, want in ((dev_a, 40, want_a), (dev_b, 17, want_b), (dev_a, 40, want_a)):
            got_ids, got_vals, got_lse = shortlist_static(dev, V, k)
            assert list(got_ids) == list(want[0])
            assert np.array_equal(got_vals, want[1])
            assert abs(got_lse - want[2]) <= 1e-9

        # Sizes beyond the static scratch are rejected before any launch.
        for k, vocab in ((257, V), (8, (1 << 20) + 1), (0, V)):
            with pytest.raises(BackendError) as e:
                shortlist_static(dev_a, vocab, k)
            assert e.value.code == _lib.TCU_EINVAL
        with pytest.raises(BackendError) as e:
            shortlist_static(dev_a, V, 300)
        assert "256" in str(e.value)
        # A row in host memory is not accepted.
        host = np.zeros(V, np.float32)
        rc = _lib.lib().tcu_shortlist_static(0, host.ctypes.data_as(C.c_void_p), V, 4, None,
                                             (C.c_int32 * 4)(), (C.c_float * 4)(), C.byref(C.c_double()),
                                             C.byref(C.c_int32()))
        assert rc == _lib.TCU_EINVAL

        # A stream under capture is refused before any work is queued (the
        # call synchronises and copies to host memory); the capture itself
        # stays valid and the next plain call works.
        side = torch.cuda.Stream()
        graph = torch.cuda.CUDAGraph()
        mark = torch.zeros(1, device="cuda:0")
        with torch.cuda.graph(graph, stream=side, capture_error_mode="relaxed"):
            rc = _lib.lib().tcu_shortlist_static(0, C.c_void_p(dev_a.data_ptr()), V, 4, C.c_void_p(side.cuda_stream),
                                                 (C.c_int32 * 4)(), (C.c_float * 4)(), C.byref(C.c_double()),
                                                 C.byref(C.c_int32()))
            mark.add_(1)
        assert rc == _lib.TCU_EINVAL
        graph.replay()
        torch.cuda.synchronize()
        assert float(mark[0]) == 1.0
        del graph
        got_ids, got_vals, _ = shortlist_static(dev_a, V, 40)
        assert list(got_ids) == list(want_a[0])
    finally:
        s.close()
        m.close()
