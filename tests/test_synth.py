"""Synthetic checkpoint generator and the bench's algorithmic byte counts (CPU)."""
import numpy as np

from oracle import oracle as oc
from tinyoai_b200.synth import CLIO_3B, prompt_ids, synth_stablelm


def test_q8_0_encoding_round_trips():
    """The Q8_0 bytes decode (matmul.go:24-34) to within half a quantisation
    step of the drawn values, and are deterministic per seed."""
    import torch
    cfg = dict(CLIO_3B, num_hidden_layers=1, hidden_size=64, intermediate_size=96, num_attention_heads=2,
               num_key_value_heads=2, vocab_size=128)
    c1, t1 = synth_stablelm(cfg, "Q8_0", seed=3)
    _, t2 = synth_stablelm(cfg, "Q8_0", seed=3)
    dt, shape, payload = t1["model.layers.0.self_attn.q_proj.weight"]
    assert dt == "Q8_0" and shape == (64, 64) and payload.nbytes == 64 * 64 // 32 * 34
    assert np.array_equal(payload, t2["model.layers.0.self_attn.q_proj.weight"][2])
    g = torch.Generator().manual_seed(3 * 1000003 + 2)  # tensor index 2 = q_proj of layer 0
    x = (torch.randn((64, 64), generator=g) * 0.02).numpy()
    dec = oc.read_values("Q8_0", payload, 64, 64).reshape(64, 64)
    step = np.abs(x).reshape(64, 2, 32).max(-1, keepdims=True) / 127
    # half a step, plus the binary16 rounding of the scale (127 * 2^-11 of a step)
    assert np.all(np.abs(dec - x).reshape(64, 2, 32) <= step * (0.5 + 127 / 2048) + 1e-7)


def test_prompt_ids():
    a = prompt_ids(512, 65536, seed=0)
    assert a.dtype == np.int32 and a.min() >= 3 and a.max() < 65536
    assert np.array_equal(a, prompt_ids(512, 65536, seed=0))


def test_decode_bytes_of_the_3b_shape():
    """Q8_0 weight bytes per decoded token: 2.874 GB for the 3B shape."""
    import bench
    total, w1 = bench.decode_bytes(CLIO_3B, -1)
    assert abs(total / 1e9 - 2.874) < 0.005
    assert w1 == (2560 * 3 + 2 * 6912) * 2560 * 34 // 32
