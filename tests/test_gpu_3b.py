"""Full-size parity: the Clio-shaped 3B StableLM with Q8_0 weights (config 2's
model) against the CPU oracle on the same bytes. The oracle restates the Go
scalar path in float64-accumulating C, so the prompt is kept short (the oracle
needs ~2.9 G multiply-adds per token); the greedy stream, the logits of the
prefill and the logits after decoding are compared."""
import numpy as np
import pytest

from oracle import oracle as oc
from tinyoai_b200 import Model
from tinyoai_b200.synth import CLIO_3B, prompt_ids, synth_stablelm

pytestmark = [pytest.mark.gpu, pytest.mark.slow]


def test_clio_3b_q8_greedy_parity():
    import os
    cfg, tensors = synth_stablelm(CLIO_3B, "Q8_0", seed=0, device="cuda")
    oc.set_threads(os.cpu_count() or 1)
    ids = prompt_ids(24, cfg["vocab_size"], seed=0)
    steps = 24
    ora = oc.StableLM(cfg, tensors, capacity=64)
    want_pf = ora.prefill(ids)
    ora.close()
    ora = oc.StableLM(cfg, tensors, capacity=64)
    want, margins = ora.greedy(ids, steps)
    last = ora.forward(int(want[-1]), len(ids) + steps - 1)
    ora.close()
    model = Model.load_stablelm(cfg, tensors)
    del tensors
    try:
        s = model.session()
        try:
            got_pf = s.forward(0, ids)
            rng = float(want_pf.max() - want_pf.min())
            assert np.max(np.abs(got_pf - want_pf)) <= 2e-3 * rng
            got = s.generate_greedy(0, ids, steps)
            bad = np.nonzero(got != want)[0]
            assert bad.size == 0, f"divergence at {bad[0]} (oracle margin {margins[bad[0]]:.3g})"
            got_last = s.forward(len(ids) + steps - 1, [int(got[-1])])
            assert np.max(np.abs(got_last - last)) <= 2e-3 * float(last.max() - last.min())
        finally:
            s.close()
    finally:
        model.close()
