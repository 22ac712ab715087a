"""Head-parallel tensor parallelism on the host (two gloo ranks on CPU).

Each rank asks the library for its share (tcu_tp_plan, no GPU needed): the
shares must partition the query heads, the KV heads and the MLP rows, every
rank's query heads must use only its own KV heads (grouped-query attention),
and the per-rank arithmetic the library runs -- the out + down partial of its
heads and MLP rows, summed over the ranks by an all-reduce -- must equal the
whole layer's parallel residual (stablelm.go:365-377). The layer is
evaluated in float64 with numpy, so the two agree to rounding.
"""
import os
import socket

import numpy as np
import pytest
import torch.multiprocessing as mp

from tinyoai_b200 import BackendError, _lib, tp_plan

CFG = dict(vocab_size=64, hidden_size=96, intermediate_size=192, num_hidden_layers=1, num_attention_heads=6,
           num_key_value_heads=2, max_position_embeddings=64, layer_norm_eps=1e-5, rope_theta=10000.0,
           partial_rotary_factor=0.25)


def free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def layer_weights():
    rng = np.random.default_rng(3)
    d, ff, H, KVH = CFG["hidden_size"], CFG["intermediate_size"], CFG["num_attention_heads"], CFG["num_key_value_heads"]
    hd = d // H
    w = {k: rng.standard_normal(s) * 0.1 for k, s in dict(q=(d, d), k=(KVH * hd, d), v=(KVH * hd, d), o=(d, d), g=(ff, d),
                                                         u=(ff, d), dn=(d, ff)).items()}
    x = rng.standard_normal(d)
    hist_k = rng.standard_normal((7, KVH * hd))  # earlier positions' keys / values
    hist_v = rng.standard_normal((7, KVH * hd))
    return w, x, hist_k, hist_v


def layer_partial(w, x, hist_k, hist_v, h0, nh, kv0, nkv, f0, nf):
    """out + down of query heads [h0, h0+nh) and MLP rows [f0, f0+nf)."""
    d, H, KVH = CFG["hidden_size"], CFG["num_attention_heads"], CFG["num_key_value_heads"]
    hd, group = d // H, H // KVH
    n = (x - x.mean()) / np.sqrt(x.var() + 1e-5)
    q, k, v = w["q"] @ n, w["k"] @ n, w["v"] @ n
    keys = np.vstack([hist_k, k])
    vals = np.vstack([hist_v, v])
    att = np.zeros(d)
    for h in range(h0, h0 + nh):
        kh = h // group
        assert kv0 <= kh < kv0 + nkv, "a query head of this rank uses another rank's KV head"
        s = keys[:, kh * hd:(kh + 1) * hd] @ q[h * hd:(h + 1) * hd] / np.sqrt(hd)
        p = np.exp(s - s.max())
        p /= p.sum()
        att[h * hd:(h + 1) * hd] = p @ vals[:, kh * hd:(kh + 1) * hd]
    cols = slice(h0 * hd, (h0 + nh) * hd)
    o = w["o"][:, cols] @ att[cols]
    g, u = w["g"][f0:f0 + nf] @ n, w["u"][f0:f0 + nf] @ n
    sw = g / (1 + np.exp(-g)) * u
    return o + w["dn"][:, f0:f0 + nf] @ sw


def _rank(rank, world, port, out):
    import torch
    import torch.distributed as dist
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    try:
        plan = tp_plan(CFG, world, rank)
        plans = [None] * world
        dist.all_gather_object(plans, plan)
        w, x, hk, hv = layer_weights()
        part = torch.from_numpy(layer_partial(w, x, hk, hv, *plan))
        dist.all_reduce(part)  # the per-layer exchange
        out.put((rank, plans, (x + part.numpy()).tolist()))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2])
def test_two_and_three_ranks_partition_and_sum(world):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = free_port()
    procs = [ctx.Process(target=_rank, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(60)
        assert p.exitcode == 0
    plans = res[0][1]
    H, KVH, ff = CFG["num_attention_heads"], CFG["num_key_value_heads"], CFG["intermediate_size"]
    for lo, cnt, total in ((0, 1, H), (2, 3, KVH), (4, 5, ff)):
        covered = sorted(i for p in plans for i in range(p[lo], p[lo] + p[cnt]))
        assert covered == list(range(total))
    w, x, hk, hv = layer_weights()
    whole = x + layer_partial(w, x, hk, hv, 0, H, 0, KVH, 0, ff)
    for _, _, y in res:
        assert np.max(np.abs(np.array(y) - whole)) <= 1e-12


def test_plan_rejects_uneven_splits():
    with pytest.raises(BackendError) as e:
        tp_plan(CFG, 4, 0)  # 4 does not divide 6 heads
    assert e.value.code == _lib.TCU_EINVAL
    with pytest.raises(BackendError):
        tp_plan(CFG, 2, 2)
