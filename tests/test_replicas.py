"""Multi-replica host logic on CPU: world-size-2 gloo ranks (127.0.0.1)
exchange only timing, and sequence shards cover every item once."""
import os
import socket

import pytest
import torch.distributed as dist
import torch.multiprocessing as mp

from tinyoai_b200 import replicas


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), WORLD_SIZE=str(world), RANK=str(rank),
                      LOCAL_RANK=str(rank))
    from datetime import timedelta
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
    try:
        ws, r, _ = replicas.world()
        # Rank r measured (r + 1) ms total and (10 - r) ms of decode.
        total, dec = replicas.max_over_ranks([r + 1.0, 10.0 - r])
        replicas.barrier()
        lo, hi = replicas.shard(64, ws, r)
        q.put((r, total, dec, lo, hi, replicas.aggregate_rate(768, ws, total / 1e3)))
    finally:
        dist.destroy_process_group()


def test_two_ranks_exchange_only_timing():
    world, port = 2, _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_rank, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(120)
        assert p.exitcode == 0
    got = sorted(q.get(timeout=10) for _ in range(world))
    for r, total, dec, lo, hi, rate in got:
        assert total == 2.0 and dec == 10.0  # the slowest rank's time, on every rank
        assert rate == pytest.approx(2 * 768 / 0.002)
    assert [(lo, hi) for _, _, _, lo, hi, _ in got] == [(0, 32), (32, 64)]


@pytest.mark.parametrize("n", [0, 1, 7, 64, 255])
@pytest.mark.parametrize("world", [1, 2, 3, 4, 8])
def test_shards_cover_items_once(n, world):
    spans = [replicas.shard(n, world, r) for r in range(world)]
    assert spans[0][0] == 0 and spans[-1][1] == n
    assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
    sizes = [hi - lo for lo, hi in spans]
    assert max(sizes) - min(sizes) <= 1


def test_single_process_is_identity():
    assert replicas.max_over_ranks([3.0, 4.0]) == [3.0, 4.0]
    with pytest.raises(ValueError):
        replicas.shard(4, 2, 2)
    with pytest.raises(ValueError):
        replicas.aggregate_rate(1, 1, 0.0)
