"""The multi-rank host logic on CPU: two gloo ranks share a batch.

Each rank predicts its contiguous shard of the rows (with the CPU oracle
standing in for the GPU predict) and montlok.distributed gathers the shards;
the result must equal a single-process prediction bit for bit, and the
timing reduction must return the slowest rank's value on every rank.
"""

from __future__ import annotations

import os
import socket

import numpy as np
import pytest

from forests import edge_inputs, random_model, same_bits
from montlok.distributed import shard


def free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def rank_main(rank: int, world: int, port: int, model: bytes, x: np.ndarray, result) -> None:
    import torch.distributed as dist

    from montlok.distributed import max_over_ranks, predict_sharded
    from oracle import Oracle

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        o = Oracle(model)
        got = predict_sharded(o.predict, x)
        slowest = max_over_ranks([1.5 + rank, -rank])
        result[rank] = (got, slowest)
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("rows", [0, 1, 7, 1001])
def test_sharded_predict_on_two_gloo_ranks(rows):
    torch = pytest.importorskip("torch")
    mp = torch.multiprocessing.get_context("spawn")
    rng = np.random.default_rng(rows)
    model = random_model(rng, features=6, trees=90, outputs=3, link="softmax")
    x = edge_inputs(rng, rows, 6)
    with mp.Manager() as manager:
        result = manager.dict()
        port = free_port()
        procs = [mp.Process(target=rank_main, args=(r, 2, port, model, x, result)) for r in range(2)]
        for p in procs:
            p.start()
        for p in procs:
            p.join(120)
            assert p.exitcode == 0
        from oracle import Oracle

        want = Oracle(model).predict(x)
        for r in range(2):
            got, slowest = result[r]
            assert same_bits(got.reshape(want.shape), want)
            assert slowest == [2.5, 0.0]


def test_shards_cover_the_batch_in_order():
    for batch in (0, 1, 5, 8, 1000, 1001):
        for world in (1, 2, 3, 8):
            spans = [shard(batch, r, world) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == batch
            for (lo0, hi0), (lo1, hi1) in zip(spans, spans[1:]):
                assert hi0 == lo1 and lo0 <= hi0
    with pytest.raises(ValueError):
        shard(10, 2, 2)
