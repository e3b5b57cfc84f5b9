"""Row sharding over ranks (no GPU): shard geometry, generator skip-ahead, and a world-size-2
gloo run whose gathered tokens equal the unsharded decode."""
import os
import socket

import numpy as np
import pytest
import torch.distributed as dist
import torch.multiprocessing as mp

from basalt_b200.sharding import advance, scramble, shard_rng_state, shard_rows
from oracle import oracle as orc


def test_shards_cover_rows_contiguously():
    for total in (0, 1, 7, 256, 8192, 1001):
        for world in (1, 2, 3, 4, 8):
            spans = [shard_rows(total, world, r) for r in range(world)]
            assert sum(c for _, c in spans) == total
            nxt = 0
            for first, count in spans:
                assert first == nxt
                nxt = first + count
            counts = [c for _, c in spans]
            assert max(counts) - min(counts) <= 1
    with pytest.raises(ValueError):
        shard_rows(10, 2, 2)


@pytest.mark.parametrize("steps", [0, 1, 2, 3, 17, 100, 1 << 10, 123457])
def test_skip_ahead_equals_stepping(steps):
    start = scramble(9)
    assert advance(start, steps) == orc.lcg_advance(start, steps)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


CONTEXTS = [[0, 0, 0], [1, 2, 3], [4, 4, 4], [2, 2, 1], [3, 0, 1], [1, 1, 0], [4, 2, 0]]
STEPS, SEED, TEMPERATURE, TOPK = 9, 5, 2.0, 4


def _rank(rank, world, port, queue):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    first, count = shard_rows(len(CONTEXTS), world, rank)
    engine = orc.OracleEngine(orc.FAMILY_LAST_TOKEN, 5, 3)
    engine.rng_state = shard_rng_state(SEED, STEPS, first)
    sampled = [engine.sample(CONTEXTS[first + i], STEPS, TEMPERATURE, TOPK).tolist()
               for i in range(count)]
    greedy = engine.generate_batch(CONTEXTS[first:first + count], STEPS).tolist() if count else []
    gathered = [None] * world
    dist.all_gather_object(gathered, (first, sampled, greedy))
    if rank == 0:
        queue.put(gathered)
    dist.barrier()
    dist.destroy_process_group()


def test_sharded_decode_over_gloo_equals_the_unsharded_run():
    world = 2
    ctx = mp.get_context("spawn")
    queue = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank, args=(r, world, port, queue)) for r in range(world)]
    for p in procs:
        p.start()
    gathered = queue.get(timeout=120)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    gathered.sort()
    sampled = [row for _, s, _ in gathered for row in s]
    greedy = [row for _, _, g in gathered for row in g]
    reference = orc.OracleEngine(orc.FAMILY_LAST_TOKEN, 5, 3)
    reference.seed(SEED)
    want = [reference.sample(c, STEPS, TEMPERATURE, TOPK).tolist() for c in CONTEXTS]
    assert sampled == want
    np.testing.assert_array_equal(np.array(greedy),
                                  reference.generate_batch(CONTEXTS, STEPS))
