"""Host logic of the multi-GPU batched decode (sequence sharding), on CPU: the shard ranges,
a sharded run against an unsharded one with a deterministic stand-in for the engine, and the
id gather across two gloo ranks."""
import os
import socket

import numpy as np
import pytest

from tinferno_b200 import shard


def test_shard_ranges_cover_once():
    for n in (1, 7, 256, 257):
        for w in (1, 2, 3, 8):
            rs = [shard.shard_range(n, r, w) for r in range(w)]
            assert rs[0][0] == 0 and rs[-1][1] == n
            assert all(a[1] == b[0] for a, b in zip(rs, rs[1:]))
            sizes = [b - a for a, b in rs]
            assert max(sizes) - min(sizes) <= 1
    with pytest.raises(ValueError):
        shard.shard_range(4, 2, 2)


class FakeEngine:
    """Stands in for Model: the next id of a slot is a hash of its history, so results depend
    on every token the slot has seen (as the real model's do)."""

    def __init__(self, vocab=97):
        self.v = vocab
        self.hist = {}

    def _next(self, slot):
        h = 0
        for t in self.hist[slot]:
            h = (h * 31 + int(t) + 7) % 1000003
        return h % self.v

    def prefill_batch(self, slots, prompts):
        out = []
        for s, p in zip(slots, prompts):
            self.hist[s] = list(p)
            out.append(self._next(s))
        return np.array(out, np.int32)

    def decode_batch(self, slots, toks):
        out = []
        for s, t in zip(slots, toks):
            self.hist[s].append(t)
            out.append(self._next(s))
        return np.array(out, np.int32)


def test_sharded_run_equals_unsharded():
    rng = np.random.default_rng(0)
    prompts = rng.integers(0, 97, size=(10, 6)).astype(np.int32)
    whole = shard.run_batched_greedy(FakeEngine(), prompts, 5)
    for w in (2, 3):
        parts = []
        for r in range(w):
            a, b = shard.shard_range(len(prompts), r, w)
            parts.append(shard.run_batched_greedy(FakeEngine(), prompts[a:b], 5))
        np.testing.assert_array_equal(np.concatenate(parts), whole)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, prompts, q):
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    a, b = shard.shard_range(len(prompts), rank, world)
    local = shard.run_batched_greedy(FakeEngine(), prompts[a:b], 4)
    ids = shard.gather_ids(local, dist)
    if rank == 0:
        q.put(ids)
    dist.barrier()
    dist.destroy_process_group()


def test_gloo_two_ranks_gather():
    import torch.multiprocessing as mp
    rng = np.random.default_rng(1)
    prompts = rng.integers(0, 97, size=(9, 5)).astype(np.int32)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, prompts, q)) for r in range(2)]
    for p in procs:
        p.start()
    ids = q.get(timeout=120)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    np.testing.assert_array_equal(ids, shard.run_batched_greedy(FakeEngine(), prompts, 4))
