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


# ---- vocab-split lm_head: the key and its max reduction ------------------------------------------
# Restatement of the device key (common.cuh argmax_key): the logit's order bits above the
# complement of the vocabulary index; NaN never wins except at index 0.  The engine's shards
# order-flip it to int64 (key ^ 2^63) for a signed max all-reduce.

def greedy_key(v: np.ndarray, idx: np.ndarray) -> np.ndarray:
    b = v.astype(np.float32).view(np.uint32).astype(np.uint64)
    ordv = np.where(b & 0x80000000, (~b) & 0xFFFFFFFF, b | 0x80000000)
    ordv = np.where(np.isnan(v), np.where(idx == 0, 0xFFFFFFFF, 0), ordv).astype(np.uint64)
    return (ordv << np.uint64(32)) | (np.uint64(0xFFFFFFFF) - idx.astype(np.uint64))


def shard_key(logits: np.ndarray, rank: int, world: int) -> int:
    r0, r1 = shard.vocab_shard_rows(len(logits), rank, world)
    f = int(greedy_key(logits[r0:r1], np.arange(r0, r1)).max()) ^ (1 << 63)  # order-flipped
    return f - (1 << 64) if f >= (1 << 63) else f  # as a signed int64


def key_index(flipped: int) -> int:
    key = (flipped % (1 << 64)) ^ (1 << 63)
    return 0xFFFFFFFF - (key & 0xFFFFFFFF)


def _cases():
    rng = np.random.default_rng(5)
    out = [rng.standard_normal(1000).astype(np.float32) for _ in range(3)]
    t = rng.standard_normal(1000).astype(np.float32)
    t[[3, 700, 999]] = 9.0  # equal maxima in different shards: the first index wins
    out.append(t)
    t = -np.abs(rng.standard_normal(1000)).astype(np.float32)  # all negative
    out.append(t)
    t = rng.standard_normal(1000).astype(np.float32)
    t[[10, 500]] = np.nan  # NaN away from index 0 never wins
    out.append(t)
    t = rng.standard_normal(1000).astype(np.float32)
    t[0] = np.nan  # NaN at index 0: the reference returns 0
    out.append(t)
    return out


def test_vocab_rows_cover_once():
    for v in (1000, 128256, 151936):
        for w in (1, 2, 3, 8):
            rs = [shard.vocab_shard_rows(v, r, w) for r in range(w)]
            assert rs[0][0] == 0 and rs[-1][1] == v and all(a[1] == b[0] for a, b in zip(rs, rs[1:]))


def test_split_key_reduction_is_sample_greedy():
    """max over the shards' flipped keys names sample_greedy's id (the oracle's restatement of
    src/sampler.cpp:8-13) for every split."""
    import pyoracle as po
    for lg in _cases():
        want = int(po.oracle_lib().tfo_sample_greedy(po._fp(np.ascontiguousarray(lg)), len(lg)))
        for w in (1, 2, 3, 8):
            red = max(shard_key(lg, r, w) for r in range(w))
            assert key_index(red) == want, (w, want)


def _key_worker(rank, world, port, cases, q):
    import torch
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    got = []
    for lg in cases:
        t = torch.tensor([shard_key(lg, rank, world)], dtype=torch.int64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        got.append(key_index(int(t.item())))
    if rank == 0:
        q.put(got)
    dist.barrier()
    dist.destroy_process_group()


def test_gloo_two_ranks_split_key_all_reduce():
    """The reduction the vocab-split lm_head runs across GPUs (one int64 max all-reduce per step),
    here over two gloo ranks: every rank ends with the whole vocabulary's first-index argmax."""
    import torch.multiprocessing as mp
    import pyoracle as po
    cases = _cases()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_key_worker, args=(r, 2, port, cases, q)) for r in range(2)]
    for p in procs:
        p.start()
    got = q.get(timeout=120)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    want = [int(po.oracle_lib().tfo_sample_greedy(po._fp(np.ascontiguousarray(lg)), len(lg))) for lg in cases]
    assert got == want
