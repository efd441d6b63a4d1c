"""Sequence sharding for batched decode across GPUs (one process per GPU), and the
vocab-split lm_head for batch-1 latency.

The batched workload (BASELINE cfg4: independent sequences, each a prompt then greedy decode)
partitions by sequence: rank r of W owns a contiguous range of sequences, holds a full copy
of the weights, and decodes its sequences as one batch.  There is no collective on the data
path; the host gathers the generated ids at the end (`gather_ids`).  The reference decodes
one sequence per Model (src/main.cpp:106-122); each shard here runs that loop for many
sequences at once through Model.prefill_batch / Model.decode_batch.
"""
from __future__ import annotations

from typing import List, Sequence, Tuple

import numpy as np


def shard_range(n_items: int, rank: int, world: int) -> Tuple[int, int]:
    """Contiguous [start, end) share of n_items for `rank` of `world` (sizes differ by <= 1)."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError("bad rank/world")
    base, extra = divmod(n_items, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


def run_batched_greedy(model, prompts: np.ndarray, steps: int, slots: Sequence[int] = None) -> np.ndarray:
    """Prefill `prompts` ([S][n] token ids) into slots 0..S-1 (or `slots`) and decode `steps`
    greedy tokens for all of them; returns ids [S][steps + 1] (the first id comes from the
    prompt, as in the CLI loop)."""
    prompts = np.asarray(prompts, np.int32)
    S = prompts.shape[0]
    slots = list(range(S)) if slots is None else list(slots)
    out = np.zeros((S, steps + 1), np.int32)
    tok = np.asarray(model.prefill_batch(slots, prompts), np.int32)
    out[:, 0] = tok
    for s in range(steps):
        tok = np.asarray(model.decode_batch(slots, tok.tolist()), np.int32)
        out[:, s + 1] = tok
    return out


def gather_ids(local: np.ndarray, dist=None) -> np.ndarray:
    """Concatenate every rank's [S_r][T] ids in rank order (the host-side gather)."""
    if dist is None or not dist.is_initialized() or dist.get_world_size() == 1:
        return np.asarray(local)
    parts: List = [None] * dist.get_world_size()
    dist.all_gather_object(parts, np.asarray(local))
    return np.concatenate(parts, axis=0)


# ---- vocab-split lm_head (batch 1) ------------------------------------------------------------
# Every GPU runs the same sequence with all layers replicated, but computes the lm_head only for
# its share of the vocabulary rows [V*r/W, V*(r+1)/W).  Its greedy key - the logit's order bits
# above the complement of the vocabulary index, so that a larger key is a larger logit and, on
# equal logits, a smaller index (sample_greedy's first-index rule, src/sampler.cpp:8-13) - is
# order-flipped to a signed int64 and reduced with one max all-reduce (NCCL over NVLink); the
# reduced key names the whole vocabulary's argmax on every GPU.

def vocab_shard_rows(n_vocab: int, rank: int, world: int) -> Tuple[int, int]:
    """Rows [start, end) of the output matrix that `rank` of `world` computes (the engine's own
    split, tf_cuda_set_vocab_shard)."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError("bad rank/world")
    return n_vocab * rank // world, n_vocab * (rank + 1) // world


def split_greedy(model, first_token: int, n: int, reduce_key, seq: int = 0) -> List[int]:
    """n greedy ids starting from first_token with the vocab-split lm_head: each step runs
    asynchronously on the model's stream, then reduce_key() max-reduces the key at
    model.shard_key_ptr across the GPUs (on the same stream); the next step reads the reduced
    key on the device.  Like generate_greedy (without its EOS rule): n decode steps, returning
    [first_token, t_1, ..., t_{n-1}], with one host synchronisation at the end."""
    if n <= 0:
        return []
    for i in range(n):
        model.decode_shard(first_token if i == 0 else -1, seq=seq)
        reduce_key()
    model.shard_token(seq=seq)  # applies the last reduced key (its history entry) and synchronises
    return [int(first_token)] + [int(t) for t in model.history(n - 1)]


class _DeviceInt64:
    """__cuda_array_interface__ view of one int64 the engine owns (the shard key), so that torch
    (and its NCCL process group) can reduce it in place."""

    def __init__(self, ptr: int):
        self.__cuda_array_interface__ = {"shape": (1,), "typestr": "<i8", "data": (int(ptr), False),
                                         "version": 3, "strides": None}


def key_tensor(model):
    """torch view (no copy) of the model's shard key."""
    import torch
    return torch.as_tensor(_DeviceInt64(model.shard_key_ptr), device="cuda")


def nccl_key_reducer(model, dist):
    """reduce_key for split_greedy: one int64 max all-reduce of the key on the model's stream
    (torch.distributed with the NCCL backend, one process per GPU)."""
    import torch
    key = key_tensor(model)
    stream = torch.cuda.ExternalStream(model.stream)

    def reduce_key():
        with torch.cuda.stream(stream):
            dist.all_reduce(key, op=dist.ReduceOp.MAX)
    return reduce_key
