"""Sequence sharding for batched decode across GPUs (one process per GPU).

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
