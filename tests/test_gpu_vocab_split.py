"""Vocab-split lm_head (batch-1 latency across GPUs) on one GPU: W engine handles on the same
device each compute the logits of V/W vocabulary rows and leave their greedy key; the keys are
max-reduced on the host (what the NCCL all-reduce does across GPUs) and written back; each
handle then continues from the reduced key on the device.  The ids must equal the full
vocabulary's greedy stream, including the first-index tie rule at shard boundaries."""
import numpy as np
import pytest

from tinferno_b200 import shard, synth
from tinferno_b200.model import Model, RunConfig

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


@pytest.mark.parametrize("world", [2, 3])
@pytest.mark.parametrize("cfg", [synth.mini(synth.CFG0, 2, 4096), synth.mini(synth.CFG1, 2, 4096)],
                         ids=lambda c: c.name)
def test_vocab_split_matches_full_vocabulary(cfg, world, model_cache):
    path = synth.model_path(cfg, model_cache)
    prompt = synth.prompt_tokens(cfg, 7, stream=61)
    n = 12
    full = Model(path, RunConfig(max_seq=64))
    first = int(np.argmax(full.prefill(prompt)))
    want = full.generate_greedy(first, n)
    full.close()
    parts = [Model(path, RunConfig(max_seq=64)) for _ in range(world)]
    for r, m in enumerate(parts):
        m.set_vocab_shard(r, world)
        assert int(np.argmax(m.prefill(prompt))) == first  # prefill computes the whole vocabulary
    keys = [shard.key_tensor(m) for m in parts]
    for i in range(n):
        for m in parts:
            m.decode_shard(first if i == 0 else -1)
        torch.cuda.synchronize()
        red = max(int(k.item()) for k in keys)  # the max all-reduce, on the host
        for k in keys:
            k.fill_(red)
        torch.cuda.synchronize()
    for m in parts:
        m.shard_token()
        assert [first] + m.history(n - 1) == want
        assert m.n_pos() == len(prompt) + n
        m.close()
