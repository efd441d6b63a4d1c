"""Batched decode at M >= 16 rows (the tensor-core GEMM path: f16-split Q8_0 GEMM, split
flash-decode attention over the rows' slots) against the batch-1 path and the oracle."""
import numpy as np
import pytest

import pyoracle as po
from tinferno_b200 import gguf, synth
from tinferno_b200.model import Model, RunConfig

pytestmark = pytest.mark.gpu

CFGS = [synth.mini(synth.CFG0, 2, 4096), synth.mini(synth.CFG1, 2, 4096), synth.mini(synth.CFG4, 2, 4096)]
LOGIT_TOL = 2e-3  # observed ~1e-5: the split keeps 22 significant bits of weights and activations


@pytest.fixture(scope="module")
def paths(model_cache):
    return {c.name: synth.model_path(c, model_cache) for c in CFGS}


@pytest.mark.parametrize("cfg", CFGS, ids=lambda c: c.name)
def test_batched_gemm_matches_single_rows(cfg, paths):
    B, steps = 20, 4
    path = paths[cfg.name]
    prompts = [synth.prompt_tokens(cfg, 3 + (b % 7), stream=100 + b) for b in range(B)]
    # batch-1 reference streams (GEMV path)
    solo = Model(path, RunConfig(max_seq=64))
    want_ids, want_lg = [], []
    for p in prompts:
        solo.reset()
        lg = solo.prefill(p)
        ids, lgs = [int(np.argmax(lg))], []
        for _ in range(steps):
            lgs.append(solo.decode(ids[-1]).copy())
            ids.append(int(np.argmax(lgs[-1])))
        want_ids.append(ids)
        want_lg.append(lgs)
    solo.close()
    m = Model(path, RunConfig(max_seq=64, max_batch=B + 4))
    toks = []
    for b, p in enumerate(prompts):
        toks.append(int(np.argmax(m.prefill(p, seq=b + 2))))  # slots 2..B+1
    assert toks == [w[0] for w in want_ids]
    seqs = [b + 2 for b in range(B)]
    err = 0.0
    for s in range(steps):
        am, lg = m.decode_batch(seqs, toks, want_logits=True)
        for b in range(B):
            err = max(err, float(np.abs(lg[b] - want_lg[b][s]).max()))
        toks = am.tolist()
        assert toks == [w[s + 1] for w in want_ids]
    assert err < LOGIT_TOL, err
    print(f"{cfg.name}: batched GEMM vs batch-1 max |logit diff| {err:.2e}")
    for b in range(B):
        assert m.n_pos(seq=b + 2) == len(prompts[b]) + steps
    m.close()


def test_batched_gemm_against_oracle(paths):
    cfg = CFGS[0]
    path = paths[cfg.name]
    B = 16
    prompts = [synth.prompt_tokens(cfg, 5, stream=300 + b) for b in range(B)]
    m = Model(path, RunConfig(max_seq=32, max_batch=B))
    first = [int(np.argmax(m.prefill(p, seq=b))) for b, p in enumerate(prompts)]
    am, lg = m.decode_batch(list(range(B)), first, want_logits=True)
    orc = po.OracleModel(gguf.GGUFReader(path), 32)
    for b in (0, 7, 15):
        orc.reset()
        orc.prefill(prompts[b])
        want = orc.decode(first[b])
        assert np.abs(lg[b] - want).max() < LOGIT_TOL
        assert int(am[b]) == int(np.argmax(want))
    m.close()
