"""Device temperature / top-p sampler (tf_cuda_sample) against the reference's own
sample_logits (built from its sources) on real model logits, with the same std::mt19937
stream: the sampled ids must be identical."""
import os

import numpy as np
import pytest

import pyoracle as po
from tinferno_b200 import synth
from tinferno_b200.model import Model, Mt19937Uniform, RunConfig

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def logits_rows(model_cache):
    cfg = synth.mini(synth.CFG0, 2, 4096)
    m = Model(synth.model_path(cfg, model_cache), RunConfig(max_seq=64))
    return m, cfg


@pytest.mark.parametrize("temp,top_p,seed", [(0.8, 0.9, 42), (1.0, 1.0, 7), (0.3, 0.5, 123), (2.0, 0.95, 5)])
def test_sampler_matches_reference(temp, top_p, seed, logits_rows):
    if not po.ref_available():
        pytest.skip("reference build (oracle/_ref) not present")
    m, cfg = logits_rows
    m.reset()
    prompt = synth.prompt_tokens(cfg, 7, stream=900 + seed)
    lg = m.prefill(prompt)
    rng = Mt19937Uniform(seed)
    rows, got = [], []
    tok = int(np.argmax(lg))
    for step in range(24):
        rows.append(lg.copy())
        got.append(m.sample(temp, top_p, rng.next()))
        tok = got[-1]
        lg = m.decode(tok)
    L = np.ascontiguousarray(np.stack(rows), np.float32)
    want = np.zeros(len(rows), np.int32)
    po.ref_lib().ref_sample_logits_steps(po._fp(L), L.shape[1], L.shape[0], temp, top_p, seed,
                                         want.ctypes.data_as(po.i32p))
    assert got == want.tolist()


def test_greedy_sample_is_argmax(logits_rows):
    m, cfg = logits_rows
    m.reset()
    lg = m.prefill(synth.prompt_tokens(cfg, 5, stream=77))
    assert m.sample(0.0, 0.9, 0.5) == int(np.argmax(lg))
