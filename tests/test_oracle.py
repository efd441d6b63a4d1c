"""The oracle (oracle/tf_oracle.c) pinned to the reference engine and to the golden fixtures.

* op by op against the reference compiled from its own sources (oracle/_ref), bit for bit;
* the whole token loop against the reference on the reference's own CI model (tiny_ci.gguf,
  written by its test generator) and on seeded synthetic models;
* against the committed golden vectors (which the reference produced).
Tests that need oracle/_ref skip where it was not built (it needs the reference sources).
"""
import os

import numpy as np
import pytest

import pyoracle as po
from tinferno_b200 import gguf, quants, synth

from conftest import GOLDEN

needs_ref = pytest.mark.skipif(not po.ref_available(), reason="oracle/_ref not built (reference absent)")
fp = po._fp
TYPES = [gguf.GGML_F32, gguf.GGML_F16, gguf.GGML_Q4_0, gguf.GGML_Q4_1, gguf.GGML_Q8_0, gguf.GGML_Q6_K]


def _weights(rng, n, k, t):
    w = rng.standard_normal((n, k)).astype(np.float32) * np.float32(0.02)
    return np.ascontiguousarray(quants.quantize(w, t))


@needs_ref
@pytest.mark.parametrize("t", TYPES)
@pytest.mark.parametrize("shape", [(37, 256, 1), (64, 512, 3), (5, 2048, 2), (9, 768, 1)])
def test_matmul_and_dequant_bitexact(t, shape):
    n, k, m = shape
    if k % gguf.BLOCK[t][0]:
        pytest.skip("K not a multiple of the block")
    rng = np.random.default_rng(hash((t, shape)) & 0xFFFF)
    raw = _weights(rng, n, k, t)
    a = rng.standard_normal((m, k)).astype(np.float32)
    c_ref = np.zeros((m, n), np.float32)
    c_or = np.zeros((m, n), np.float32)
    assert po.ref_lib().ref_matmul(fp(c_ref), fp(a), t, raw.ctypes.data, n, k, m, 2, 1, 0) == 0
    po.oracle_lib().tfo_matmul(fp(c_or), fp(a), t, raw.ctypes.data, n, k, m, 2)
    assert np.array_equal(c_ref, c_or)
    for row in (0, n - 1):
        d1 = np.zeros(k, np.float32)
        d2 = np.zeros(k, np.float32)
        po.ref_lib().ref_dequant_row(fp(d1), t, raw.ctypes.data, k, row)
        po.oracle_lib().tfo_dequant_row(fp(d2), t, raw.ctypes.data, k, row)
        assert np.array_equal(d1, d2)
        # the numpy dequantiser used by the host tooling agrees too
        assert np.array_equal(quants.dequant(raw[row:row + 1], t, k)[0], d1)


@needs_ref
def test_elementwise_bitexact():
    R, O = po.ref_lib(), po.oracle_lib()
    rng = np.random.default_rng(7)
    for n in (1, 7, 896, 2048, 8192):
        x = rng.standard_normal(n).astype(np.float32) * 3
        w = rng.standard_normal(n).astype(np.float32)
        o1, o2 = np.zeros(n, np.float32), np.zeros(n, np.float32)
        R.ref_rmsnorm(fp(o1), fp(x), fp(w), n, 1e-5)
        O.tfo_rmsnorm(fp(o2), fp(x), fp(w), n, 1e-5)
        assert np.array_equal(o1, o2)
        g1, g2 = x.copy(), x.copy()
        R.ref_silu_mul(fp(g1), fp(w), n)
        O.tfo_silu_mul(fp(g2), fp(w), n)
        assert np.array_equal(g1, g2)
        s1, s2 = x.copy(), x.copy()
        R.ref_softmax(fp(s1), n)
        O.tfo_softmax(fp(s2), n)
        assert np.array_equal(s1, s2)
        assert R.ref_sample_greedy(fp(x), n) == O.tfo_sample_greedy(fp(x), n) == int(np.argmax(x))


@needs_ref
@pytest.mark.parametrize("hd", [8, 64, 128])
@pytest.mark.parametrize("llama3", [0, 1])
def test_rope_attention_bitexact(hd, llama3):
    R, O = po.ref_lib(), po.oracle_lib()
    rng = np.random.default_rng(hd + llama3)
    f1, f2 = np.zeros(hd // 2, np.float32), np.zeros(hd // 2, np.float32)
    R.ref_rope_freqs(fp(f1), hd, 500000.0, llama3, 32.0, 1.0, 4.0, 8192.0)
    O.tfo_rope_freqs(fp(f2), hd, 500000.0, llama3, 32.0, 1.0, 4.0, 8192.0)
    assert np.array_equal(f1, f2)
    q = rng.standard_normal((6, 4, hd)).astype(np.float32)
    q1, q2 = q.copy(), q.copy()
    R.ref_apply_rope_many(fp(q1), 6, 4, hd, 1234, fp(f1))
    O.tfo_rope(fp(q2), 6, 4, hd, 1234, fp(f1))
    assert np.array_equal(q1, q2)
    S, H, KV = 33, 8, 2
    q = rng.standard_normal((S, H, hd)).astype(np.float32)
    k = rng.standard_normal((S, KV, hd)).astype(np.float32)
    v = rng.standard_normal((S, KV, hd)).astype(np.float32)
    o1, o2 = np.zeros((S, H, hd), np.float32), np.zeros((S, H, hd), np.float32)
    R.ref_attn_prefill(fp(o1), fp(q), fp(k), fp(v), S, H, KV, hd)
    O.tfo_attn_prefill(fp(o2), fp(q), fp(k), fp(v), S, H, KV, hd)
    assert np.array_equal(o1, o2)
    qq = np.ascontiguousarray(q[-1])
    for head_major in (0, 1):
        a1, a2 = np.zeros((H, hd), np.float32), np.zeros((H, hd), np.float32)
        R.ref_attn_decode(fp(a1), fp(qq), fp(k), fp(v), S, H, KV, hd, head_major)
        O.tfo_attn_decode(fp(a2), fp(qq), fp(k), fp(v), S, H, KV, hd)
        assert np.array_equal(a1, a2)


def test_f16_conversions():
    O = po.oracle_lib()
    vals = np.array([0.0, -0.0, 1.5, 65504.0, 65520.0, 1e-8, 6.1e-5, 5.96e-8, 3.0e-8, -2.5, 1 / 3.0,
                     np.inf, -np.inf], np.float32)
    for v in vals:
        h = O.tfo_f32_to_f16(float(v))
        assert h == int(np.float32(v).astype(np.float16).view(np.uint16))
        assert O.tfo_f16_to_f32(h) == float(np.float16(v).astype(np.float32))
    for h in range(0, 0x10000, 7):
        if (h & 0x7C00) == 0x7C00 and (h & 0x3FF):
            continue  # NaN payloads
        assert O.tfo_f16_to_f32(h) == float(np.uint16(h).view(np.float16).astype(np.float32))
    if po.ref_available():
        R = po.ref_lib()
        for v in vals:
            assert R.ref_f32_to_f16(float(v)) == O.tfo_f32_to_f16(float(v))


@needs_ref
def test_quantisers_match_reference():
    R = po.ref_lib()
    rng = np.random.default_rng(3)
    x = (rng.standard_normal((4, 256)) * 0.02).astype(np.float32)
    x[0, :32] = 0.0  # an all-zero block
    for t, fn in ((gguf.GGML_Q8_0, R.ref_quant_q8_0_row), (gguf.GGML_Q4_0, R.ref_quant_q4_0_row)):
        ours = quants.quantize(x, t)
        theirs = np.zeros_like(ours)
        for r in range(4):
            fn(theirs[r].ctypes.data, fp(np.ascontiguousarray(x[r])), 256)
        assert np.array_equal(ours, theirs)


def test_new_quantisers_roundtrip():
    rng = np.random.default_rng(5)
    x = (rng.standard_normal((8, 512)) * 0.02).astype(np.float32)
    for t, tol in ((gguf.GGML_Q4_1, 0.2), (gguf.GGML_Q6_K, 0.05), (gguf.GGML_Q8_0, 0.01), (gguf.GGML_Q4_0, 0.2)):
        y = quants.dequant(quants.quantize(x, t), t, 512)
        rel = np.abs(y - x).max() / np.abs(x).max()
        assert rel < tol, (t, rel)


@needs_ref
def test_reference_ci_model_bitexact():
    """The reference's own correctness gate model and prompts: the oracle reproduces the
    reference's v2 logits bit for bit at every step."""
    path = os.path.join(GOLDEN, "tiny_ci.gguf")
    g = gguf.GGUFReader(path)
    gold = np.load(os.path.join(GOLDEN, "tiny_ci.npz"))
    for i, pr in enumerate(gold["prompts"][:6]):
        orc = po.OracleModel(g, 64, threads=1)
        ref = po.RefModel(path, 64, stage="v2")
        lo, lr = orc.prefill(pr), ref.prefill(pr)
        for s in range(8):
            assert np.array_equal(lo, lr)
            t = int(np.argmax(lo))
            assert t == gold["tokens_v2"][i][s]
            lo, lr = orc.decode(t), ref.decode(t)
        orc.close()
        ref.close()


def test_oracle_against_golden_ci():
    """No reference needed: the committed fixtures pin the oracle."""
    path = os.path.join(GOLDEN, "tiny_ci.gguf")
    g = gguf.GGUFReader(path)
    gold = np.load(os.path.join(GOLDEN, "tiny_ci.npz"))
    assert np.array_equal(gold["tokens_v0"], gold["tokens_v2"])  # the reference's own gate
    for i, pr in enumerate(gold["prompts"]):
        orc = po.OracleModel(g, 64, threads=1)
        ids, steps = po.greedy_stream(orc, pr, 8, keep_logits=True)
        assert ids == gold["tokens_v2"][i].tolist()
        assert np.array_equal(np.stack(steps), gold["logits_v2"][i])
        orc.close()


MINI = [synth.mini(synth.CFG0, 2, 4096), synth.mini(synth.CFG1, 2, 4096), synth.mini(synth.CFG2, 2, 4096),
        synth.mini(synth.CFG4, 2, 4096), synth.mini(synth.CFG0_LLAMA3, 2, 4096)]


@pytest.mark.parametrize("cfg", MINI, ids=lambda c: c.name)
def test_oracle_against_golden_synthetic(cfg, model_cache):
    gold = np.load(os.path.join(GOLDEN, cfg.name + ".npz"))
    path = synth.model_path(cfg, model_cache)
    assert synth.file_digest(path) == str(gold["sha256"]), "synthetic generator is not reproducing the fixture"
    g = gguf.GGUFReader(path)
    orc = po.OracleModel(g, cfg.max_seq)
    n = len(gold["tokens"])
    ids, steps = po.greedy_stream(orc, gold["prompt"], n, keep_logits=True)
    assert ids == gold["tokens"].tolist()
    for s, lg in enumerate(steps):
        assert np.array_equal(lg[gold["topi"][s]], gold["topv"][s])
        assert abs(np.sum(lg, dtype=np.float64) - gold["lsum"][s]) < 1e-9 * max(1.0, abs(gold["lsum"][s]))
    orc.close()


def test_llama3_rope_branch_matters(model_cache):
    """The llama3 fixture exercises the frequency-smoothing branch (src/attention.cpp:14-26):
    the same weights with standard RoPE give different logits on the same prompt."""
    l3, std = synth.mini(synth.CFG0_LLAMA3, 2, 4096), synth.mini(synth.CFG0, 2, 4096)
    prompt = np.load(os.path.join(GOLDEN, l3.name + ".npz"))["prompt"]
    outs = []
    for cfg in (l3, std):
        orc = po.OracleModel(gguf.GGUFReader(synth.model_path(cfg, model_cache)), cfg.max_seq)
        outs.append(orc.prefill(prompt))
        orc.close()
    assert np.abs(outs[0] - outs[1]).max() > 1e-4


def test_weight_bytes_of_the_configs():
    # GGUF::weight_bytes() (src/gguf.cpp:219-223, the sum of tensor bytes) of the four
    # benchmark configurations: the decode roofline's bytes per token.
    assert synth.weight_bytes(synth.CFG0) == 1_313_251_328
    assert synth.weight_bytes(synth.CFG1) == 525_120_000
    assert synth.weight_bytes(synth.CFG2) == 765_194_240
    assert synth.weight_bytes(synth.CFG4) == 1_640_622_080


@pytest.mark.slow
@pytest.mark.parametrize("key", ["cfg1", "cfg2"])
def test_oracle_against_golden_full_size(key, model_cache):
    """The oracle reproduces the reference build's full-size cfg1 (512 + 128 tokens) and cfg2
    (128 + 128, Q4_0 / Q6_K / Q4_1) streams bit for bit.  Opt-in (TFB200_FULL_GOLDEN=1): the
    GGUF files take minutes of host time to generate."""
    if os.environ.get("TFB200_FULL_GOLDEN") != "1":
        pytest.skip("full-size streams run with TFB200_FULL_GOLDEN=1")
    cfg = synth.CONFIGS[key]
    gold = np.load(os.path.join(GOLDEN, cfg.name + ".npz"))
    path = synth.model_path(cfg, model_cache)
    assert synth.file_digest(path) == str(gold["sha256"])
    orc = po.OracleModel(gguf.GGUFReader(path), cfg.max_seq, threads=os.cpu_count() or 1)
    ids, steps = po.greedy_stream(orc, gold["prompt"], len(gold["tokens"]), keep_logits=True)
    assert ids == gold["tokens"].tolist()
    for s, lg in enumerate(steps):
        assert np.array_equal(lg[gold["topi"][s]], gold["topv"][s])
    orc.close()


@needs_ref
@pytest.mark.parametrize("temp,top_p,seed", [(0.8, 0.9, 42), (1.0, 1.0, 7), (0.3, 0.5, 123), (2.0, 0.95, 5),
                                             (0.0, 0.9, 1)])
def test_sampler_restatement_matches_reference(temp, top_p, seed):
    """sample_logits (src/sampler.cpp:15-52): the oracle's restatement fed by the host's
    std::mt19937 + uniform_real_distribution<float> restatement (tinferno_b200.model.Mt19937Uniform,
    one draw per step as src/main.cpp:109-114) picks the ids the reference's own sampler picks
    with the same seed."""
    from tinferno_b200.model import Mt19937Uniform
    n, steps = 4096, 64
    rng = np.random.default_rng(seed)
    rows = np.ascontiguousarray((rng.standard_normal((steps, n)) * 2.5).astype(np.float32))
    want = np.zeros(steps, np.int32)
    po.ref_lib().ref_sample_logits_steps(fp(rows), n, steps, temp, top_p, seed, want.ctypes.data_as(po.i32p))
    draws = Mt19937Uniform(seed)
    O = po.oracle_lib()
    got = [int(O.tfo_sample_logits(fp(rows[i].copy()), n, temp, top_p, draws.next() if temp > 0 else 0.0))
           for i in range(steps)]
    assert got == want.tolist()
