"""Model-level parity of the CUDA engine (through the C-ABI, host mirror tinferno_b200.Model)
against the reference's golden streams and the oracle: greedy token streams must match
exactly; logits must agree within 1e-2 max-abs (observed
differences are ~1e-5)."""
import os

import numpy as np
import pytest

import pyoracle as po
from tinferno_b200 import gguf, native, synth
from tinferno_b200.model import Model, RunConfig

from conftest import GOLDEN

pytestmark = pytest.mark.gpu
LOGIT_TOL = 1e-2

MINI = [synth.mini(synth.CFG0, 2, 4096), synth.mini(synth.CFG1, 2, 4096), synth.mini(synth.CFG2, 2, 4096),
        synth.mini(synth.CFG4, 2, 4096), synth.mini(synth.CFG0_LLAMA3, 2, 4096)]


def greedy(model, prompt, n, seq=0):
    logits = model.prefill(prompt, seq=seq)
    ids, steps = [], []
    for _ in range(n):
        steps.append(logits.copy())
        t = int(po.oracle_lib().tfo_sample_greedy(po._fp(logits), len(logits)))
        ids.append(t)
        logits = model.decode(t, seq=seq)
    return ids, steps


def test_reference_ci_model():
    """The reference's own correctness gate: its CI model, its 20 prompts, 8 greedy tokens."""
    path = os.path.join(GOLDEN, "tiny_ci.gguf")
    gold = np.load(os.path.join(GOLDEN, "tiny_ci.npz"))
    m = Model(path, RunConfig(max_seq=64))
    for i, pr in enumerate(gold["prompts"]):
        m.reset()
        ids, steps = greedy(m, pr, 8)
        assert ids == gold["tokens_v0"][i].tolist()
        err = np.abs(np.stack(steps) - gold["logits_v2"][i]).max()
        assert err < 1e-4, err
    m.close()


@pytest.fixture(scope="module")
def mini_models(model_cache):
    return {cfg.name: synth.model_path(cfg, model_cache) for cfg in MINI}


@pytest.mark.parametrize("cfg", MINI, ids=lambda c: c.name)
def test_mini_stream_matches_reference(cfg, mini_models):
    gold = np.load(os.path.join(GOLDEN, cfg.name + ".npz"))
    path = mini_models[cfg.name]
    assert synth.file_digest(path) == str(gold["sha256"])
    m = Model(path, RunConfig(max_seq=cfg.max_seq))
    ids, steps = greedy(m, gold["prompt"], len(gold["tokens"]))
    assert ids == gold["tokens"].tolist()
    for s, lg in enumerate(steps):
        assert np.abs(lg[gold["topi"][s]] - gold["topv"][s]).max() < LOGIT_TOL
    # full logits against the oracle at every step
    orc = po.OracleModel(gguf.GGUFReader(path), cfg.max_seq)
    o_ids, o_steps = po.greedy_stream(orc, gold["prompt"], len(gold["tokens"]), keep_logits=True)
    assert o_ids == ids
    err = max(np.abs(a - b).max() for a, b in zip(steps, o_steps))
    assert err < LOGIT_TOL, err
    print(f"{cfg.name}: max |logit diff| vs oracle {err:.2e}")
    m.close()


@pytest.mark.parametrize("ci,n_prompt,n_decode", [(0, 270, 24), (0, 1016, 16), (1, 500, 16), (0, 1500, 8)])
def test_long_context_crosses_fused_attention_limit(ci, n_prompt, n_decode, mini_models):
    """Batch-1 decode across the fused attention's hand-overs: one CTA per query head up to
    two tiles (~280 positions for cfg0, ~120 for cfg1), then position splits inside the QKV
    kernel (cfg0 across 1024, cfg1 at 500-516: five splits of 14 heads), then the separate
    split flash-decode kernel (cfg0 at 1500: more splits than half the GEMV slots hold):
    token-exact and logits within 1e-2 of the oracle after a chunked tensor-core prefill."""
    cfg = MINI[ci]
    path = mini_models[cfg.name]
    prompt = synth.prompt_tokens(cfg, n_prompt, stream=4242)
    m = Model(path, RunConfig(max_seq=2048))
    ids, steps = greedy(m, prompt, n_decode)
    assert m.n_pos() == n_prompt + n_decode
    orc = po.OracleModel(gguf.GGUFReader(path), 2048)
    o_ids, o_steps = po.greedy_stream(orc, prompt, n_decode, keep_logits=True)
    assert o_ids == ids
    err = max(np.abs(a - b).max() for a, b in zip(steps, o_steps))
    assert err < LOGIT_TOL, err
    print(f"positions {n_prompt}..{n_prompt + n_decode - 1} token-exact, max |logit diff| {err:.2e}")
    m.close()
    orc.close()


# the persistent kernel takes models whose matrices are all Q8_0 with rows of 64-element
# units that fit its lanes (cfg0, cfg1, llama3 RoPE); cfg2's Q4_0 / Q6_K / Q4_1 matrices and
# cfg4's K = 8960 down rows stay on the per-kernel path
PERSISTENT = [MINI[0], MINI[1], MINI[4]]


def test_persistent_mode_rejects_other_models(mini_models):
    for cfg in (MINI[2], MINI[3]):
        with pytest.raises(native.TFError, match="persistent decode kernel does not take"):
            Model(mini_models[cfg.name], RunConfig(max_seq=cfg.max_seq, decode_mode=native.TF_DECODE_PERSISTENT))


@pytest.mark.parametrize("cfg", PERSISTENT, ids=lambda c: c.name)
def test_persistent_mode_matches_reference(cfg, mini_models):
    """The one-launch-per-call persistent kernel: same golden stream, logits within
    tolerance of the per-kernel path, and its fused prefill + greedy generation."""
    gold = np.load(os.path.join(GOLDEN, cfg.name + ".npz"))
    path = mini_models[cfg.name]
    m = Model(path, RunConfig(max_seq=cfg.max_seq, decode_mode=native.TF_DECODE_PERSISTENT))
    k = Model(path, RunConfig(max_seq=cfg.max_seq))
    ids, steps = greedy(m, gold["prompt"], len(gold["tokens"]))
    assert ids == gold["tokens"].tolist()
    k_ids, k_steps = greedy(k, gold["prompt"], len(gold["tokens"]))
    assert k_ids == ids
    for a, b in zip(steps, k_steps):
        np.testing.assert_allclose(a, b, rtol=0, atol=1e-4)
    m.reset()
    lg = m.prefill(gold["prompt"])
    assert m.generate_greedy(int(np.argmax(lg)), len(ids)) == ids
    m.close()
    k.close()


def test_q4_integer_path_on_every_matrix(mini_models, tmp_path):
    """cfg2 with no size threshold for the Q4_0 exact-integer GEMV (TFB200_Q4_INT_MIN_MB=0, read
    once per process, so in a child process): the 2-4 MB QKV and wo matrices take the integer
    path that only 32 MB matrices take by default (gate/up pairs and the K = 8192 down rows
    exceed its 32 units per warp and stay on the fp32 path); the golden stream stays
    token-exact and the logits within 1e-2 of the oracle."""
    import subprocess
    import sys
    cfg = MINI[2]
    path = mini_models[cfg.name]
    gold = os.path.join(GOLDEN, cfg.name + ".npz")
    out = tmp_path / "q4int.npz"
    code = (
        "import numpy as np\n"
        "from tinferno_b200.model import Model, RunConfig\n"
        f"g = np.load({gold!r})\n"
        f"m = Model({path!r}, RunConfig(max_seq={cfg.max_seq}))\n"
        "lg = m.prefill(g['prompt']); ids, steps = [], []\n"
        "for _ in range(len(g['tokens'])):\n"
        "    steps.append(lg.copy()); ids.append(int(np.argmax(lg))); lg = m.decode(ids[-1])\n"
        f"np.savez({str(out)!r}, ids=np.array(ids), steps=np.stack(steps))\n"
    )
    env = dict(os.environ, TFB200_Q4_INT_MIN_MB="0")
    env["PYTHONPATH"] = os.pathsep.join(sys.path)
    r = subprocess.run([sys.executable, "-c", code], env=env, capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr[-2000:]
    got = np.load(out)
    g = np.load(gold)
    assert got["ids"].tolist() == g["tokens"].tolist()
    orc = po.OracleModel(gguf.GGUFReader(path), cfg.max_seq)
    o_ids, o_steps = po.greedy_stream(orc, g["prompt"], len(g["tokens"]), keep_logits=True)
    assert o_ids == got["ids"].tolist()
    err = max(np.abs(a - b).max() for a, b in zip(got["steps"], o_steps))
    assert err < LOGIT_TOL, err
    orc.close()


def test_graph_and_eager_identical(mini_models):
    cfg = MINI[0]
    path = mini_models[cfg.name]
    prompt = synth.prompt_tokens(cfg, 9)
    a = Model(path, RunConfig(max_seq=128, use_graph=True))
    b = Model(path, RunConfig(max_seq=128, use_graph=False))
    ia, sa = greedy(a, prompt, 6)
    ib, sb = greedy(b, prompt, 6)
    assert ia == ib
    for x, y in zip(sa, sb):
        assert np.array_equal(x, y)  # the kernels are deterministic
    a.close()
    b.close()


def test_generate_greedy_matches_decode_loop(mini_models):
    cfg = MINI[1]
    path = mini_models[cfg.name]
    m = Model(path, RunConfig(max_seq=256))
    prompt = synth.prompt_tokens(cfg, 10)
    ids, _ = greedy(m, prompt, 20)
    m.reset()
    lg = m.prefill(prompt)
    first = int(np.argmax(lg))
    got = m.generate_greedy(first, 20)
    assert got == ids
    assert m.n_pos() == 10 + 20
    # EOS rule of the CLI loop (src/main.cpp:116): stop before an eos id at i > 0
    eos = ids[5]
    m.reset()
    m.prefill(prompt)
    cut = m.generate_greedy(first, 20, eos=eos)
    j = next(i for i in range(1, 20) if ids[i] == eos)
    assert cut == ids[:j]
    assert m.n_pos() == 10 + j
    # decoding continues from the truncated position exactly like the reference
    nxt = m.decode(eos)
    ref_m = Model(path, RunConfig(max_seq=256))
    ref_m.prefill(prompt)
    for t in ids[:j]:
        ref_m.decode(t)
    np.testing.assert_array_equal(nxt, ref_m.decode(eos))
    m.close()
    ref_m.close()


def test_slots_and_batch(mini_models):
    cfg = MINI[0]
    path = mini_models[cfg.name]
    m = Model(path, RunConfig(max_seq=128, max_batch=4))
    p0, p1, p2 = (synth.prompt_tokens(cfg, n, stream=s) for n, s in ((7, 1), (11, 2), (5, 3)))
    solo = []
    for p in (p0, p1, p2):
        s = Model(path, RunConfig(max_seq=128))
        solo.append(greedy(s, p, 5))
        s.close()
    # interleaved single-slot decoding
    lg = [m.prefill(p, seq=i) for i, p in enumerate((p0, p1, p2))]
    toks = [int(np.argmax(x)) for x in lg]
    for i in range(3):
        assert toks[i] == solo[i][0][0]
    # batched steps over the three slots
    got = [[t] for t in toks]
    for step in range(4):
        am, logits = m.decode_batch([0, 1, 2], toks, want_logits=True)
        for i in range(3):
            # the batched kernels sum in another order than the persistent batch-1 kernel
            np.testing.assert_allclose(logits[i], solo[i][1][step + 1], rtol=0, atol=1e-4)
        toks = am.tolist()
        for i in range(3):
            got[i].append(toks[i])
    for i in range(3):
        assert got[i] == solo[i][0]
    m.close()


def test_prefill_after_decode_sees_its_chunk_only(mini_models):
    """Model::prefill at n_pos > 0 attends within the new chunk only (attn_prefill over fresh
    k/v, src/attention.cpp:82-111) while its KV lands after the old positions."""
    cfg = MINI[2]
    path = mini_models[cfg.name]
    a, b = synth.prompt_tokens(cfg, 6, stream=4), synth.prompt_tokens(cfg, 5, stream=5)
    m = Model(path, RunConfig(max_seq=64))
    orc = po.OracleModel(gguf.GGUFReader(path), 64)
    m.prefill(a)
    orc.prefill(a)
    t = 17
    m.decode(t)
    orc.decode(t)
    got = m.prefill(b)
    want = orc.prefill(b)
    assert np.abs(got - want).max() < LOGIT_TOL
    got = m.decode(int(np.argmax(got)))
    want = orc.decode(int(np.argmax(want)))
    assert np.abs(got - want).max() < LOGIT_TOL
    m.close()


def test_errors_leave_model_usable(mini_models):
    cfg = MINI[0]
    m = Model(mini_models[cfg.name], RunConfig(max_seq=16))
    with pytest.raises(native.TFError, match="token id out of range"):
        m.decode(cfg.n_vocab)
    with pytest.raises(native.TFError, match="prefill exceeds max_seq"):
        m.prefill(list(range(17)))
    m.prefill(list(range(15)))
    m.decode(3)
    with pytest.raises(native.TFError, match="decode exceeds max_seq"):
        m.decode(4)
    m.reset()
    assert m.n_pos() == 0
    m.prefill([1, 2, 3])
    m.close()


@pytest.mark.parametrize("kv", [native.TF_KV_F16, native.TF_KV_BF16])
def test_reduced_precision_kv_close(kv, mini_models):
    """fp16 / bf16 caches are an opt-in: logits stay within tolerance of the fp32 cache on
    a short stream (token identity over long streams is only promised for fp32)."""
    cfg = MINI[3]
    path = mini_models[cfg.name]
    prompt = synth.prompt_tokens(cfg, 12)
    a = Model(path, RunConfig(max_seq=64))
    b = Model(path, RunConfig(max_seq=64, kv_type=kv))
    la, lb = a.prefill(prompt), b.prefill(prompt)
    assert np.abs(la - lb).max() < (2e-2 if kv == native.TF_KV_BF16 else 5e-3)
    a.close()
    b.close()


FULL = [("cfg0", 32, 64), ("cfg1", 512, 128), ("cfg2", 128, 128)]


@pytest.mark.slow
@pytest.mark.parametrize("key,n_prompt,n_decode", FULL)
def test_full_config_stream(key, n_prompt, n_decode, model_cache):
    """BASELINE-size model: token-exact greedy stream and logits vs the reference: cfg0
    (32 + 64), cfg1 (512 prompt tokens in tensor-core chunks, decode across the split fused
    attention, 128 steps) and cfg2 (mixed Q4_0 / Q6_K / Q4_1, 128 + 128)."""
    cfg = synth.CONFIGS[key]
    gold_path = os.path.join(GOLDEN, cfg.name + ".npz")
    if not os.path.exists(gold_path):
        pytest.skip("no golden fixture")
    gold = np.load(gold_path)
    path = synth.model_path(cfg, model_cache)
    assert synth.file_digest(path) == str(gold["sha256"])
    m = Model(path, RunConfig(max_seq=cfg.max_seq))
    ids, steps = greedy(m, gold["prompt"], len(gold["tokens"]))
    assert ids == gold["tokens"].tolist()
    err = max(np.abs(lg[gold["topi"][s]] - gold["topv"][s]).max() for s, lg in enumerate(steps))
    assert err < LOGIT_TOL, err
    lsum = max(abs(np.sum(lg, dtype=np.float64) - gold["lsum"][s]) / len(lg) for s, lg in enumerate(steps))
    assert lsum < 1e-4
    print(f"{cfg.name}: token-exact over {len(ids)} steps, top-8 max |diff| {err:.2e}")
    m.close()


@pytest.mark.parametrize("cfg", [MINI[1], MINI[2]], ids=lambda c: c.name)
def test_streamed_upload_matches_synchronous(cfg, mini_models, monkeypatch):
    """The pinned, double-buffered weight upload (host copies overlapping the DMA, small tensors
    packed into one staging buffer, gate/up rows interleaved by 2-D copies) puts the same bytes
    in HBM as one synchronous cudaMemcpy per tensor: bit-identical logits."""
    path = mini_models[cfg.name]
    prompt = synth.prompt_tokens(cfg, 9, stream=31)
    monkeypatch.setenv("TFB200_UPLOAD_SYNC", "1")
    a = Model(path, RunConfig(max_seq=64))
    la = a.prefill(prompt)
    a.close()
    monkeypatch.delenv("TFB200_UPLOAD_SYNC")
    b = Model(path, RunConfig(max_seq=64))
    lb = b.prefill(prompt)
    b.close()
    assert np.array_equal(la, lb)


def test_page_locked_logits_buffer(mini_models):
    """Logits into a tf_host_alloc buffer (direct DMA, no host staging copy) equal those into
    ordinary memory, for prefill and decode."""
    cfg = MINI[0]
    path = mini_models[cfg.name]
    prompt = synth.prompt_tokens(cfg, 20, stream=41)  # >= 16: the tensor-core prefill chunk
    a = Model(path, RunConfig(max_seq=64))
    b = Model(path, RunConfig(max_seq=64))
    pin = native.HostArray(a.n_vocab)
    la = a.prefill(prompt)
    b.prefill(prompt, logits=pin.array)
    assert np.array_equal(la, pin.array)
    t = int(np.argmax(la))
    for _ in range(3):
        la = a.decode(t)
        b.decode(t, logits=pin.array)
        assert np.array_equal(la, pin.array)
        t = int(np.argmax(la))
    pin.close()
    a.close()
    b.close()
