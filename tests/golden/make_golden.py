"""Generate the golden fixtures in tests/golden/ from the REFERENCE engine itself.

Run in a container where the reference sources are present (make -C oracle ref builds
oracle/_ref/ from them); the fixtures are committed and the GPU tests read only them.

  tiny_ci.gguf / tiny_ci.npz   the reference's own CI model, written by its own
                               test_correctness generator (tests/test_correctness.cpp:29-85),
                               and the greedy streams of its 20-prompt gate
                               (tests/test_correctness.cpp:102-109) at stages v0 and v2,
                               with every step's full logits.
  <name>.npz                   seeded synthetic models (tinferno_b200.synth): sha256 of the
                               GGUF the generator must reproduce, the prompt, the stage-v2
                               greedy stream, and per step the top-8 (index, logit) plus the
                               float64 sum and sum of squares of all logits.

  <cfg4 name>-subset.npz       cfg4 (256 sequences x (1024 + 128)): the reference's greedy
                               streams of 4 of the 256 sequences (the batched benchmark's
                               sequences 0, 85, 170 and 255, prompt streams 1000 + g), run
                               one after another as the reference decodes them.

usage: python tests/golden/make_golden.py [--full]   (--full adds the BASELINE-size configs
       and the cfg4 subset)
"""
import argparse
import os
import shutil
import subprocess
import sys
import time

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(ROOT, "agent-serve_b200"))
sys.path.insert(0, os.path.join(ROOT, "oracle"))

import pyoracle as po  # noqa: E402
from tinferno_b200 import synth  # noqa: E402

TOPK = 8


def stream_summary(ref, prompt, n_predict):
    logits = ref.prefill(prompt)
    ids, topi, topv, sums, sq = [], [], [], [], []
    for _ in range(n_predict):
        order = np.argsort(-logits, kind="stable")[:TOPK]
        topi.append(order.astype(np.int32))
        topv.append(logits[order].astype(np.float32))
        sums.append(float(np.sum(logits, dtype=np.float64)))
        sq.append(float(np.sum(logits.astype(np.float64) ** 2)))
        t = int(po.ref_lib().ref_sample_greedy(po._fp(logits), len(logits)))
        ids.append(t)
        logits = ref.decode(t)
    return dict(tokens=np.array(ids, np.int32), topi=np.stack(topi), topv=np.stack(topv),
                lsum=np.array(sums), lsq=np.array(sq))


def tiny_ci():
    subprocess.check_call(["make", "-s", "-C", os.path.join(ROOT, "oracle"), "ref"])
    refdir = os.path.join(ROOT, "oracle", "_ref")
    subprocess.check_call([os.path.join(refdir, "test_correctness")], cwd=refdir)
    dst = os.path.join(HERE, "tiny_ci.gguf")
    shutil.copyfile(os.path.join(refdir, "tiny_ci.gguf"), dst)
    prompts = np.array([[1, 3 + (i % 20), 5 + (i * 3) % 30, 7] for i in range(20)], np.int32)
    out = {"prompts": prompts}
    for stage in ("v0", "v2"):
        toks, logs = [], []
        for pr in prompts:
            ref = po.RefModel(dst, 64, stage=stage)
            lg = ref.prefill(pr)
            st_t, st_l = [], []
            for _ in range(8):
                st_l.append(lg.copy())
                t = int(po.ref_lib().ref_sample_greedy(po._fp(lg), len(lg)))
                st_t.append(t)
                lg = ref.decode(t)
            ref.close()
            toks.append(st_t)
            logs.append(np.stack(st_l))
        out[f"tokens_{stage}"] = np.array(toks, np.int32)
        out[f"logits_{stage}"] = np.stack(logs).astype(np.float32)
    np.savez_compressed(os.path.join(HERE, "tiny_ci.npz"), **out)
    print("tiny_ci: v0 == v2:", np.array_equal(out["tokens_v0"], out["tokens_v2"]))


def synthetic(cfg, n_prompt, n_decode, cache):
    path = os.path.join(cache, f"{cfg.name}-s{cfg.seed}.gguf")
    if not os.path.exists(path):
        synth.write_model(cfg, path)
    prompt = synth.prompt_tokens(cfg, n_prompt)
    t0 = time.time()
    ref = po.RefModel(path, max(cfg.max_seq, n_prompt + n_decode + 1), stage="v2")
    s = stream_summary(ref, prompt, n_decode)
    ref.close()
    name = cfg.name
    np.savez_compressed(os.path.join(HERE, f"{name}.npz"), sha256=synth.file_digest(path), prompt=prompt,
                        n_threads=0, **s)
    print(f"{name}: {n_prompt}+{n_decode} in {time.time() - t0:.1f}s tokens[:8]={s['tokens'][:8].tolist()}")


CFG4_SUBSET = (0, 85, 170, 255)   # sequences of the batched benchmark (prompt stream 1000 + g)


def cfg4_subset(cache):
    cfg = synth.CFG4
    path = os.path.join(cache, f"{cfg.name}-s{cfg.seed}.gguf")
    if not os.path.exists(path):
        synth.write_model(cfg, path)
    out = {"sha256": synth.file_digest(path), "seqs": np.array(CFG4_SUBSET, np.int32)}
    per = {k: [] for k in ("prompt", "tokens", "topi", "topv", "lsum", "lsq")}
    for g in CFG4_SUBSET:
        t0 = time.time()
        prompt = synth.prompt_tokens(cfg, cfg.n_prompt, stream=1000 + g)
        ref = po.RefModel(path, cfg.max_seq, stage="v2")
        s = stream_summary(ref, prompt, cfg.n_decode)
        ref.close()
        per["prompt"].append(prompt)
        for k in ("tokens", "topi", "topv", "lsum", "lsq"):
            per[k].append(s[k])
        print(f"cfg4 seq {g}: {cfg.n_prompt}+{cfg.n_decode} in {time.time() - t0:.1f}s "
              f"tokens[:8]={s['tokens'][:8].tolist()}", flush=True)
    for k, v in per.items():
        out[k] = np.stack(v)
    np.savez_compressed(os.path.join(HERE, f"{cfg.name}-subset.npz"), **out)


MINIS = [
    (synth.mini(synth.CFG0, 2, 4096), 12, 12),
    (synth.mini(synth.CFG1, 2, 4096), 12, 12),
    (synth.mini(synth.CFG2, 2, 4096), 12, 12),
    (synth.mini(synth.CFG4, 2, 4096), 12, 12),
    (synth.mini(synth.CFG0_LLAMA3, 2, 4096), 40, 24),
]


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--full", action="store_true")
    ap.add_argument("--only", default="")
    args = ap.parse_args()
    cache = os.environ.get("TFB200_CACHE", "/tmp/tfb200_models")
    os.makedirs(cache, exist_ok=True)
    if not args.only or args.only == "tiny":
        tiny_ci()
    for cfg, npr, ndec in MINIS:
        if not args.only or args.only in cfg.name:
            synthetic(cfg, npr, ndec, cache)
    if args.full:
        for key, n_prompt, n_decode in (("cfg0", 32, 64), ("cfg1", 512, 128), ("cfg2", 128, 128)):
            cfg = synth.CONFIGS[key]
            if not args.only or args.only in cfg.name:
                synthetic(cfg, n_prompt, n_decode, cache)
        if not args.only or args.only == "cfg4-subset":
            cfg4_subset(cache)


if __name__ == "__main__":
    main()
