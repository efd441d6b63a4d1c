"""Benchmark of the hot path: greedy decode of the BASELINE cfg0 model (Llama-3.2-1B
architecture, Q8_0, synthetic seeded weights) at batch 1 on each GPU.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

A step is one decoded token.  The timed region holds K steps after W warm-up steps, after a
32-token prompt prefill, bracketed by a barrier and a device synchronise, timed with CUDA
events on the engine's stream; the job value is the max over ranks.  With N > 1 every rank
runs an independent replica of the batch-1 decode on its own GPU (the batch-1 path does not
shard: replicas only) and the value is the aggregate tok/s.

  value      tok/s with the token fed back on the device (graph replays, no host round trip)
  e2e        tok/s through the reference-facing call tf_cuda_decode(token -> host logits),
             one host->device token copy and one device->host logits copy per step
  roofline   the step's kernel (every launch of the decode step runs it): the bytes a step
             must read (weights + cached K/V) over the CUDA-event time per step, vs
             MEASURED_PEAKS.json (frac) and the 8 TB/s specification (frac_of_nominal);
             roofline_lmhead is the same kernel timed alone on the lm_head shape
  configs    (N = 1) batch-1 prefill + decode of cfg0 / cfg1 / cfg2 at their BASELINE lengths
  batched    cfg4: 256 sequences sharded over the ranks, with the greedy ids of the golden
             subset compared against the reference build's (after the timed region)
  cpu_baseline  the reference engine's stage-v2 path (oracle/_ref, built from the reference's
             own sources) on this host's cores, on a bounded sample of the same decode

--impl reference times only the reference's CPU decode of the same workload (rank 0).
"""
import argparse
import ctypes as C
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "agent-serve_b200"))

from tinferno_b200 import synth  # noqa: E402

CFG = synth.CFG0
PROMPT = 32
# DRAM bytes (read + write) of one lm_head GEMV launch, from an ncu capture of
# `bench.py --kernel lmhead` (profiles/gemv_q8_0_lmhead_128256x2048.md)
LMHEAD_TRAFFIC = 283_513_088
# the kernel every launch of the batch-1 decode step runs, and its DRAM bytes per step (sum
# over the step's launches of one ncu capture), when measured
STEP_KERNEL = "tf_gemv_kernel<1, 1> (Q8_0 integer-path GEMV; attention fused into the QKV launches)"
STEP_TRAFFIC = 1_323_928_576
STEP_TRAFFIC_SOURCE = ("ncu dram__bytes_read+write summed over the 65 launches of one step at position 35, "
                       "profiles/decode_step_cfg0_dram.md")


# B200 HBM3e bandwidth as specified (8 TB/s), reported beside the measured copy peak
HBM_NOMINAL_GBS = 8000.0


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 20 ms during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        self.idx = gpu_index
        self.proc = None
        self.path = None

    def start(self):
        """Start sampling and wait (up to 3 s) for the first sample, so that even a short timed
        region that follows is covered."""
        fd, self.path = tempfile.mkstemp(suffix=".csv")
        os.close(fd)
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                                          "-lms", "20", "-i", str(self.idx)], stdout=open(self.path, "w"),
                                         stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None
            return
        t0 = time.time()
        while time.time() - t0 < 3.0 and os.path.getsize(self.path) == 0:
            time.sleep(0.05)

    def stop(self):
        if not self.proc:
            return None
        self.proc.terminate()
        try:
            self.proc.wait(5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        rows = []
        for line in open(self.path):
            f = [x.strip() for x in line.split(",")]
            if len(f) >= 9:
                rows.append(f)
        os.unlink(self.path)
        if not rows:
            return None
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        reasons = set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in rows:
            for n, v in zip(names, r[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None,
                "sm_max_mhz": float(rows[0][2]) if rows[0][2].replace(".", "").isdigit() else None,
                "reasons": sorted(reasons), "samples": len(rows)}


def model_file(cfg=None):
    cache = os.environ.get("TFB200_CACHE", "/tmp/tfb200_models")
    return synth.model_path(cfg or CFG, cache)


BATCH_CFG = synth.CFG4
BATCH_SEQS = 256      # cfg4: 256 independent sequences
BATCH_PROMPT = 1024   # each with a 1024-token prompt


def run_batched(args, rank, world, local_rank, dist):
    """cfg4 batched greedy decode: the 256 sequences sharded contiguously over the ranks
    (weights replicated, no collective on the data path).  Each rank prefills its shard
    (tf_cuda_prefill_batch: 1024 steps of S rows on the tensor-core GEMM path), runs W
    untimed decode steps, then times K steps of tf_cuda_decode_batch (host token ids in,
    greedy ids out, every step) with CUDA events; the job value is all sequences' tokens over
    the slowest rank's time."""
    import torch
    from tinferno_b200 import shard
    from tinferno_b200.model import Model, RunConfig

    cfg = BATCH_CFG
    steps, warm = args.batched_steps, 3
    s0, s1 = shard.shard_range(BATCH_SEQS, rank, world)
    S = s1 - s0
    if rank == 0:
        model_file(cfg)
    if dist:
        dist.barrier()
    m = Model(model_file(cfg), RunConfig(max_seq=BATCH_PROMPT + warm + steps, max_batch=S, device=local_rank))
    stream = torch.cuda.ExternalStream(m.stream)
    prompts = np.stack([synth.prompt_tokens(cfg, BATCH_PROMPT, stream=1000 + g) for g in range(s0, s1)])
    slots = list(range(S))
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    tok = m.prefill_batch(slots, prompts)
    torch.cuda.synchronize()
    prefill_s = time.perf_counter() - t0
    hist = [tok]  # every step's ids come back to the host anyway; kept for the parity check
    for _ in range(warm):
        tok = m.decode_batch(slots, tok.tolist())
        hist.append(tok)
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev0.record(stream)
    for _ in range(steps):
        tok = m.decode_batch(slots, tok.tolist())
        hist.append(tok)
    ev1.record(stream)
    torch.cuda.synchronize()
    ms = ev0.elapsed_time(ev1)
    # parity (after the timed region): the reference build's greedy ids of the golden subset
    # of sequences, where this rank holds them
    checked, failed, compared = 0, 0, 0
    gold_path = os.path.join(ROOT, "tests", "golden", cfg.name + "-subset.npz")
    if os.path.exists(gold_path):
        gold = np.load(gold_path)
        ids = np.stack(hist)  # [1 + warm + steps][S]
        for i, g in enumerate(gold["seqs"].tolist()):
            if s0 <= g < s1:
                n = min(ids.shape[0], gold["tokens"].shape[1])
                checked += 1
                compared = n
                failed += int(not np.array_equal(ids[:n, g - s0], gold["tokens"][i][:n]))
    t = torch.tensor([ms, prefill_s], device="cuda")
    pc = torch.tensor([checked, failed, compared], device="cuda", dtype=torch.float64)
    if dist:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        dist.all_reduce(pc, op=dist.ReduceOp.SUM)
    ms_max, prefill_max = float(t[0].item()), float(t[1].item())
    n_chk, n_fail = int(pc[0].item()), int(pc[1].item())
    parity = {"status": ("ok" if n_fail == 0 else "fail") if n_chk else "no golden",
              "sequences_checked": n_chk, "sequences_failed": n_fail,
              "ids_per_sequence": compared if n_chk else 0,
              "against": "greedy ids of the reference build (tests/golden/" + cfg.name + "-subset.npz)"}
    kps = m.kernels_per_step
    m.close()
    cpu = batched_cpu_baseline(cfg) if (rank == 0 and world == 1 and not args.no_cpu) else None
    wb = synth.weight_bytes(cfg)
    kv_pos = 2 * cfg.n_layer * cfg.n_kv_head * (cfg.n_embd // cfg.n_head) * 4  # fp32 K+V bytes per position
    ctx = BATCH_PROMPT + warm + steps / 2
    step_bytes = wb + S * ctx * kv_pos
    return {"metric": "batched decode tok/s (cfg4 Qwen2.5-1.5B Q8_0, 256 sequences, 1024-token prompts)",
            "value": round(BATCH_SEQS * steps / (ms_max / 1e3), 1), "unit": "tok/s", "n_gpus": world,
            "sequences_per_gpu": S, "steps": steps, "warmup": warm, "ms_per_step": round(ms_max / steps, 3),
            "scaling": "strong", "prefill_s": round(prefill_max, 2),
            "prefill_tok_s": round(BATCH_SEQS * BATCH_PROMPT / prefill_max, 1),
            "hbm_roofline": {"bytes_per_step_per_gpu": int(step_bytes),
                             "achieved_gbs": round(step_bytes / (ms_max / steps / 1e3) / 1e9, 1),
                             "frac_of_peak": round(step_bytes / (ms_max / steps / 1e3) / 1e9 / peaks()[0], 4),
                             "frac_of_nominal": round(step_bytes / (ms_max / steps / 1e3) / 1e9 / HBM_NOMINAL_GBS, 4)},
            "parity": parity,
            "path": "tcgen05 GEMM (f16-split, TMEM accumulator) at >= 16 rows per step, split flash-decode attention",
            "e2e": "every step copies S token ids in and S greedy ids out (host)", "cpu_baseline": cpu}


def batched_cpu_baseline(cfg):
    """The reference's CPU path on the batched workload: it decodes one sequence per Model, so
    its aggregate rate over the 256 sequences is its one-sequence rate.  Bounded sample: one
    sequence, a 32-token prompt instead of 1024 (untimed), 3 untimed + up to 64 timed decode
    steps (~10 s); at the 1024-token context its per-token K/V reads add ~4 % to the 1.64 GB
    of weights a step reads."""
    try:
        prompt = synth.prompt_tokens(cfg, 32, stream=1000)
        tps, n, threads, kind = cpu_reference_decode(model_file(cfg), prompt, 64, max_seconds=10.0)
        return {"value": round(tps, 3), "unit": "tok/s", "cores": threads, "kind": kind,
                "sample": f"1 of the 256 sequences, 32-token prompt (untimed), 3 untimed + {n} timed decode "
                          "steps; sequences run one after another, so this is the aggregate rate"}
    except Exception as e:  # the baseline must never take the GPU measurement down with it
        return {"unavailable": f"{type(e).__name__}: {e}"[:200]}


def cpu_reference_decode(path, prompt, n_tokens, max_seconds=None, warm=3):
    """Reference (oracle/_ref, stage v2, all host threads) when built, else the oracle port.
    Prefill and `warm` decode steps untimed; times up to n_tokens further decode steps;
    returns (tok/s, tokens, threads, kind)."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import pyoracle as po
    if po.ref_available():
        m = po.RefModel(path, 2048, stage="v2")
        kind, threads = "reference", m.n_threads
    else:
        from tinferno_b200 import gguf
        threads = os.cpu_count() or 1
        m = po.OracleModel(gguf.GGUFReader(path), 2048, threads=threads)
        kind = "port"
    logits = m.prefill(prompt)
    t = int(np.argmax(logits))
    for _ in range(warm):
        t = int(np.argmax(m.decode(t)))
    n = 0
    t0 = time.perf_counter()
    while n < n_tokens:
        logits = m.decode(t)
        t = int(np.argmax(logits))
        n += 1
        if max_seconds and time.perf_counter() - t0 > max_seconds:
            break
    dt = time.perf_counter() - t0
    m.close()
    return n / dt, n, threads, kind


def run_reference(args, rank):
    if rank != 0:
        return
    path = model_file()
    prompt = synth.prompt_tokens(CFG, PROMPT)
    # W untimed warm-up steps, then K timed steps, within one generation (positions 32 .. 32+W+K)
    warm = max(3, args.warmup)
    tps, n, threads, kind = cpu_reference_decode(path, prompt, args.steps, warm=warm)
    line = {"metric": "decode tok/s (batch 1, cfg0 Llama-3.2-1B Q8_0)", "value": round(tps, 3), "unit": "tok/s",
            "impl": "reference", "n_gpus": args.gpus, "steps": n, "warmup": warm, "ms_per_step": round(1e3 / tps, 3),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": "cfg0 batch-1 greedy decode after a 32-token prompt", "model": CFG.name,
                       "global_batch": 1, "seq_len": PROMPT + warm + n, "parallelism": "cpu threads"},
            "cpu_baseline": {"value": round(tps, 3), "unit": "tok/s", "cores": threads, "kind": kind,
                             "sample": f"1 sequence, {PROMPT}-token prompt (untimed prefill), {warm} untimed + "
                                       f"{n} timed decode steps"},
            "e2e": {"value": round(tps, 3), "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def run_ours(args, rank, world, local_rank, dist):
    import torch
    from tinferno_b200 import native
    from tinferno_b200.model import Model, RunConfig

    torch.cuda.set_device(local_rank)
    if rank == 0:
        path = model_file()
    if dist:
        dist.barrier()
    path = model_file()
    m = Model(path, RunConfig(max_seq=CFG.max_seq, device=local_rank))
    stream = torch.cuda.ExternalStream(m.stream)
    prompt = synth.prompt_tokens(CFG, PROMPT)
    L = m.L

    def prefill():
        m.reset(0)
        return int(np.argmax(m.prefill(prompt)))

    # ---- value: device-resident decode (graph replays, argmax fed back on the device) ----
    out = np.zeros(args.steps, np.int32)
    n_out = C.c_int(0)
    first = prefill()
    ids = m.generate_greedy(first, args.warmup)  # W untimed steps (graph captured and warm)
    nxt = ids[-1]  # the timed steps continue the stream at positions 32+W ..
    replica_ids = list(ids)
    clocks = ClockSampler(local_rank)
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    clocks.start()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev0.record(stream)
    native.check(L.tf_cuda_generate_greedy(m.h, 0, int(nxt), args.steps, -1, out.ctypes.data_as(native.i32p),
                                           C.byref(n_out)), m.h)
    ev1.record(stream)
    torch.cuda.synchronize()
    ms = ev0.elapsed_time(ev1)
    clk = clocks.stop()
    replica_ids += [int(v) for v in out[1:n_out.value]]
    if dist:
        dist.barrier()
    t = torch.tensor([ms], device="cuda")
    if dist:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms_max = float(t.item())
    value = world * args.steps / (ms_max / 1e3)

    # ---- e2e: the reference-facing call with host token in and host logits out ----
    first = prefill()
    tok = first
    # the caller's logits buffer in page-locked memory (tf_host_alloc): the D2H copy lands in
    # it directly
    host_logits = native.HostArray(m.n_vocab)
    logits = host_logits.array
    for _ in range(args.warmup):
        m.decode(tok, logits)
        tok = m.last_argmax
    if dist:
        dist.barrier()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        m.decode(tok, logits)
        tok = m.last_argmax
    e2e_s = time.perf_counter() - t0
    t = torch.tensor([e2e_s], device="cuda")
    if dist:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    e2e = world * args.steps / float(t.item())
    host_logits.close()

    # ---- vocab-split lm_head (N > 1): every rank decodes the same sequence and computes V/N of
    # the lm_head rows; one NCCL int64 max all-reduce of the greedy key per step ----
    vsplit = None
    if dist and world > 1:
        from tinferno_b200 import shard
        first = prefill()
        m.set_vocab_shard(rank, world)
        red = shard.nccl_key_reducer(m, dist)
        ids_w = shard.split_greedy(m, first, args.warmup, red)
        dist.barrier()
        torch.cuda.synchronize()
        ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        ev0.record(stream)
        for i in range(args.steps):
            m.decode_shard(ids_w[-1] if i == 0 else -1)
            red()
        ev1.record(stream)
        m.shard_token()
        torch.cuda.synchronize()
        ids_k = [ids_w[-1]] + m.history(args.steps - 1)
        t = torch.tensor([ev0.elapsed_time(ev1)], device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms_split = float(t.item())
        # the same stream as the replica leg (value): [first, W warm-up ids] then the timed ids
        same = ids_w == replica_ids[:len(ids_w)] and ids_k == replica_ids[len(ids_w) - 1:len(ids_w) - 1 + len(ids_k)]
        ok = torch.tensor([1 if same else 0], device="cuda")
        dist.all_reduce(ok, op=dist.ReduceOp.MIN)
        m.set_vocab_shard(0, 1)
        vsplit = {"metric": "batch-1 decode tok/s of ONE sequence with the lm_head split over the GPUs",
                  "tok_s": round(args.steps / (ms_split / 1e3), 1), "ms_per_step": round(ms_split / args.steps, 4),
                  "n_gpus": world, "lm_head_rows_per_gpu": CFG.n_vocab // world,
                  "collective": "NCCL int64 max all-reduce of the greedy key, one per step, on the model's stream",
                  "ids_equal_replica_stream": bool(ok.item())}

    # ---- the lm_head-shape GEMV alone (secondary roofline figure) ----
    roof_lm = None
    if rank == 0:
        roof_lm = gemv_roofline(torch, native, m)
    kps = m.kernels_per_step
    m.close()
    upload = upload_timing(path, local_rank) if rank == 0 else None

    if rank == 0:
        cpu = None
        if not args.no_cpu and world == 1:
            tps, n, threads, kind = cpu_reference_decode(path, prompt, 512, max_seconds=15.0)
            cpu = {"value": round(tps, 3), "unit": "tok/s", "cores": threads, "kind": kind,
                   "sample": f"1 sequence, {PROMPT}-token prompt (untimed prefill), 3 untimed + {n} timed "
                             "decode steps (~15 s)"}
        wb = synth.weight_bytes(CFG)
        # bytes one decode step reads: every weight (GGUF::weight_bytes, src/gguf.cpp:219-223)
        # + the fp32 K/V rows of every cached position, at the timed region's mean position
        kv_pos = 2 * CFG.n_layer * CFG.n_kv_head * CFG.head_dim * 4
        mean_pos = PROMPT + args.warmup + args.steps / 2
        step_bytes = wb + kv_pos * mean_pos
        peak, peak_kind = peaks()
        ach = step_bytes / (ms_max / args.steps / 1e3) / 1e9
        roof = {"bound": "hbm", "kernel": STEP_KERNEL, "scope": "every launch of the decode step (the whole "
                "step runs on this kernel), timed with CUDA events over the timed region",
                "achieved": round(ach, 1), "peak": peak, "unit": "GB/s", "frac": round(ach / peak, 4),
                "nominal_peak": HBM_NOMINAL_GBS, "frac_of_nominal": round(ach / HBM_NOMINAL_GBS, 4),
                "peak_kind": peak_kind, "traffic": STEP_TRAFFIC, "traffic_source": STEP_TRAFFIC_SOURCE,
                "algorithmic_bytes_per_step": int(step_bytes)}
        line = {"metric": "decode tok/s (batch 1, cfg0 Llama-3.2-1B Q8_0)", "value": round(value, 2), "unit": "tok/s",
                "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
                "ms_per_step": round(ms_max / args.steps, 4), "higher_is_better": True, "scaling": "weak",
                "vs_baseline": None, "dtype": "f32", "data": "synthetic",
                "config": {"workload": "cfg0 batch-1 greedy decode after a 32-token prompt (replicas per GPU)",
                           "model": CFG.name, "global_batch": world, "seq_len": PROMPT + args.warmup + args.steps,
                           "parallelism": f"replicas x{world}", "kv_cache": "f32",
                           "l2": "weights 1.31 GB per step stream through the 126 MB L2 (inputs larger than L2)"},
                "roofline": roof, "roofline_lmhead": roof_lm, "cpu_baseline": cpu,
                "e2e": {"value": round(e2e, 2), "unit": "tok/s", "h2d_bytes_per_step": 8,
                        "d2h_bytes_per_step": 4 * CFG.n_vocab + 8},
                "gpu_launches": kps * args.steps, "kernels_per_step": kps, "clocks": clk, "upload": upload,
                "vocab_split": vsplit}
        if world == 1 and not args.no_configs:
            try:
                line["configs"] = config_runs()
            except Exception as e:  # never fatal to the headline line
                line["configs"] = {"unavailable": f"{type(e).__name__}: {e}"[:200]}
            try:  # BASELINE cfg3, the isolated dequant-matmul sweep (bounded in time)
                sw = matmul_sweep(quiet=True, max_seconds=60)
                line["cfg3_sweep"] = {"columns": ["type", "N", "K", "M", "path", "us", "GB_s", "hbm_frac", "TFLOP_s"],
                                      "rows": [[r["type"], r["N"], r["K"], r["M"], r["path"], r["us"], r["GB_s"],
                                                r["hbm_frac"], r["TFLOP_s"]] for r in sw]}
            except Exception as e:  # never fatal to the headline line
                line["cfg3_sweep"] = {"unavailable": f"{type(e).__name__}: {e}"[:200]}
    batched = None
    if not args.no_batched:
        batched = run_batched(args, rank, world, local_rank, dist)
    if rank == 0:
        line["batched"] = batched
        print(json.dumps(line), flush=True)


def upload_timing(path, device):
    """Seconds tf_cuda_create takes for the cfg0 model (1.31 GB, file pages already cached by
    the earlier load), with the pinned double-buffered upload and with one synchronous
    pageable cudaMemcpy per tensor (TFB200_UPLOAD_SYNC=1)."""
    from tinferno_b200.model import Model, RunConfig
    out = {}
    for name, env in (("streamed", None), ("synchronous", "1")):
        if env:
            os.environ["TFB200_UPLOAD_SYNC"] = env
        else:
            os.environ.pop("TFB200_UPLOAD_SYNC", None)
        t0 = time.perf_counter()
        m = Model(path, RunConfig(max_seq=64, device=device))
        out[name + "_s"] = round(time.perf_counter() - t0, 3)
        m.close()
    os.environ.pop("TFB200_UPLOAD_SYNC", None)
    out["bytes"] = synth.weight_bytes(CFG)
    out["streamed_GB_s"] = round(out["bytes"] / out["streamed_s"] / 1e9, 2)
    out["scope"] = "tf_cuda_create wall time (upload, KV cache, tables, graph-free set-up)"
    return out


def gemv_roofline(torch, native, m, reps=50, warm=5):
    """Time tf_op_matmul (the engine's dequant-GEMV kernel) on the lm_head shape: 128256 x 2048
    Q8_0 weights (279 MB, > L2) times one fp32 row."""
    from tinferno_b200 import quants
    N, K = CFG.n_vocab, CFG.n_embd
    rb = K // 32 * 34
    nbytes = N * rb
    W = torch.empty(nbytes, dtype=torch.uint8, device="cuda")
    # fill with valid Q8_0 blocks: random int8 quants, scale 1/127
    W.view(N, K // 32, 34)[:, :, 2:] = torch.randint(-127, 128, (N, K // 32, 32), device="cuda").to(torch.int8).view(torch.uint8)
    d = np.float16(1.0 / 127).view(np.uint16)
    W.view(N, K // 32, 34)[:, :, 0] = int(d & 0xFF)
    W.view(N, K // 32, 34)[:, :, 1] = int(d >> 8)
    x = torch.randn(K, device="cuda")
    y = torch.empty(N, device="cuda")
    st = torch.cuda.current_stream()
    L = native.lib()
    for _ in range(warm):
        native.check(L.tf_op_matmul(C.c_void_p(y.data_ptr()), C.c_void_p(x.data_ptr()), native.TF_Q8_0,
                                    C.c_void_p(W.data_ptr()), N, K, 1, C.c_void_p(st.cuda_stream)))
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(reps)]
    for a, b in evs:
        a.record(st)
        native.check(L.tf_op_matmul(C.c_void_p(y.data_ptr()), C.c_void_p(x.data_ptr()), native.TF_Q8_0,
                                    C.c_void_p(W.data_ptr()), N, K, 1, C.c_void_p(st.cuda_stream)))
        b.record(st)
    torch.cuda.synchronize()
    ts = sorted(a.elapsed_time(b) for a, b in evs)
    t = statistics.median(ts) / 1e3
    alg = nbytes + K * 4 + N * 4
    peak, kind = peaks()
    ach = alg / t / 1e9
    return {"bound": "hbm", "kernel": "tf_gemv_kernel<1> (Q8_0, lm_head 128256x2048)", "achieved": round(ach, 1),
            "peak": peak, "unit": "GB/s", "frac": round(ach / peak, 4), "peak_kind": kind,
            "traffic": LMHEAD_TRAFFIC, "traffic_source": "ncu dram__bytes_read+write of one launch, "
            "profiles/gemv_q8_0_lmhead_128256x2048.md", "algorithmic_bytes": alg, "launch_us": round(t * 1e6, 2)}


def q6k_gemv():
    """The Q6_K integer-path GEMV (the kind of cfg2's 215 MB lm_head) on 16384 x 2048 weights
    (N(0, 0.02) quantised, 27.5 MB) times one N(0, 1) fp32 row: eight device copies rotate so
    every timed launch reads its weights from HBM (220 MB > L2); CUDA events, median of 20."""
    import torch
    from tinferno_b200 import native, quants, gguf
    N, K = 16384, CFG.n_embd
    rng = np.random.default_rng(6)
    raw = np.ascontiguousarray(quants.quantize((rng.standard_normal((N, K)) * 0.02).astype(np.float32),
                                               gguf.GGML_Q6_K)).reshape(-1)
    W = [torch.from_numpy(raw).cuda() for _ in range(8)]
    x = torch.randn(K, device="cuda")
    y = torch.empty(N, device="cuda")
    st = torch.cuda.current_stream()
    L = native.lib()

    def launch(i):
        native.check(L.tf_op_matmul(C.c_void_p(y.data_ptr()), C.c_void_p(x.data_ptr()), native.TF_Q6_K,
                                    C.c_void_p(W[i % 8].data_ptr()), N, K, 1, C.c_void_p(st.cuda_stream)))

    for i in range(3):
        launch(i)
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(20)]
    for i, (a, b) in enumerate(evs):
        a.record(st)
        launch(i)
        b.record(st)
    torch.cuda.synchronize()
    t = statistics.median(sorted(a.elapsed_time(b) for a, b in evs)) / 1e3
    alg = raw.nbytes + K * 4 + N * 4
    peak, kind = peaks()
    return {"kernel": "tf_gemv_kernel<1, 3> (Q6_K integer path, 16384x2048)", "achieved": round(alg / t / 1e9, 1),
            "peak": peak, "unit": "GB/s", "frac": round(alg / t / 1e9 / peak, 4), "peak_kind": kind,
            "algorithmic_bytes": alg, "launch_us": round(t * 1e6, 2)}


def config_runs():
    """Batch-1 runs of cfg0 / cfg1 / cfg2 as BASELINE states them (prompt, decode tokens): the
    prompt prefill (tf_cuda_prefill: chunked tensor-core GEMM for the Q8_0 / Q4_0 matrices, the
    multi-row GEMV for cfg2's Q4_1 / Q6_K ones) and the device-resident greedy decode
    (tf_cuda_generate_greedy), each
    timed with CUDA events; decode against the weight + KV bytes per token."""
    import torch
    from tinferno_b200 import native
    from tinferno_b200.model import Model, RunConfig
    peak = peaks()[0]
    out = []
    for cfg, n_prompt, n_decode in ((synth.CFG0, 32, 64), (synth.CFG1, 512, 128), (synth.CFG2, 128, 128)):
        m = Model(model_file(cfg), RunConfig(max_seq=cfg.max_seq))
        stream = torch.cuda.ExternalStream(m.stream)
        prompt = synth.prompt_tokens(cfg, n_prompt)
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(4)]
        for rep in range(2):  # the second prefill and decode are timed (graphs captured, warm)
            m.reset(0)
            torch.cuda.synchronize()
            ev[0].record(stream)
            first = int(np.argmax(m.prefill(prompt)))
            ev[1].record(stream)
            ids = np.zeros(n_decode, np.int32)
            n_out = C.c_int(0)
            ev[2].record(stream)
            native.check(m.L.tf_cuda_generate_greedy(m.h, 0, first, n_decode, -1, ids.ctypes.data_as(native.i32p),
                                                     C.byref(n_out)), m.h)
            ev[3].record(stream)
            torch.cuda.synchronize()
        pre_ms, dec_ms = ev[0].elapsed_time(ev[1]), ev[2].elapsed_time(ev[3])
        kv_per_pos = 2 * cfg.n_layer * cfg.n_kv_head * (cfg.n_embd // cfg.n_head) * 4
        mean_pos = n_prompt + n_decode / 2
        bytes_tok = synth.weight_bytes(cfg) + kv_per_pos * mean_pos
        tok_s = n_decode / (dec_ms / 1e3)
        out.append({"config": cfg.name, "prompt": n_prompt, "decode": n_decode,
                    "prefill_tok_s": round(n_prompt / (pre_ms / 1e3), 1), "decode_tok_s": round(tok_s, 1),
                    "bytes_per_token": int(bytes_tok), "hbm_frac": round(bytes_tok * tok_s / 1e9 / peak, 3)})
        m.close()
    return out


def launch_trace(steps=6, model_path=None):
    """Per-launch breakdown of one cfg0 decode step on the per-kernel path: every CTA of every
    GEMV launch stamps %globaltimer at entry, after griddepcontrol.wait, prologue done, rows
    done and exit (TFB200_GV_TRACE=1, tf_cuda_launch_trace); the chain per launch kind is
    averaged over the layers (times in us, relative to the previous launch's last exit)."""
    from tinferno_b200 import native
    from tinferno_b200.model import Model, RunConfig
    os.environ["TFB200_GV_TRACE"] = "1"
    try:
        m = Model(model_path or model_file(), RunConfig(max_seq=CFG.max_seq))
    finally:
        del os.environ["TFB200_GV_TRACE"]
    t = int(np.argmax(m.prefill(synth.prompt_tokens(CFG, PROMPT))))
    for _ in range(steps):
        t = m.decode_argmax(t)
    ML, CT, SL = 192, 512, 10
    buf = np.zeros(ML * CT * SL, np.uint64)
    meta = np.zeros(ML * 3, np.int32)
    nl = np.zeros(1, np.int32)
    native.check(m.L.tf_cuda_launch_trace(m.h, buf.ctypes.data_as(C.POINTER(C.c_ulonglong)), ML,
                                          meta.ctypes.data_as(native.i32p), nl.ctypes.data_as(native.i32p)), m.h)
    m.close()
    n = int(nl[0])
    tr = buf.reshape(ML, CT, SL)[:n].astype(np.int64)
    meta = meta.reshape(ML, 3)[:n]
    kinds = {0: "qkv+attention", 1: "wo", 2: "gate/up", 3: "down", 4: "lm_head"}
    seg, prev_exit, t0 = {}, None, None
    for i in range(n):
        grid, na, kind = (int(v) for v in meta[i])
        g, at = tr[i, na:grid], tr[i, :na]
        ex = max(int(g[:, 4].max()), int(at[:, 4].max()) if na else 0)
        t0 = int(g[:, 0].min()) if t0 is None else t0
        if prev_exit is not None:
            d = seg.setdefault(kinds[kind], {})
            wf = int(g[:, 1].min())
            vals = [("first entry", int(g[:, 0].min()) - prev_exit),
                    ("last entry", int(g[:, 0].max()) - prev_exit),
                    ("first wait release", wf - prev_exit),
                    ("last wait release", int(g[:, 1].max()) - prev_exit),
                    ("longest prologue", int((g[:, 2] - g[:, 1]).max())),
                    ("last prologue done", int(g[:, 2].max()) - prev_exit),
                    ("last rows done", int(g[:, 3].max()) - prev_exit),
                    ("last GEMV exit", int(g[:, 4].max()) - prev_exit)]
            # the GEMV CTA whose wait released last, stamp by stamp
            lc = g[int(np.argmax(g[:, 1]))]
            vals += [("latest CTA: entry", int(lc[0]) - prev_exit), ("latest CTA: before wait", int(lc[5]) - prev_exit),
                     ("latest CTA: wait release", int(lc[1]) - prev_exit)]
            if kind != 4 and int(g[:, 6].min()) > 0:
                vals += [("longest: wait release -> activation loaded", int((g[:, 6] - g[:, 1]).max())),
                         ("longest: activation loaded -> first barrier", int((g[:, 7] - g[:, 6]).max())),
                         ("longest: first barrier -> prologue done", int((g[:, 2] - g[:, 7]).max()))]
            if na:
                vals += [("attention, longest: q/k/v ready -> loaded", int((at[:, 5] - at[:, 2]).max())),
                         ("attention, longest: loaded -> tiles done", int((at[:, 6] - at[:, 5]).max())),
                         ("attention, longest: loaded -> rotated and stored", int((at[:, 8] - at[:, 5]).max())),
                         ("attention, longest: rotated and stored -> first tile's scores", int((at[:, 9] - at[:, 8]).max())),
                         ("attention, longest: first tile's scores -> softmax sums", int((at[:, 7] - at[:, 9]).max())),
                         ("attention, longest: first tile's softmax sums -> tiles done", int((at[:, 6] - at[:, 7]).max())),
                         ("attention, mean: loaded -> tiles done", float((at[:, 6] - at[:, 5]).mean())),
                         ("attention, longest: tiles done -> output written", int((at[:, 3] - at[:, 6]).max()))]
                vals += [("attention: last q/k/v ready", int(at[:, 2].max()) - prev_exit),
                         ("attention: last done", int(at[:, 3].max()) - prev_exit)]
            vals.append(("launch exit (chain)", ex - prev_exit))
            for name, v in vals:
                d.setdefault(name, []).append(v / 1e3)
        prev_exit = ex
    return {"kernel": "gvtrace", "step_us": round((prev_exit - t0) / 1e3, 1), "launches": n,
            "per_kind_mean_us_after_previous_exit": {k: {s: round(float(np.mean(v)), 2) for s, v in d.items()}
                                                     for k, d in seg.items()}}


def matmul_sweep(quiet=False, max_seconds=None):
    """BASELINE cfg3: Y[M,N] = X[M,K] W[N,K]^T for Q8_0 and Q4_0 weights (N(0, 0.02) quantised),
    X ~ N(0, 1); K=2048 with N in {512, 2048, 8192, 128256}, K=8192 with N=2048; M in
    {1, 8, 64, 512}.  Weight copies rotate so that every timed launch reads its weights from
    HBM (the rotation exceeds the 126 MB L2).  M <= 8 runs the dequant-GEMV, M >= 16 the
    tensor-core GEMM for both types (timed without the one-off scale pass of the matrix).
    quiet: no per-shape lines on stdout; max_seconds: stop after the shape that passes it."""
    import torch
    from tinferno_b200 import gguf, native, quants
    L = native.lib()
    st = torch.cuda.current_stream()
    rows = []
    peak = peaks()[0]
    t_start = time.perf_counter()
    for t, tname in ((gguf.GGML_Q8_0, "Q8_0"), (gguf.GGML_Q4_0, "Q4_0")):
        for K, N in ((2048, 512), (2048, 2048), (2048, 8192), (2048, 128256), (8192, 2048)):
            if max_seconds and time.perf_counter() - t_start > max_seconds:
                break
            rng = np.random.default_rng(K + N)
            w = (rng.standard_normal((N, K)) * 0.02).astype(np.float32)
            raw = np.ascontiguousarray(quants.quantize(w, t)).reshape(-1)
            nbytes = raw.nbytes
            copies = max(1, int(np.ceil(256e6 / nbytes)))
            W = [torch.from_numpy(raw).cuda() for _ in range(min(copies, 512))]
            sw = C.c_int(0)
            native.check(L.tf_op_weight_scale(C.c_void_p(W[0].data_ptr()), t, N, K, C.byref(sw), C.c_void_p(st.cuda_stream)))
            for M in (1, 8, 64, 512):
                X = torch.randn(M, K, device="cuda")
                Y = torch.empty(M, N, device="cuda")
                tc = M >= 16

                def run(i):
                    wp = C.c_void_p(W[i % len(W)].data_ptr())
                    if tc:
                        native.check(L.tf_op_matmul_tc(C.c_void_p(Y.data_ptr()), C.c_void_p(X.data_ptr()), t, wp, N, K,
                                                       M, sw.value, C.c_void_p(st.cuda_stream)))
                    else:
                        native.check(L.tf_op_matmul(C.c_void_p(Y.data_ptr()), C.c_void_p(X.data_ptr()), t, wp, N, K, M,
                                                    C.c_void_p(st.cuda_stream)))
                for i in range(3):
                    run(i)
                reps = 10
                evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(reps)]
                for i, (a, b) in enumerate(evs):
                    a.record(st)
                    run(i + 3)
                    b.record(st)
                torch.cuda.synchronize()
                ms = statistics.median(a.elapsed_time(b) for a, b in evs)
                alg = nbytes + M * K * 4 + M * N * 4
                fl = 2.0 * M * N * K
                rows.append({"type": tname, "N": N, "K": K, "M": M, "path": "tensor-core GEMM" if tc else "GEMV",
                             "us": round(ms * 1e3, 2), "GB_s": round(alg / (ms / 1e3) / 1e9, 1),
                             "hbm_frac": round(alg / (ms / 1e3) / 1e9 / peak, 3),
                             "TFLOP_s": round(fl / (ms / 1e3) / 1e12, 2)})
                if not quiet:
                    print(json.dumps(rows[-1]), flush=True)
            del W
            torch.cuda.empty_cache()
    return rows


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=64)
    ap.add_argument("--warmup", type=int, default=8)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu", action="store_true", help="skip the cpu_baseline sample")
    ap.add_argument("--no-batched", action="store_true", help="skip the cfg4 batched-decode measurement")
    ap.add_argument("--no-configs", action="store_true", help="skip the cfg1 / cfg2 batch-1 runs (N = 1 only)")
    ap.add_argument("--batched-steps", type=int, default=128, help="timed cfg4 batched decode steps")
    ap.add_argument("--rows", type=int, default=None,
                    help="--kernel bstep: rows of the batched step (128); --kernel gemm: activation rows (256)")
    ap.add_argument("--ctx", type=int, default=512, help="--kernel bstep: prompt length before the step")
    ap.add_argument("--trace-k", dest="trace_k", type=int, default=0, help="--kernel gemmtrace: K of the traced GEMM (1536)")
    ap.add_argument("--kernel", default="", choices=["", "lmhead", "step", "step0", "pktrace", "gvtrace", "sweep", "bstep", "gemm", "gemmtrace", "configs", "q6k"],
                    help="profiling cases: 'lmhead' = only the dequant-GEMV on the lm_head shape (1 warm-up + "
                         "3 launches); 'step' = the cfg0 layer shapes on a 2-layer model, 4-token prefill + 2 "
                         "eager decode steps")
    args = ap.parse_args()
    if args.kernel == "lmhead":
        import torch
        from tinferno_b200 import native
        print(json.dumps(gemv_roofline(torch, native, None, reps=3, warm=1)))
        return
    if args.kernel == "sweep":
        matmul_sweep()
        return
    if args.kernel == "q6k":
        print(json.dumps(q6k_gemv()))
        return
    if args.kernel == "step":
        from tinferno_b200.model import Model, RunConfig
        cfg = synth.mini(CFG, 2, 4096)
        m = Model(synth.model_path(cfg), RunConfig(max_seq=CFG.max_seq, use_graph=False))
        t = int(np.argmax(m.prefill(synth.prompt_tokens(cfg, 4))))
        for _ in range(2):
            t = int(np.argmax(m.decode(t)))
        m.close()
        print(json.dumps({"kernel": "step", "kernels_per_step": 2 * 4 + 1, "last_token": t}))
        return
    if args.kernel == "pktrace":
        # per-phase breakdown of one cfg0 decode step on the persistent kernel (phase trace of
        # the first CTA: the time between consecutive trace points, averaged over the layers)
        from tinferno_b200 import native
        from tinferno_b200.model import Model, RunConfig
        os.environ["TFB200_PK_TRACE"] = "1"
        m = Model(model_file(), RunConfig(max_seq=CFG.max_seq, decode_mode=native.TF_DECODE_PERSISTENT))
        t = int(np.argmax(m.prefill(synth.prompt_tokens(CFG, PROMPT))))
        for _ in range(6):
            t = m.decode_argmax(t)
        cap = 8192
        buf = np.zeros(2 * cap, np.uint64)
        n = np.zeros(2, np.int32)
        t = m.decode_argmax(t)
        native.check(m.L.tf_cuda_trace_read(m.h, buf.ctypes.data_as(C.POINTER(C.c_ulonglong)), cap,
                                            n.ctypes.data_as(native.i32p)), m.h)
        m.close()
        names = {0: "qkv", 1: "wo", 2: "gate/up", 3: "down", 5: "lm_head"}
        stage = {10: "start", 20: "read", 30: "prologue", 40: "rows", 50: "attn_start", 53: "attn_qkv_read",
                 51: "attn_done"}
        out = {}
        for w, who in ((0, "cta0 (attention + GEMV rows)"), (1, "last cta (GEMV rows only)")):
            ev = buf[w * cap:w * cap + n[w]]
            ts = (ev >> np.uint64(8)).astype(np.int64)
            tags = (ev & np.uint64(255)).astype(np.int64)
            def lab(g):
                g = int(g)
                return f"{stage.get(g - g % 10, '?')}/{names.get(g % 10, '?')}" if g < 50 else stage.get(g, "?")
            seg = {}
            for t0, g0, t1, g1 in zip(ts, tags, ts[1:], tags[1:]):
                seg.setdefault(f"{lab(g0)} -> {lab(g1)}", []).append((t1 - t0) / 1e3)
            out[who] = {"step_us": round((ts[-1] - ts[0]) / 1e3, 1),
                        "segments_us": {k: {"n": len(v), "mean": round(float(np.mean(v)), 3), "sum": round(float(np.sum(v)), 1)}
                                        for k, v in sorted(seg.items(), key=lambda kv: -sum(kv[1]))}}
        print(json.dumps(out, indent=1))
        return
    if args.kernel == "gvtrace":
        print(json.dumps(launch_trace(), indent=1))
        return
    if args.kernel == "step0":
        # one full-size cfg0 batch-1 decode step (the graph of the timed region) between
        # cudaProfilerStart / Stop, after a 32-token prefill and 3 decode steps, for a launch
        # list with DRAM bytes under `ncu --profile-from-start off`
        import torch
        from tinferno_b200.model import Model, RunConfig
        m = Model(model_file(), RunConfig(max_seq=CFG.max_seq))
        t = int(np.argmax(m.prefill(synth.prompt_tokens(CFG, PROMPT))))
        for _ in range(3):
            t = m.decode_argmax(t)
        torch.cuda.synchronize()
        torch.cuda.profiler.start()
        t = m.decode_argmax(t)
        torch.cuda.synchronize()
        torch.cuda.profiler.stop()
        kps = m.kernels_per_step
        m.close()
        print(json.dumps({"kernel": "step0", "kernels_per_step": kps, "last_token": t}))
        return
    if args.kernel == "gemm":
        # the cfg4 gate/up GEMM of a batched step (N = 2 x 8960, K = 1536; 256 rows unless --rows), Q8_0,
        # 1 warm-up + 3 launches through tf_op_matmul_tc (for an ncu capture of launch 2)
        import torch
        from tinferno_b200 import gguf, native, quants
        L = native.lib()
        N, K, M = 17920, 1536, args.rows or 256
        rng = np.random.default_rng(7)
        raw = np.ascontiguousarray(quants.quantize((rng.standard_normal((N, K)) * 0.02).astype(np.float32),
                                                   gguf.GGML_Q8_0)).reshape(-1)
        W = torch.from_numpy(raw).cuda()
        X = torch.randn(M, K, device="cuda")
        Y = torch.empty(M, N, device="cuda")
        st = torch.cuda.current_stream()
        sw = C.c_int(0)
        native.check(L.tf_op_weight_scale(C.c_void_p(W.data_ptr()), gguf.GGML_Q8_0, N, K, C.byref(sw),
                                          C.c_void_p(st.cuda_stream)))
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(2)]
        for i in range(4):
            if i == 3:
                ev[0].record(st)
            native.check(L.tf_op_matmul_tc(C.c_void_p(Y.data_ptr()), C.c_void_p(X.data_ptr()), gguf.GGML_Q8_0,
                                           C.c_void_p(W.data_ptr()), N, K, M, sw.value, C.c_void_p(st.cuda_stream)))
        ev[1].record(st)
        torch.cuda.synchronize()
        us = ev[0].elapsed_time(ev[1]) * 1e3
        print(json.dumps({"kernel": "gemm", "N": N, "K": K, "M": M, "us_incl_prep": round(us, 2),
                          "TFLOP_s": round(2 * N * K * M / us / 1e6, 1)}))
        return
    if args.kernel == "gemmtrace":
        # the --kernel gemm launch with the pipeline trace of its first CTA (tf_op_gemm_trace):
        # per k stage, in SM cycles from the kernel's entry, when dequantising warp 0 passed its
        # chunk and buffer waits and arrived, when warp 15 arrived, when the MMA thread passed its
        # waits and committed, and when the copy warp issued the chunk and activation copies
        import torch
        from tinferno_b200 import gguf, native, quants
        L = native.lib()
        N, K, M = 17920, args.trace_k or 1536, args.rows or 32
        rng = np.random.default_rng(7)
        raw = np.ascontiguousarray(quants.quantize((rng.standard_normal((N, K)) * 0.02).astype(np.float32),
                                                   gguf.GGML_Q8_0)).reshape(-1)
        W = torch.from_numpy(raw).cuda()
        X = torch.randn(M, K, device="cuda")
        Y = torch.empty(M, N, device="cuda")
        st = torch.cuda.current_stream()
        sw = C.c_int(0)
        native.check(L.tf_op_weight_scale(C.c_void_p(W.data_ptr()), gguf.GGML_Q8_0, N, K, C.byref(sw),
                                          C.c_void_p(st.cuda_stream)))
        tr = torch.zeros(968, dtype=torch.int64, device="cuda")
        for i in range(4):
            if i == 3:
                torch.cuda.synchronize()
                native.check(L.tf_op_gemm_trace(C.c_void_p(tr.data_ptr())))
            native.check(L.tf_op_matmul_tc(C.c_void_p(Y.data_ptr()), C.c_void_p(X.data_ptr()), gguf.GGML_Q8_0,
                                           C.c_void_p(W.data_ptr()), N, K, M, sw.value, C.c_void_p(st.cuda_stream)))
        torch.cuda.synchronize()
        native.check(L.tf_op_gemm_trace(None))
        t = tr.cpu().numpy().astype(np.int64)
        t0 = int(t[0])
        rel = lambda v: int(v) - t0 if v else None
        nk = K // 64
        stages = []
        for k in range(min(nk, 128)):
            last = int(t[75 + 4 * k])
            stages.append({"k": k, "dq0_chunk": rel(t[72 + 4 * k]), "dq0_buf": rel(t[73 + 4 * k]),
                           "dq0_arr": rel(t[74 + 4 * k]), "dq_last_arr": rel(last >> 5), "dq_last_warp": last & 31,
                           "mma_go": rel(t[584 + 2 * k]), "mma_cmt": rel(t[585 + 2 * k]),
                           "x_iss": rel(t[840 + k])})
        print(json.dumps({"kernel": "gemmtrace", "N": N, "K": K, "M": M, "setup": rel(t[1]), "copy_wait_done": rel(t[2]),
                          "mma_all_done": rel(t[3]), "epilogue_done": rel(t[4]),
                          "chunks_issued": [rel(v) for v in t[8:8 + nk // 4]], "stages": stages}))
        return
    if args.kernel == "configs":
        for line in config_runs():
            print(json.dumps(line), flush=True)
        return
    if args.kernel == "bstep":
        # one cfg4 batched decode step (--rows rows at context --ctx) between cudaProfilerStart /
        # Stop, for a launch list under `ncu --profile-from-start off`
        import torch
        from tinferno_b200.model import Model, RunConfig
        S, P = args.rows or 128, args.ctx
        m = Model(synth.model_path(synth.CFG4), RunConfig(max_seq=P + 16, max_batch=S))
        prompts = np.stack([synth.prompt_tokens(synth.CFG4, P, stream=1000 + g) for g in range(S)])
        tok = m.prefill_batch(list(range(S)), prompts)
        tok = m.decode_batch(list(range(S)), tok.tolist())
        torch.cuda.synchronize()
        torch.cuda.profiler.start()
        tok = m.decode_batch(list(range(S)), tok.tolist())
        torch.cuda.synchronize()
        torch.cuda.profiler.stop()
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(2)]
        st = torch.cuda.ExternalStream(m.stream)
        ev[0].record(st)
        for _ in range(5):
            tok = m.decode_batch(list(range(S)), tok.tolist())
        ev[1].record(st)
        torch.cuda.synchronize()
        m.close()
        print(json.dumps({"kernel": "bstep", "rows": S, "context": P + 2, "ms_per_step": round(ev[0].elapsed_time(ev[1]) / 5, 3),
                          "first_ids": [int(v) for v in tok[:4]]}))
        return
    if args.warmup < 3:
        args.warmup = 3
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        return run_reference(args, rank)
    dist = None
    if world > 1:
        import datetime
        import torch
        import torch.distributed as td
        torch.cuda.set_device(local_rank)
        td.init_process_group("nccl", timeout=datetime.timedelta(seconds=600))
        dist = td
    try:
        run_ours(args, rank, world, local_rank, dist)
    finally:
        if dist:
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
