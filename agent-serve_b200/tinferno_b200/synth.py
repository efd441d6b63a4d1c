"""Seeded synthetic GGUF models with the BASELINE architectures (no checkpoints are
available offline, so weights are random with the stated distribution).

Every matmul weight and token_embd row is drawn N(0, 0.02) from a per-(tensor, row-chunk)
numpy SeedSequence derived from the config seed (42 unless stated, the reference's
default seed, src/common.hpp:111), then quantised to the config's type; norm weights are
fp32 ones; Q/K/V biases (qwen2) are F32 N(0, 0.02); embeddings are tied (no
output.weight).  Tensor names, metadata keys and tensor order follow what the reference
loader binds (src/model.cpp:14-65).  Because generation is chunked by fixed row counts,
the bytes do not depend on the number of worker threads.
"""
from __future__ import annotations

import hashlib
import os
from concurrent.futures import ThreadPoolExecutor
from dataclasses import dataclass, field, replace
from typing import Dict, List, Optional, Tuple

import numpy as np

from .gguf import (GGML_F32, GGML_Q4_0, GGML_Q4_1, GGML_Q6_K, GGML_Q8_0, TensorSpec,
                   row_nbytes, write_gguf)
from .quants import quantize

CHUNK_ELEMS = 1 << 22  # weights per generation chunk (fixed: determines the bytes)


@dataclass(frozen=True)
class ModelConfig:
    name: str
    arch: str                 # "llama" | "qwen2"
    n_vocab: int
    n_embd: int
    n_layer: int
    n_head: int
    n_kv_head: int
    n_ff: int
    rope_theta: float
    rms_eps: float
    wtype: int = GGML_Q8_0     # attention / FFN matmul weights
    etype: int = GGML_Q8_0     # token_embd (= lm_head, tied)
    down_override: Tuple[Tuple[int, int], ...] = ()  # (layer, type) for ffn_down
    bias: bool = False
    rope_llama3: bool = False  # rope.scaling.type = "llama3" (Llama 3.x frequency smoothing)
    seed: int = 42
    n_prompt: int = 32
    n_decode: int = 64
    max_seq: int = 2048

    @property
    def head_dim(self) -> int:
        return self.n_embd // self.n_head

    def down_type(self, layer: int) -> int:
        for li, t in self.down_override:
            if li == layer:
                return t
        return self.wtype


# The BASELINE configurations (BASELINE.json "configs").
CFG0 = ModelConfig("cfg0-llama32-1b-q8_0", "llama", 128256, 2048, 16, 32, 8, 8192, 500000.0, 1e-5,
                   n_prompt=32, n_decode=64, max_seq=2048)
CFG1 = ModelConfig("cfg1-qwen25-0.5b-q8_0-bias", "qwen2", 151936, 896, 24, 14, 2, 4864, 1e6, 1e-6,
                   bias=True, n_prompt=512, n_decode=128, max_seq=2048)
CFG2 = ModelConfig("cfg2-llama32-1b-q4_0-q6_k-q4_1", "llama", 128256, 2048, 16, 32, 8, 8192, 500000.0,
                   1e-5, wtype=GGML_Q4_0, etype=GGML_Q6_K,
                   down_override=((0, GGML_Q4_1), (15, GGML_Q4_1)), n_prompt=128, n_decode=128,
                   max_seq=2048)
CFG4 = ModelConfig("cfg4-qwen25-1.5b-q8_0-bias", "qwen2", 151936, 1536, 28, 12, 2, 8960, 1e6, 1e-6,
                   bias=True, n_prompt=1024, n_decode=128, max_seq=1152)

CONFIGS: Dict[str, ModelConfig] = {"cfg0": CFG0, "cfg1": CFG1, "cfg2": CFG2, "cfg4": CFG4}

# cfg0 with the llama3 RoPE frequency scaling of real Llama 3.2 files (src/attention.cpp:14-26);
# a parity case for that branch, not a benchmark configuration
CFG0_LLAMA3 = replace(CFG0, name="cfg0-llama3rope-q8_0", rope_llama3=True, n_prompt=40, n_decode=24)


def mini(cfg: ModelConfig, n_layer: int = 2, n_vocab: int = 4096, **kw) -> ModelConfig:
    """Same per-layer shapes and formats, fewer layers and a smaller vocabulary: the CPU
    oracle finishes these in seconds."""
    over = tuple((li, t) for li, t in cfg.down_override if li < n_layer)
    if cfg.down_override and not over:
        over = ((0, cfg.down_override[0][1]),)
    return replace(cfg, name=cfg.name + f"-mini{n_layer}", n_layer=n_layer, n_vocab=n_vocab,
                   down_override=over, **kw)


def tensor_plan(cfg: ModelConfig) -> List[Tuple[str, int, Tuple[int, ...], str]]:
    """(name, ggml type, ne, init) in file order; init in {"normal", "ones"}."""
    D, H, KV = cfg.n_embd, cfg.n_head * cfg.head_dim, cfg.n_kv_head * cfg.head_dim
    plan = [("token_embd.weight", cfg.etype, (D, cfg.n_vocab), "normal"),
            ("output_norm.weight", GGML_F32, (D,), "ones")]
    for i in range(cfg.n_layer):
        p = f"blk.{i}."
        plan += [(p + "attn_norm.weight", GGML_F32, (D,), "ones"),
                 (p + "attn_q.weight", cfg.wtype, (D, H), "normal"),
                 (p + "attn_k.weight", cfg.wtype, (D, KV), "normal"),
                 (p + "attn_v.weight", cfg.wtype, (D, KV), "normal")]
        if cfg.bias:
            plan += [(p + "attn_q.bias", GGML_F32, (H,), "normal"),
                     (p + "attn_k.bias", GGML_F32, (KV,), "normal"),
                     (p + "attn_v.bias", GGML_F32, (KV,), "normal")]
        plan += [(p + "attn_output.weight", cfg.wtype, (H, D), "normal"),
                 (p + "ffn_norm.weight", GGML_F32, (D,), "ones"),
                 (p + "ffn_gate.weight", cfg.wtype, (D, cfg.n_ff), "normal"),
                 (p + "ffn_up.weight", cfg.wtype, (D, cfg.n_ff), "normal"),
                 (p + "ffn_down.weight", cfg.down_type(i), (cfg.n_ff, D), "normal")]
    return plan


def metadata(cfg: ModelConfig):
    a = cfg.arch
    ms = {"general.architecture": a, "general.name": cfg.name}
    mu = {f"{a}.vocab_size": cfg.n_vocab, f"{a}.embedding_length": cfg.n_embd,
          f"{a}.feed_forward_length": cfg.n_ff, f"{a}.block_count": cfg.n_layer,
          f"{a}.attention.head_count": cfg.n_head, f"{a}.attention.head_count_kv": cfg.n_kv_head,
          f"{a}.rope.dimension_count": cfg.head_dim, f"{a}.context_length": cfg.max_seq}
    mf = {f"{a}.rope.freq_base": cfg.rope_theta, f"{a}.attention.layer_norm_rms_epsilon": cfg.rms_eps}
    if cfg.rope_llama3:
        # the keys src/model.cpp:28-37 reads, with Llama 3.2's published values
        ms[f"{a}.rope.scaling.type"] = "llama3"
        mf[f"{a}.rope.scaling.factor"] = 32.0
        mf[f"{a}.rope.scaling.low_freq_factor"] = 1.0
        mf[f"{a}.rope.scaling.high_freq_factor"] = 4.0
        mu[f"{a}.rope.scaling.original_context_length"] = 8192
    return ms, mu, mf


def _gen_chunk(seed: int, tidx: int, cidx: int, rows: int, k: int, ggml_type: int) -> bytes:
    rng = np.random.default_rng(np.random.SeedSequence([seed, tidx, cidx]))
    w = rng.standard_normal((rows, k), dtype=np.float32)
    w *= np.float32(0.02)
    return quantize(w, ggml_type).tobytes()


def _producer(cfg: ModelConfig, tidx: int, ggml_type: int, ne, init: str, pool: ThreadPoolExecutor):
    k = int(ne[0])
    rows = 1
    for d in ne[1:]:
        rows *= int(d)

    def produce():
        if init == "ones":
            yield np.ones(rows * k, dtype=np.float32).tobytes()
            return
        if ggml_type == GGML_F32 and rows == 1:  # biases
            rng = np.random.default_rng(np.random.SeedSequence([cfg.seed, tidx, 0]))
            yield (rng.standard_normal(k, dtype=np.float32) * np.float32(0.02)).tobytes()
            return
        rpc = max(1, CHUNK_ELEMS // k)
        starts = list(range(0, rows, rpc))
        futs = [pool.submit(_gen_chunk, cfg.seed, tidx, ci, min(rpc, rows - r0), k, ggml_type)
                for ci, r0 in enumerate(starts)]
        for f in futs:
            yield f.result()

    return produce


def weight_bytes(cfg: ModelConfig) -> int:
    total = 0
    for _, t, ne, _ in tensor_plan(cfg):
        rows = 1
        for d in ne[1:]:
            rows *= d
        total += rows * row_nbytes(t, ne[0])
    return total


def write_model(cfg: ModelConfig, path: str, threads: Optional[int] = None) -> str:
    ms, mu, mf = metadata(cfg)
    threads = threads or min(16, os.cpu_count() or 4)
    with ThreadPoolExecutor(threads) as pool:
        specs = [TensorSpec(name, t, ne, _producer(cfg, i, t, ne, init, pool))
                 for i, (name, t, ne, init) in enumerate(tensor_plan(cfg))]
        write_gguf(path, ms, mu, mf, specs)
    return path


def model_path(cfg: ModelConfig, cache_dir: Optional[str] = None) -> str:
    """Create (once) and return the GGUF for cfg under cache_dir (default $TFB200_CACHE or
    /tmp/tfb200_models)."""
    d = cache_dir or os.environ.get("TFB200_CACHE", "/tmp/tfb200_models")
    os.makedirs(d, exist_ok=True)
    p = os.path.join(d, f"{cfg.name}-s{cfg.seed}.gguf")
    if not os.path.exists(p):
        write_model(cfg, p)
    return p


def prompt_tokens(cfg: ModelConfig, n: Optional[int] = None, stream: int = 0) -> np.ndarray:
    """Seeded prompt ids uniform in [0, n_vocab); stream selects an independent sequence."""
    rng = np.random.default_rng(np.random.SeedSequence([cfg.seed, 0x70726F6D, stream]))
    return rng.integers(0, cfg.n_vocab, size=n or cfg.n_prompt, dtype=np.int64).astype(np.int32)


def file_digest(path: str) -> str:
    h = hashlib.sha256()
    with open(path, "rb") as f:
        while True:
            b = f.read(1 << 24)
            if not b:
                break
            h.update(b)
    return h.hexdigest()
