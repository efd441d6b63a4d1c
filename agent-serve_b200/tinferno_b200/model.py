"""Host-side mirror of the reference engine's ``Model`` API (src/model.hpp:24-90 of
RohanDisa/agent-serve) over the CUDA C-ABI.

    m = Model(path, RunConfig(max_seq=2048))
    logits = m.prefill(tokens)          # Model::prefill(tokens, n, logits)
    logits = m.decode(token)            # Model::decode(token, logits)
    m.reset()                           # Model::reset()

Hyper-parameters are read from the GGUF exactly as the reference reads them
(src/model.cpp:14-41); tensors are handed to the library by pointer and copied once into
HBM in their GGUF block layouts.  Failures raise ``TFError`` (the reference throws
std::runtime_error).  ``stage_preset("b200")`` is the GPU stage next to the reference's
v0..v5 (src/common.hpp:289-322).
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass
from typing import Optional, Sequence

import numpy as np

from . import native
from .gguf import GGUFReader


class Mt19937Uniform:
    """std::uniform_real_distribution<float>(0, 1) over std::mt19937(seed) as libstdc++ draws
    it: one 32-bit output x per value, r = float(x) * 2^-32 (rounded to float first), and a
    value that rounds to 1 becomes the float just below 1."""

    def __init__(self, seed: int):
        self.bg = np.random.MT19937()
        self.bg._legacy_seeding(seed)  # init_genrand(seed), std::mt19937's seeding

    def next(self) -> float:
        x = int(self.bg.random_raw())
        r = np.float32(np.float32(x) / np.float32(4294967296.0))
        if r >= np.float32(1.0):
            r = np.nextafter(np.float32(1.0), np.float32(0.0))
        return float(r)


@dataclass
class RunConfig:
    """RunConfig (src/common.hpp:103-116) fields that apply to the GPU stage."""
    stage: str = "b200"
    max_seq: int = 4096
    max_batch: int = 1
    device: int = 0
    kv_type: int = native.TF_KV_F32
    use_graph: bool = True
    decode_mode: int = native.TF_DECODE_KERNELS
    n_predict: int = 64
    temperature: float = 0.0
    top_p: float = 0.9
    seed: int = 42


def stage_preset(stage: str) -> RunConfig:
    if stage != "b200":
        raise ValueError(f"unknown stage {stage} (the CUDA engine is stage b200)")
    return RunConfig()


_KV_NAMES = {native.TF_KV_F32: "f32", native.TF_KV_F16: "f16", native.TF_KV_BF16: "bf16"}


def describe(arch: str, hp: native.HParams, weight_bytes: int, cfg: RunConfig) -> str:
    """Model::describe (src/model.cpp:91-105): one line of the model's shape and the run
    configuration, with the GPU stage's own settings in place of threads / SIMD / blocking."""
    mode = "persistent" if cfg.decode_mode == native.TF_DECODE_PERSISTENT else "kernels"
    return (f"arch={arch} layers={hp.n_layer} dim={hp.n_embd} heads={hp.n_head}/{hp.n_kv_head} "
            f"ff={hp.n_ff} vocab={hp.n_vocab} weights={weight_bytes / 1e6:g} MB stage={cfg.stage} "
            f"device={cfg.device} kv={_KV_NAMES.get(cfg.kv_type, cfg.kv_type)} max_seq={cfg.max_seq} "
            f"slots={cfg.max_batch} graph={'on' if cfg.use_graph else 'off'} decode={mode}")


def hparams_from_gguf(g: GGUFReader) -> native.HParams:
    a = g.arch
    key = lambda f: f"{a}.{f}"
    n_embd = g.u64(key("embedding_length"))
    n_head = g.u64(key("attention.head_count"))
    n_vocab = g.u64(key("vocab_size"), 0)
    if not n_vocab:
        toks = g.kv.get("tokenizer.ggml.tokens")
        n_vocab = len(toks) if isinstance(toks, list) else 0
    if not n_vocab:
        n_vocab = g.tensors["token_embd.weight"].rows
    hp = native.HParams()
    hp.n_vocab = n_vocab
    hp.n_embd = n_embd
    hp.n_ff = g.u64(key("feed_forward_length"))
    hp.n_layer = g.u64(key("block_count"))
    hp.n_head = n_head
    hp.n_kv_head = g.u64(key("attention.head_count_kv"), n_head)
    hp.head_dim = n_embd // n_head if n_head else 0
    hp.rms_eps = g.f32(key("attention.layer_norm_rms_epsilon"), 1e-5)
    hp.rope_theta = g.f32(key("rope.freq_base"), 10000.0)
    llama3 = g.str(key("rope.scaling.type"), "") == "llama3"
    hp.rope_llama3 = 1 if llama3 else 0
    hp.rope_scale = g.f32(key("rope.scaling.factor"), 32.0) if llama3 else 1.0
    hp.rope_low_freq_f = g.f32(key("rope.scaling.low_freq_factor"), 1.0) if llama3 else 1.0
    hp.rope_high_freq_f = g.f32(key("rope.scaling.high_freq_factor"), 4.0) if llama3 else 4.0
    hp.rope_orig_ctx = float(g.u64(key("rope.scaling.original_context_length"), 8192)) if llama3 else 8192.0
    hp.bos = g.u64("tokenizer.ggml.bos_token_id", 1)
    hp.eos = g.u64("tokenizer.ggml.eos_token_id", 2)
    return hp


def tensor_descs(g: GGUFReader):
    names = list(g.order)
    arr = (native.TensorDesc * len(names))()
    keep = []
    for i, n in enumerate(names):
        t = g.tensors[n]
        nb = n.encode()
        keep.append(nb)
        arr[i].name = nb
        arr[i].ggml_type = t.ggml_type
        arr[i].ndim = len(t.ne)
        for d in range(4):
            arr[i].ne[d] = int(t.ne[d]) if d < len(t.ne) else 1
        arr[i].data = t.data.ctypes.data
        arr[i].nbytes = t.nbytes
    return arr, keep


class Model:
    def __init__(self, path: str, cfg: Optional[RunConfig] = None):
        self.cfg = cfg or RunConfig()
        self.L = native.lib()
        self.gguf = GGUFReader(path)
        self.hp = hparams_from_gguf(self.gguf)
        descs, keep = tensor_descs(self.gguf)
        opt = native.Options(self.cfg.max_seq, self.cfg.max_batch, self.cfg.device, self.cfg.kv_type,
                             1 if self.cfg.use_graph else 0, self.cfg.decode_mode)
        h = C.c_void_p()
        native.check(self.L.tf_cuda_create(descs, len(descs), C.byref(self.hp), C.byref(opt), C.byref(h)))
        self.h = h
        del keep
        self.gguf.close()  # weights now live in HBM
        self.n_vocab = self.hp.n_vocab
        self.n_embd = self.hp.n_embd
        self.n_layer = self.hp.n_layer
        self.bos = self.hp.bos
        self.eos = self.hp.eos
        self.weight_bytes = int(self.L.tf_cuda_weight_bytes(self.h))
        self.kernels_per_step = int(self.L.tf_cuda_kernels_per_step(self.h))
        self.arch = self.gguf.str("general.architecture", "llama")

    def describe(self) -> str:
        return describe(self.arch, self.hp, self.weight_bytes, self.cfg)

    # ---- the reference API ----
    def prefill(self, tokens: Sequence[int], logits: Optional[np.ndarray] = None, seq: int = 0) -> np.ndarray:
        toks = np.ascontiguousarray(tokens, dtype=np.int32)
        out = logits if logits is not None else np.empty(self.n_vocab, np.float32)
        am = C.c_int(-1)
        native.check(self.L.tf_cuda_prefill(self.h, seq, toks.ctypes.data_as(native.i32p), len(toks),
                                            out.ctypes.data_as(native.f32p), C.byref(am)), self.h)
        self.last_argmax = am.value
        return out

    def decode(self, token: int, logits: Optional[np.ndarray] = None, seq: int = 0) -> np.ndarray:
        out = logits if logits is not None else np.empty(self.n_vocab, np.float32)
        am = C.c_int(-1)
        native.check(self.L.tf_cuda_decode(self.h, seq, int(token), out.ctypes.data_as(native.f32p), C.byref(am)),
                     self.h)
        self.last_argmax = am.value
        return out

    def decode_argmax(self, token: int, seq: int = 0) -> int:
        am = C.c_int(-1)
        native.check(self.L.tf_cuda_decode(self.h, seq, int(token), None, C.byref(am)), self.h)
        return am.value

    def reset(self, seq: int = -1):
        native.check(self.L.tf_cuda_reset(self.h, seq), self.h)

    def n_pos(self, seq: int = 0) -> int:
        return int(self.L.tf_cuda_n_pos(self.h, seq))

    # ---- engine extras ----
    def generate_greedy(self, first_token: int, n: int, eos: int = -1, seq: int = 0) -> list:
        out = np.zeros(max(1, n), np.int32)
        n_out = C.c_int(0)
        native.check(self.L.tf_cuda_generate_greedy(self.h, seq, int(first_token), int(n), int(eos),
                                                     out.ctypes.data_as(native.i32p), C.byref(n_out)), self.h)
        return out[:n_out.value].tolist()

    def decode_batch(self, seq_ids: Sequence[int], tokens: Sequence[int], want_logits: bool = False):
        s = np.ascontiguousarray(seq_ids, dtype=np.int32)
        t = np.ascontiguousarray(tokens, dtype=np.int32)
        am = np.zeros(len(t), np.int32)
        lg = np.empty((len(t), self.n_vocab), np.float32) if want_logits else None
        native.check(self.L.tf_cuda_decode_batch(self.h, s.ctypes.data_as(native.i32p), t.ctypes.data_as(native.i32p),
                                                 len(t), am.ctypes.data_as(native.i32p),
                                                 lg.ctypes.data_as(native.f32p) if lg is not None else None), self.h)
        return (am, lg) if want_logits else am

    def prefill_batch(self, seq_ids: Sequence[int], prompts) -> np.ndarray:
        """Prefill equal-length prompts of several sequences at once; returns each sequence's
        greedy next id."""
        s = np.ascontiguousarray(seq_ids, dtype=np.int32)
        t = np.ascontiguousarray(prompts, dtype=np.int32)
        if t.ndim != 2 or t.shape[0] != len(s):
            raise ValueError("prompts must be [len(seq_ids)][n]")
        am = np.zeros(len(s), np.int32)
        native.check(self.L.tf_cuda_prefill_batch(self.h, s.ctypes.data_as(native.i32p), t.ctypes.data_as(native.i32p),
                                                  len(s), t.shape[1], am.ctypes.data_as(native.i32p)), self.h)
        return am

    def sample(self, temperature: float, top_p: float, r: float, row: int = 0) -> int:
        """sample_logits (src/sampler.cpp:15-52) on the device over the last step's logits of
        `row`, with the caller's uniform draw r (see Mt19937Uniform)."""
        out = C.c_int(0)
        native.check(self.L.tf_cuda_sample(self.h, row, float(temperature), float(top_p), float(r), C.byref(out)),
                     self.h)
        return out.value

    def generate(self, prompt: Sequence[int], n: int, temperature: float, top_p: float, seed: int = 42,
                 eos: int = -1) -> list:
        """The CLI's generation loop (src/main.cpp:106-122): prefill, then sample / stop at eos
        (i > 0) / decode, with std::mt19937(seed) draws for temperature > 0."""
        rng = Mt19937Uniform(seed)
        self.prefill(prompt)
        out = []
        for i in range(n):
            t = self.sample(temperature, top_p, rng.next() if temperature > 0 else 0.0)
            if t == eos and i > 0:
                break
            out.append(t)
            self.decode(t)
        return out

    # ---- vocab-split lm_head (include/tinferno_b200.h, tf_cuda_set_vocab_shard) ----
    def set_vocab_shard(self, rank: int, world: int):
        native.check(self.L.tf_cuda_set_vocab_shard(self.h, int(rank), int(world)), self.h)

    @property
    def shard_key_ptr(self) -> int:
        """Device address of this GPU's order-flipped greedy key (one int64)."""
        return int(self.L.tf_cuda_shard_key(self.h) or 0)

    def decode_shard(self, token: int = -1, seq: int = 0):
        """One asynchronous step with the split lm_head; token < 0 continues from the reduced key."""
        native.check(self.L.tf_cuda_decode_shard(self.h, seq, int(token)), self.h)

    def shard_token(self, seq: int = 0) -> int:
        out = C.c_int(0)
        native.check(self.L.tf_cuda_shard_token(self.h, seq, C.byref(out)), self.h)
        return out.value

    def history(self, n: int) -> list:
        """The first n ids of the last device-side greedy run (tf_cuda_history)."""
        out = np.zeros(max(1, n), np.int32)
        native.check(self.L.tf_cuda_history(self.h, int(n), out.ctypes.data_as(native.i32p)), self.h)
        return out[:n].tolist()

    @property
    def stream(self) -> int:
        return int(self.L.tf_cuda_stream(self.h) or 0)

    def close(self):
        if getattr(self, "h", None):
            self.L.tf_cuda_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
