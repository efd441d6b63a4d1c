"""Test infrastructure (the checker), not product.

ctypes bindings for
  * ``oracle/_build/libtf_oracle.so`` - the plain-C restatement (tf_oracle.c), and
  * ``oracle/_ref/libtinferno_ref.so`` - the reference engine compiled from its own sources
    plus ref_shim.cpp (present only where the reference was available at build time;
    the built file travels with the tree).
Only tests/, __graft_entry__.smoke() and bench.py (cpu_baseline / --impl reference) use
this module.  ``build_oracle()`` compiles the restatement with gcc if it is missing.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess
from typing import Dict, Optional

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ORACLE_SO = os.path.join(HERE, "_build", "libtf_oracle.so")
REF_SO = os.path.join(HERE, "_ref", "libtinferno_ref.so")

f32p = C.POINTER(C.c_float)
i32p = C.POINTER(C.c_int)


def _fp(a: np.ndarray):
    return a.ctypes.data_as(f32p)


def _ip(a: np.ndarray):
    return a.ctypes.data_as(i32p)


def build_oracle(force: bool = False) -> str:
    src = os.path.join(HERE, "tf_oracle.c")
    if force or not os.path.exists(ORACLE_SO) or os.path.getmtime(ORACLE_SO) < os.path.getmtime(src):
        subprocess.check_call(["make", "-s", "-C", HERE, "oracle"])
    return ORACLE_SO


class TensorDesc(C.Structure):
    """Same field order as tf_tensor_desc in include/tinferno_b200.h."""
    _fields_ = [("name", C.c_char_p), ("ggml_type", C.c_int), ("ndim", C.c_int),
                ("ne", C.c_int64 * 4), ("data", C.c_void_p), ("nbytes", C.c_size_t)]


class HParams(C.Structure):
    _fields_ = [("n_vocab", C.c_int), ("n_embd", C.c_int), ("n_ff", C.c_int), ("n_layer", C.c_int),
                ("n_head", C.c_int), ("n_kv_head", C.c_int), ("head_dim", C.c_int),
                ("rms_eps", C.c_float), ("rope_llama3", C.c_int), ("rope_theta", C.c_float),
                ("rope_scale", C.c_float), ("rope_low_freq_f", C.c_float),
                ("rope_high_freq_f", C.c_float), ("rope_orig_ctx", C.c_float),
                ("bos", C.c_int), ("eos", C.c_int)]


_oracle = None
_ref = None


def oracle_lib():
    global _oracle
    if _oracle is None:
        lib = C.CDLL(build_oracle())
        lib.tfo_f16_to_f32.restype = C.c_float
        lib.tfo_f16_to_f32.argtypes = [C.c_uint16]
        lib.tfo_f32_to_f16.restype = C.c_uint16
        lib.tfo_f32_to_f16.argtypes = [C.c_float]
        lib.tfo_matmul.argtypes = [f32p, f32p, C.c_int, C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_int]
        lib.tfo_dequant_row.argtypes = [f32p, C.c_int, C.c_void_p, C.c_int, C.c_int64]
        lib.tfo_rmsnorm.argtypes = [f32p, f32p, f32p, C.c_int, C.c_float]
        lib.tfo_silu_mul.argtypes = [f32p, f32p, C.c_int]
        lib.tfo_softmax.argtypes = [f32p, C.c_int]
        lib.tfo_rope_freqs.argtypes = [f32p, C.c_int, C.c_float, C.c_int, C.c_float, C.c_float,
                                       C.c_float, C.c_float]
        lib.tfo_rope.argtypes = [f32p, C.c_int, C.c_int, C.c_int, C.c_int, f32p]
        lib.tfo_attn_decode.argtypes = [f32p, f32p, f32p, f32p, C.c_int, C.c_int, C.c_int, C.c_int]
        lib.tfo_attn_prefill.argtypes = [f32p, f32p, f32p, f32p, C.c_int, C.c_int, C.c_int, C.c_int]
        lib.tfo_sample_greedy.argtypes = [f32p, C.c_int]
        lib.tfo_sample_logits.argtypes = [f32p, C.c_int, C.c_float, C.c_float, C.c_float]
        lib.tfo_model_create.restype = C.c_void_p
        lib.tfo_model_create.argtypes = [C.POINTER(TensorDesc), C.c_int, C.POINTER(HParams), C.c_int,
                                         C.c_int]
        lib.tfo_model_prefill.argtypes = [C.c_void_p, i32p, C.c_int, f32p]
        lib.tfo_model_decode.argtypes = [C.c_void_p, C.c_int, f32p]
        lib.tfo_model_reset.argtypes = [C.c_void_p]
        lib.tfo_model_n_pos.argtypes = [C.c_void_p]
        lib.tfo_model_destroy.argtypes = [C.c_void_p]
        lib.tfo_last_error.restype = C.c_char_p
        _oracle = lib
    return _oracle


def ref_available() -> bool:
    return os.path.exists(REF_SO)


def ref_lib():
    global _ref
    if _ref is None:
        if not ref_available():
            raise FileNotFoundError(REF_SO)
        lib = C.CDLL(REF_SO)
        lib.ref_last_error.restype = C.c_char_p
        lib.ref_model_create.restype = C.c_void_p
        lib.ref_model_create.argtypes = [C.c_char_p, C.c_char_p, C.c_int, C.c_int, C.c_int]
        lib.ref_model_destroy.argtypes = [C.c_void_p]
        lib.ref_model_prefill.argtypes = [C.c_void_p, i32p, C.c_int, f32p]
        lib.ref_model_decode.argtypes = [C.c_void_p, C.c_int, f32p]
        lib.ref_model_reset.argtypes = [C.c_void_p]
        for f in ("ref_model_n_vocab", "ref_model_n_pos", "ref_model_eos", "ref_model_n_threads"):
            getattr(lib, f).argtypes = [C.c_void_p]
        lib.ref_model_weight_bytes.restype = C.c_ulonglong
        lib.ref_model_weight_bytes.argtypes = [C.c_void_p]
        lib.ref_matmul.argtypes = [f32p, f32p, C.c_int, C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_int,
                                   C.c_int, C.c_int]
        lib.ref_dequant_row.argtypes = [f32p, C.c_int, C.c_void_p, C.c_int, C.c_longlong]
        lib.ref_quant_q8_0_row.argtypes = [C.c_void_p, f32p, C.c_int]
        lib.ref_quant_q4_0_row.argtypes = [C.c_void_p, f32p, C.c_int]
        lib.ref_f16_to_f32.restype = C.c_float
        lib.ref_f16_to_f32.argtypes = [C.c_uint16]
        lib.ref_f32_to_f16.restype = C.c_uint16
        lib.ref_f32_to_f16.argtypes = [C.c_float]
        lib.ref_rmsnorm.argtypes = [f32p, f32p, f32p, C.c_int, C.c_float]
        lib.ref_silu_mul.argtypes = [f32p, f32p, C.c_int]
        lib.ref_softmax.argtypes = [f32p, C.c_int]
        lib.ref_rope_freqs.argtypes = [f32p, C.c_int, C.c_float, C.c_int, C.c_float, C.c_float,
                                       C.c_float, C.c_float]
        lib.ref_apply_rope_many.argtypes = [f32p, C.c_int, C.c_int, C.c_int, C.c_int, f32p]
        lib.ref_attn_prefill.argtypes = [f32p, f32p, f32p, f32p, C.c_int, C.c_int, C.c_int, C.c_int]
        lib.ref_attn_decode.argtypes = [f32p, f32p, f32p, f32p, C.c_int, C.c_int, C.c_int, C.c_int,
                                        C.c_int]
        lib.ref_sample_greedy.argtypes = [f32p, C.c_int]
        lib.ref_sample_logits_steps.argtypes = [f32p, C.c_int, C.c_int, C.c_float, C.c_float, C.c_int,
                                                i32p]
        _ref = lib
    return _ref


def hparams_from_gguf(g) -> HParams:
    """Hyper-parameters exactly as the reference derives them (src/model.cpp:14-41)."""
    a = g.arch
    key = lambda f: f"{a}.{f}"
    n_embd = g.u64(key("embedding_length"))
    n_head = g.u64(key("attention.head_count"))
    tok = g.tensors["token_embd.weight"]
    n_vocab = g.u64(key("vocab_size"), 0) or tok.rows
    hp = HParams()
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


def tensor_descs(g):
    """A TensorDesc array over the reader's memory map (keeps names alive on the array)."""
    names = list(g.order)
    arr = (TensorDesc * len(names))()
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
    arr._keep = keep
    return arr


class OracleModel:
    """The restated token loop over a GGUF opened with gguf.GGUFReader."""

    def __init__(self, g, max_seq: int, threads: int = 0):
        self.lib = oracle_lib()
        self.g = g
        self.hp = hparams_from_gguf(g)
        self.descs = tensor_descs(g)
        threads = threads or (os.cpu_count() or 1)
        self.h = self.lib.tfo_model_create(self.descs, len(self.descs), C.byref(self.hp), max_seq, threads)
        if not self.h:
            raise RuntimeError(self.lib.tfo_last_error().decode())
        self.n_vocab = self.hp.n_vocab

    def prefill(self, tokens) -> np.ndarray:
        toks = np.ascontiguousarray(tokens, dtype=np.int32)
        out = np.empty(self.n_vocab, np.float32)
        if self.lib.tfo_model_prefill(self.h, _ip(toks), len(toks), _fp(out)):
            raise RuntimeError(self.lib.tfo_last_error().decode())
        return out

    def decode(self, token: int) -> np.ndarray:
        out = np.empty(self.n_vocab, np.float32)
        if self.lib.tfo_model_decode(self.h, int(token), _fp(out)):
            raise RuntimeError(self.lib.tfo_last_error().decode())
        return out

    def reset(self):
        self.lib.tfo_model_reset(self.h)

    def close(self):
        if self.h:
            self.lib.tfo_model_destroy(self.h)
            self.h = None

    __del__ = close


class RefModel:
    """The reference engine's Model through ref_shim.cpp."""

    def __init__(self, path: str, max_seq: int, stage: str = "v2", threads: int = 0):
        self.lib = ref_lib()
        self.h = self.lib.ref_model_create(path.encode(), stage.encode(), threads, max_seq, -1)
        if not self.h:
            raise RuntimeError(self.lib.ref_last_error().decode())
        self.n_vocab = self.lib.ref_model_n_vocab(self.h)
        self.n_threads = self.lib.ref_model_n_threads(self.h)

    def prefill(self, tokens, logits: Optional[np.ndarray] = None) -> np.ndarray:
        toks = np.ascontiguousarray(tokens, dtype=np.int32)
        out = logits if logits is not None else np.empty(self.n_vocab, np.float32)
        if self.lib.ref_model_prefill(self.h, _ip(toks), len(toks), _fp(out)):
            raise RuntimeError(self.lib.ref_last_error().decode())
        return out

    def decode(self, token: int, logits: Optional[np.ndarray] = None) -> np.ndarray:
        out = logits if logits is not None else np.empty(self.n_vocab, np.float32)
        if self.lib.ref_model_decode(self.h, int(token), _fp(out)):
            raise RuntimeError(self.lib.ref_last_error().decode())
        return out

    def reset(self):
        self.lib.ref_model_reset(self.h)

    def close(self):
        if self.h:
            self.lib.ref_model_destroy(self.h)
            self.h = None

    __del__ = close


def greedy_stream(model, prompt, n_predict: int, keep_logits: bool = False):
    """Prefill then n_predict x (argmax, decode), the loop of the reference's own
    correctness test (tests/test_correctness.cpp:87-99).  Returns (ids, logits_per_step)
    where logits_per_step[i] is the distribution ids[i] was drawn from."""
    lib = oracle_lib()
    logits = model.prefill(prompt)
    ids, steps = [], []
    for i in range(n_predict):
        if keep_logits:
            steps.append(logits.copy())
        t = int(lib.tfo_sample_greedy(_fp(logits), len(logits)))
        ids.append(t)
        logits = model.decode(t)
    return ids, steps
