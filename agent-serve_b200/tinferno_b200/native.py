"""ctypes binding of libtinferno_b200.so (the C-ABI in include/tinferno_b200.h).

There is no fallback: if the library is missing, ``lib()`` raises.  ``build()`` compiles it
in-tree with nvcc for sm_100a (``make -C agent-serve_b200``).
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

PKG_ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))  # agent-serve_b200/
REPO_ROOT = os.path.dirname(PKG_ROOT)
LIB_PATH = os.path.join(PKG_ROOT, "lib", "libtinferno_b200.so")
HEADER = os.path.join(REPO_ROOT, "include", "tinferno_b200.h")

f32p = C.POINTER(C.c_float)
i32p = C.POINTER(C.c_int)

TF_F32, TF_F16, TF_Q4_0, TF_Q4_1, TF_Q8_0, TF_Q6_K = 0, 1, 2, 3, 8, 14
TF_KV_F32, TF_KV_F16, TF_KV_BF16 = 0, 1, 2
TF_DECODE_KERNELS, TF_DECODE_PERSISTENT = 0, 1
(TF_DEV_ERR_NONE, TF_DEV_ERR_WAIT_FULL, TF_DEV_ERR_WAIT_EMPTY, TF_DEV_ERR_BAD_INDEX, TF_DEV_ERR_POS,
 TF_DEV_ERR_GRID_SYNC) = range(6)


class TensorDesc(C.Structure):
    _fields_ = [("name", C.c_char_p), ("ggml_type", C.c_int), ("ndim", C.c_int),
                ("ne", C.c_int64 * 4), ("data", C.c_void_p), ("nbytes", C.c_size_t)]


class HParams(C.Structure):
    _fields_ = [("n_vocab", C.c_int), ("n_embd", C.c_int), ("n_ff", C.c_int), ("n_layer", C.c_int),
                ("n_head", C.c_int), ("n_kv_head", C.c_int), ("head_dim", C.c_int),
                ("rms_eps", C.c_float), ("rope_llama3", C.c_int), ("rope_theta", C.c_float),
                ("rope_scale", C.c_float), ("rope_low_freq_f", C.c_float),
                ("rope_high_freq_f", C.c_float), ("rope_orig_ctx", C.c_float),
                ("bos", C.c_int), ("eos", C.c_int)]


class Options(C.Structure):
    _fields_ = [("max_seq", C.c_int), ("max_batch", C.c_int), ("device", C.c_int),
                ("kv_type", C.c_int), ("use_graph", C.c_int), ("decode_mode", C.c_int)]


# (name, restype, argtypes) of every entry point declared in include/tinferno_b200.h
_V = C.c_void_p
SIGNATURES = [
    ("tf_cuda_create", C.c_int, [C.POINTER(TensorDesc), C.c_int, C.POINTER(HParams), C.POINTER(Options),
                                 C.POINTER(C.c_void_p)]),
    ("tf_cuda_destroy", C.c_int, [_V]),
    ("tf_cuda_prefill", C.c_int, [_V, C.c_int, i32p, C.c_int, f32p, i32p]),
    ("tf_cuda_decode", C.c_int, [_V, C.c_int, C.c_int, f32p, i32p]),
    ("tf_cuda_generate_greedy", C.c_int, [_V, C.c_int, C.c_int, C.c_int, C.c_int, i32p, i32p]),
    ("tf_cuda_decode_batch", C.c_int, [_V, i32p, i32p, C.c_int, i32p, f32p]),
    ("tf_cuda_prefill_batch", C.c_int, [_V, i32p, i32p, C.c_int, C.c_int, i32p]),
    ("tf_cuda_sample", C.c_int, [_V, C.c_int, C.c_float, C.c_float, C.c_float, i32p]),
    ("tf_cuda_set_vocab_shard", C.c_int, [_V, C.c_int, C.c_int]),
    ("tf_cuda_shard_key", C.c_void_p, [_V]),
    ("tf_cuda_decode_shard", C.c_int, [_V, C.c_int, C.c_int]),
    ("tf_cuda_shard_token", C.c_int, [_V, C.c_int, i32p]),
    ("tf_cuda_history", C.c_int, [_V, C.c_int, i32p]),
    ("tf_cuda_trace_read", C.c_int, [_V, C.POINTER(C.c_ulonglong), C.c_int, i32p]),
    ("tf_cuda_launch_trace", C.c_int, [_V, C.POINTER(C.c_ulonglong), C.c_int, i32p, i32p]),
    ("tf_cuda_reset", C.c_int, [_V, C.c_int]),
    ("tf_cuda_n_pos", C.c_int, [_V, C.c_int]),
    ("tf_cuda_n_vocab", C.c_int, [_V]),
    ("tf_cuda_weight_bytes", C.c_ulonglong, [_V]),
    ("tf_cuda_stream", C.c_void_p, [_V]),
    ("tf_cuda_kernels_per_step", C.c_int, [_V]),
    ("tf_cuda_last_error", C.c_char_p, [_V]),
    ("tf_host_alloc", C.c_int, [C.c_size_t, C.POINTER(C.c_void_p)]),
    ("tf_host_free", C.c_int, [_V]),
    ("tf_op_matmul", C.c_int, [_V, _V, C.c_int, _V, C.c_int, C.c_int, C.c_int, _V]),
    ("tf_op_dequant_rows", C.c_int, [_V, C.c_int, _V, C.c_int, C.c_int, _V, C.c_int, _V]),
    ("tf_op_gemm_trace", C.c_int, [_V]),
    ("tf_op_device_error", C.c_int, [_V, i32p]),
    ("tf_op_rmsnorm", C.c_int, [_V, _V, _V, C.c_int, C.c_int, C.c_float, _V]),
    ("tf_op_silu_mul", C.c_int, [_V, _V, C.c_int, _V]),
    ("tf_op_softmax", C.c_int, [_V, C.c_int, C.c_int, _V]),
    ("tf_op_rope", C.c_int, [_V, C.c_int, C.c_int, C.c_int, C.c_int, _V, _V]),
    ("tf_op_attn_decode", C.c_int, [_V, _V, _V, _V, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, _V]),
    ("tf_op_q8_scale", C.c_int, [_V, C.c_int, C.c_int, i32p, _V]),
    ("tf_op_matmul_q8_tc", C.c_int, [_V, _V, _V, C.c_int, C.c_int, C.c_int, C.c_int, _V]),
    ("tf_op_weight_scale", C.c_int, [_V, C.c_int, C.c_int, C.c_int, i32p, _V]),
    ("tf_op_matmul_tc", C.c_int, [_V, _V, C.c_int, _V, C.c_int, C.c_int, C.c_int, C.c_int, _V]),
    ("tf_op_attn_decode_noalloc", C.c_int, [_V, _V, _V, _V, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, C.c_int, _V]),
    ("tf_op_attn_prefill", C.c_int, [_V, _V, _V, _V, C.c_int, C.c_int, C.c_int, C.c_int, _V]),
    ("tf_op_argmax", C.c_int, [_V, C.c_int, C.c_int, _V, _V]),
]

_lib = None


def build(force: bool = False) -> str:
    cmd = ["make", "-s", "-C", PKG_ROOT, "-j8"]
    if force:
        subprocess.check_call(["make", "-s", "-C", PKG_ROOT, "clean"])
    subprocess.check_call(cmd)
    return LIB_PATH


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(f"CUDA library not built: {LIB_PATH} (run make -C {PKG_ROOT})")
        L = C.CDLL(LIB_PATH)
        for name, res, args in SIGNATURES:
            f = getattr(L, name)
            f.restype = res
            f.argtypes = args
        _lib = L
    return _lib


class TFError(RuntimeError):
    pass


def check(rc: int, handle=None):
    if rc != 0:
        msg = lib().tf_cuda_last_error(handle)
        raise TFError(msg.decode() if msg else f"status {rc}")


class HostArray:
    """A page-locked host buffer (tf_host_alloc) viewed as a numpy array: logits written into
    it by the engine arrive by DMA with no staging copy.  Keep the object alive while the
    array is in use; close() (or garbage collection) frees it."""

    def __init__(self, n: int, dtype=None):
        import numpy as np
        dtype = np.dtype(dtype or np.float32)
        self._p = C.c_void_p()
        check(lib().tf_host_alloc(int(n) * dtype.itemsize, C.byref(self._p)))
        buf = (C.c_byte * (int(n) * dtype.itemsize)).from_address(self._p.value)
        self.array = np.frombuffer(buf, dtype=dtype, count=int(n))

    def close(self):
        if self._p:
            self.array = None
            lib().tf_host_free(self._p)
            self._p = C.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
