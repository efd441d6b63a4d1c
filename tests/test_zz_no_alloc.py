"""tf_op_attn_decode_noalloc (static device scratch, no allocation) against the allocating
tf_op_attn_decode: identical results on consecutive calls of different shapes (the
arrival counters must come back to zero after each call), and the size limit is enforced.
Named to be collected last, so it also runs after every other GPU test in the session."""
import ctypes as C

import numpy as np
import pytest

from tinferno_b200 import native

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")


def _ptr(t):
    return C.c_void_p(t.data_ptr())


def _case(n_pos, H, KV, hd, kv_type, seed):
    cap = n_pos + 7
    g = torch.Generator().manual_seed(seed)
    tdt = {native.TF_KV_F32: torch.float32, native.TF_KV_F16: torch.float16,
           native.TF_KV_BF16: torch.bfloat16}[kv_type]
    q = torch.randn((H, hd), generator=g).cuda()
    kc = torch.randn((KV, cap, hd), generator=g).to(tdt).cuda()
    vc = torch.randn((KV, cap, hd), generator=g).to(tdt).cuda()
    return q, kc, vc, cap


def _run(fn, q, kc, vc, kv_type, cap, n_pos, H, KV, hd):
    out = torch.full((H, hd), float("nan"), device="cuda")
    native.check(fn(_ptr(out), _ptr(q), _ptr(kc), _ptr(vc), kv_type, cap, n_pos, H, KV, hd, None))
    torch.cuda.synchronize()
    return out.cpu().numpy()


SHAPES = [  # (n_pos, H, KV, hd, kv_type): split and unsplit, all cache types
    (1000, 32, 8, 64, native.TF_KV_F32),
    (300, 14, 2, 64, native.TF_KV_F16),
    (40, 12, 2, 128, native.TF_KV_BF16),
    (2049, 12, 2, 128, native.TF_KV_F32),
    # F32 caches with >= 16 kv heads and head_dim % 32 == 0 take the streaming kernel (its own
    # split count, partial layout and combine)
    (1000, 32, 16, 64, native.TF_KV_F32),
    (2049, 64, 16, 128, native.TF_KV_F32),
]


def test_noalloc_matches_allocating_entry_point():
    lib = native.lib()
    for rep in range(2):  # two calls in a row for every shape
        for i, (n_pos, H, KV, hd, kv) in enumerate(SHAPES):
            q, kc, vc, cap = _case(n_pos, H, KV, hd, kv, seed=10 * i + rep)
            want = _run(lib.tf_op_attn_decode, q, kc, vc, kv, cap, n_pos, H, KV, hd)
            got = _run(lib.tf_op_attn_decode_noalloc, q, kc, vc, kv, cap, n_pos, H, KV, hd)
            assert np.isfinite(got).all()
            # same kernel, same split: bit-identical
            np.testing.assert_array_equal(got, want)
    code = C.c_int(-1)
    native.check(lib.tf_op_device_error(None, C.byref(code)))
    assert code.value == 0  # no device-side problem was recorded


def test_noalloc_rejects_bad_head_dim():
    lib = native.lib()
    q, kc, vc, cap = _case(10, 4, 2, 64, native.TF_KV_F32, seed=5)
    out = torch.zeros((4, 64), device="cuda")
    for hd in (0, -2, 12):
        with pytest.raises(native.TFError, match="head_dim"):
            native.check(lib.tf_op_attn_decode_noalloc(_ptr(out), _ptr(q), _ptr(kc), _ptr(vc), native.TF_KV_F32, cap,
                                                       10, 4, 2, hd, None))


def test_noalloc_rejects_oversized_scratch():
    lib = native.lib()
    n_pos, H, KV, hd = 8192, 32, 8, 128  # 32 * 128 * 130 floats > 524288
    q, kc, vc, cap = _case(n_pos, H, KV, hd, native.TF_KV_F32, seed=3)
    out = torch.zeros((H, hd), device="cuda")
    with pytest.raises(native.TFError, match="static limit"):
        native.check(lib.tf_op_attn_decode_noalloc(_ptr(out), _ptr(q), _ptr(kc), _ptr(vc), native.TF_KV_F32, cap,
                                                   n_pos, H, KV, hd, None))
    # a valid call still works afterwards
    q, kc, vc, cap = _case(500, H, KV, hd, native.TF_KV_F32, seed=4)
    want = _run(lib.tf_op_attn_decode, q, kc, vc, native.TF_KV_F32, cap, 500, H, KV, hd)
    got = _run(lib.tf_op_attn_decode_noalloc, q, kc, vc, native.TF_KV_F32, cap, 500, H, KV, hd)
    np.testing.assert_array_equal(got, want)
