"""Op-level parity: every tf_op_* kernel against the oracle restatement of the reference op,
on the same seeded inputs, through the C-ABI (device buffers from torch)."""
import ctypes as C

import numpy as np
import pytest

import pyoracle as po
from tinferno_b200 import gguf, native, quants

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
fp = po._fp
TYPES = [gguf.GGML_F32, gguf.GGML_F16, gguf.GGML_Q4_0, gguf.GGML_Q4_1, gguf.GGML_Q8_0, gguf.GGML_Q6_K]


_alive = []


def dev(a: np.ndarray):
    """Device copy of `a`, kept alive for the module so that a pointer taken from a temporary
    is never recycled by the caching allocator before the kernel reads it."""
    t = torch.from_numpy(np.ascontiguousarray(a)).cuda()
    _alive.append(t)
    if len(_alive) > 64:
        torch.cuda.synchronize()
        del _alive[:32]
    return t


def ptr(t):
    return C.c_void_p(t.data_ptr())


def call(rc):
    native.check(rc)
    torch.cuda.synchronize()


# Tolerances: the kernels compute in fp32 like the reference but sum in a different order;
# a dot of length K then differs by a few ulp of sum(|a*w|).
def assert_dot_close(got, want, a, w_deq):
    scale = np.abs(a) @ np.abs(w_deq).T
    err = np.abs(got - want)
    assert np.all(err <= 4e-6 * scale + 1e-7), float((err / (scale + 1e-30)).max())


@pytest.mark.parametrize("t", TYPES)
@pytest.mark.parametrize("shape", [(37, 256, 1), (1000, 2048, 1), (300, 2048, 3), (130, 896, 2),
                                   (64, 8192, 1), (48, 96, 5), (257, 1536, 9), (96, 4864, 1)])
def test_matmul(t, shape):
    n, k, m = shape
    if k % gguf.BLOCK[t][0]:
        pytest.skip("K not a multiple of the block")
    rng = np.random.default_rng(k * 7 + n + m + t)
    w = (rng.standard_normal((n, k)) * 0.02).astype(np.float32)
    raw = np.ascontiguousarray(quants.quantize(w, t))
    a = rng.standard_normal((m, k)).astype(np.float32)
    want = np.zeros((m, n), np.float32)
    po.oracle_lib().tfo_matmul(fp(want), fp(a), t, raw.ctypes.data, n, k, m, 4)
    # the weight block sits at the very end of its allocation: the kernel must not read past it
    wd = dev(raw.reshape(-1))
    ad, cd = dev(a), torch.full((m, n), float("nan"), device="cuda")
    call(native.lib().tf_op_matmul(ptr(cd), ptr(ad), t, ptr(wd), n, k, m, None))
    got = cd.cpu().numpy()
    assert_dot_close(got, want, a, quants.dequant(raw, t, k))


@pytest.mark.parametrize("t,shape", [(gguf.GGML_Q4_0, (30000, 2048, 1)), (gguf.GGML_Q4_0, (8200, 8192, 1)),
                                     (gguf.GGML_Q6_K, (30000, 2048, 1)), (gguf.GGML_Q6_K, (2100, 8192, 1)),
                                     (gguf.GGML_Q6_K, (77, 512, 1))])
def test_matmul_integer_path_large(t, shape):
    """Q4_0 matrices of 32 MB and more take the exact-integer GEMV (nibbles against the
    activation's digit planes, the -8 offset through per-block digit sums); Q6_K rows with
    K % 512 == 0 take it at any size (six-bit quants against the same planes, the -32 offset
    through 16-element digit sums, super-blocks at 2-byte offsets realigned)."""
    n, k, m = shape
    rng = np.random.default_rng(n + k + t)
    w = (rng.standard_normal((n, k)) * 0.02).astype(np.float32)
    raw = np.ascontiguousarray(quants.quantize(w, t))
    assert t == gguf.GGML_Q6_K or raw.nbytes >= 32 << 20
    a = rng.standard_normal((m, k)).astype(np.float32)
    want = np.zeros((m, n), np.float32)
    po.oracle_lib().tfo_matmul(fp(want), fp(a), t, raw.ctypes.data, n, k, m, 4)
    wd = dev(raw.reshape(-1))
    ad, cd = dev(a), torch.full((m, n), float("nan"), device="cuda")
    call(native.lib().tf_op_matmul(ptr(cd), ptr(ad), t, ptr(wd), n, k, m, None))
    assert_dot_close(cd.cpu().numpy(), want, a, quants.dequant(raw, t, k))


@pytest.mark.parametrize("t", [gguf.GGML_Q8_0, gguf.GGML_Q4_0])
@pytest.mark.parametrize("shape", [(256, 2048, 16), (1000, 2048, 64), (130, 896, 130), (96, 4864, 33),
                                   (2048, 8192, 40), (515, 1536, 300), (384, 1536, 32)])
def test_matmul_tensor_core(shape, t):
    """Q8_0 and Q4_0 at M >= 16 run the tensor-core GEMM (f16-split products, fp32
    accumulation, split-K clusters when the tiles do not cover the SMs)."""
    n, k, m = shape
    rng = np.random.default_rng(k + n + m)
    w = (rng.standard_normal((n, k)) * 0.02).astype(np.float32)
    raw = np.ascontiguousarray(quants.quantize(w, t))
    a = rng.standard_normal((m, k)).astype(np.float32)
    want = np.zeros((m, n), np.float32)
    po.oracle_lib().tfo_matmul(fp(want), fp(a), t, raw.ctypes.data, n, k, m, 4)
    wd = dev(raw.reshape(-1))
    ad, cd = dev(a), torch.full((m, n), float("nan"), device="cuda")
    call(native.lib().tf_op_matmul(ptr(cd), ptr(ad), t, ptr(wd), n, k, m, None))
    got = cd.cpu().numpy()
    scale = np.abs(a) @ np.abs(quants.dequant(raw, t, k)).T
    err = np.abs(got - want)
    assert np.all(err <= 2e-5 * scale + 1e-6), float((err / (scale + 1e-30)).max())


@pytest.mark.parametrize("t", TYPES)
def test_dequant_rows_exact(t):
    k = 512
    rng = np.random.default_rng(t)
    raw = np.ascontiguousarray(quants.quantize((rng.standard_normal((40, k)) * 0.02).astype(np.float32), t))
    rows = np.array([0, 39, 7, 7, 21], np.int32)
    want = quants.dequant(raw[rows], t, k)
    for i, r in enumerate(rows):
        o = np.zeros(k, np.float32)
        po.oracle_lib().tfo_dequant_row(fp(o), t, raw.ctypes.data, k, int(r))
        assert np.array_equal(o, want[i])
    out = torch.zeros((len(rows), k), device="cuda")
    call(native.lib().tf_op_dequant_rows(ptr(out), t, ptr(dev(raw.reshape(-1))), 40, k, ptr(dev(rows)), len(rows), None))
    assert np.array_equal(out.cpu().numpy(), want)


def test_device_status_word():
    """A row id outside the matrix is caught on the device: nothing outside W is read, the row
    comes back zero, and tf_op_device_error reports TF_DEV_ERR_BAD_INDEX once, then 0."""
    L = native.lib()
    k, n = 256, 10
    rng = np.random.default_rng(5)
    raw = np.ascontiguousarray(quants.quantize((rng.standard_normal((n, k)) * 0.02).astype(np.float32), native.TF_Q8_0))
    want = quants.dequant(raw[[3, 9]], native.TF_Q8_0, k)
    code = C.c_int(-1)
    call(L.tf_op_device_error(None, C.byref(code)))
    assert code.value == 0
    rows = np.array([3, n, -1, 9], np.int32)  # n and -1 are out of range (chosen on the host)
    out = torch.full((len(rows), k), 7.0, device="cuda")
    call(L.tf_op_dequant_rows(ptr(out), native.TF_Q8_0, ptr(dev(raw.reshape(-1))), n, k, ptr(dev(rows)), len(rows),
                              None))
    call(L.tf_op_device_error(None, C.byref(code)))
    assert code.value == native.TF_DEV_ERR_BAD_INDEX
    o = out.cpu().numpy()
    assert np.all(o[1] == 0) and np.all(o[2] == 0)
    assert np.array_equal(o[0], want[0]) and np.array_equal(o[3], want[1])
    call(L.tf_op_device_error(None, C.byref(code)))  # read once: cleared
    assert code.value == 0


def test_rmsnorm_silu_softmax():
    O, L = po.oracle_lib(), native.lib()
    rng = np.random.default_rng(11)
    for n in (7, 896, 2048, 8960):
        x = (rng.standard_normal((3, n)) * 2).astype(np.float32)
        w = rng.standard_normal(n).astype(np.float32)
        want = np.zeros_like(x)
        for r in range(3):
            O.tfo_rmsnorm(fp(want[r]), fp(np.ascontiguousarray(x[r])), fp(w), n, 1e-5)
        out = torch.zeros((3, n), device="cuda")
        call(L.tf_op_rmsnorm(ptr(out), ptr(dev(x)), ptr(dev(w)), n, 3, C.c_float(1e-5), None))
        np.testing.assert_allclose(out.cpu().numpy(), want, rtol=2e-7, atol=1e-7)
        g = x[0].copy()
        O.tfo_silu_mul(fp(g), fp(w), n)
        gd = dev(x[0].copy())
        call(L.tf_op_silu_mul(ptr(gd), ptr(dev(w)), n, None))
        np.testing.assert_allclose(gd.cpu().numpy(), g, rtol=1e-6, atol=1e-7)
        s = x.copy()
        for r in range(3):
            O.tfo_softmax(fp(s[r]), n)
        sd = dev(x.copy())
        call(L.tf_op_softmax(ptr(sd), n, 3, None))
        np.testing.assert_allclose(sd.cpu().numpy(), s, rtol=1e-5, atol=1e-9)


def test_rope():
    O, L = po.oracle_lib(), native.lib()
    for hd, theta in ((64, 500000.0), (128, 1e6), (8, 1e4)):
        f = np.zeros(hd // 2, np.float32)
        O.tfo_rope_freqs(fp(f), hd, theta, 0, 1, 1, 4, 8192)
        x = np.random.default_rng(hd).standard_normal((5, 6, hd)).astype(np.float32)
        want = x.copy()
        O.tfo_rope(fp(want), 5, 6, hd, 1000, fp(f))
        xd = dev(x)
        call(L.tf_op_rope(ptr(xd), 5, 6, hd, 1000, ptr(dev(f)), None))
        # device cosf/sinf vs glibc: a few ulp
        np.testing.assert_allclose(xd.cpu().numpy(), want, rtol=0, atol=2e-5)


def test_argmax_ties_and_nan():
    L = native.lib()
    rows = np.random.default_rng(2).standard_normal((6, 151936)).astype(np.float32)
    rows[1, [5, 900, 151935]] = 50.0                 # tie: first index wins
    rows[2, :] = -3.0                                # all equal -> 0
    rows[3, 0] = np.nan                              # NaN at 0 -> 0 (every compare is false)
    rows[4, 17] = np.nan                             # NaN elsewhere is skipped
    rows[5, 77] = np.inf
    want = [po.oracle_lib().tfo_sample_greedy(fp(np.ascontiguousarray(r)), r.size) for r in rows]
    out = torch.zeros(6, dtype=torch.int32, device="cuda")
    call(L.tf_op_argmax(ptr(dev(rows)), rows.shape[1], 6, ptr(out), None))
    assert out.cpu().tolist() == want
    assert want[1] == 5 and want[2] == 0 and want[3] == 0


@pytest.mark.parametrize("kv_type", [native.TF_KV_F32, native.TF_KV_F16, native.TF_KV_BF16])
@pytest.mark.parametrize("shape", [(1, 32, 8, 64), (300, 14, 2, 64), (1100, 12, 2, 128), (9, 4, 2, 8),
                                   (8192, 32, 8, 64)])
def test_attn_decode(kv_type, shape):
    n_pos, H, KV, hd = shape
    cap = n_pos + 5
    rng = np.random.default_rng(n_pos + kv_type)
    q = rng.standard_normal((H, hd)).astype(np.float32)
    k = rng.standard_normal((n_pos, KV, hd)).astype(np.float32)
    v = rng.standard_normal((n_pos, KV, hd)).astype(np.float32)
    tdt = {native.TF_KV_F32: torch.float32, native.TF_KV_F16: torch.float16, native.TF_KV_BF16: torch.bfloat16}[kv_type]
    kc = torch.zeros((KV, cap, hd), dtype=tdt, device="cuda")
    vc = torch.zeros((KV, cap, hd), dtype=tdt, device="cuda")
    kc[:, :n_pos] = dev(k).permute(1, 0, 2).to(tdt)
    vc[:, :n_pos] = dev(v).permute(1, 0, 2).to(tdt)
    # the oracle sees exactly the stored (rounded) values
    kr = kc[:, :n_pos].float().permute(1, 0, 2).contiguous().cpu().numpy()
    vr = vc[:, :n_pos].float().permute(1, 0, 2).contiguous().cpu().numpy()
    want = np.zeros((H, hd), np.float32)
    po.oracle_lib().tfo_attn_decode(fp(want), fp(q), fp(kr), fp(vr), n_pos, H, KV, hd)
    out = torch.zeros((H, hd), device="cuda")
    call(native.lib().tf_op_attn_decode(ptr(out), ptr(dev(q)), ptr(kc), ptr(vc), kv_type, cap, n_pos, H, KV, hd, None))
    np.testing.assert_allclose(out.cpu().numpy(), want, rtol=0, atol=2e-5)


@pytest.mark.parametrize("shape", [(17, 8, 2, 64), (64, 14, 2, 64), (33, 12, 2, 128)])
def test_attn_prefill(shape):
    S, H, KV, hd = shape
    rng = np.random.default_rng(S)
    q = rng.standard_normal((S, H, hd)).astype(np.float32)
    k = rng.standard_normal((S, KV, hd)).astype(np.float32)
    v = rng.standard_normal((S, KV, hd)).astype(np.float32)
    want = np.zeros_like(q)
    po.oracle_lib().tfo_attn_prefill(fp(want), fp(q), fp(k), fp(v), S, H, KV, hd)
    out = torch.zeros_like(dev(q))
    call(native.lib().tf_op_attn_prefill(ptr(out), ptr(dev(q)), ptr(dev(k)), ptr(dev(v)), S, H, KV, hd, None))
    np.testing.assert_allclose(out.cpu().numpy(), want, rtol=0, atol=2e-5)
