"""CPU restatement of the exact-integer GEMV arithmetic (dots.cuh), checked against the oracle's
dequantised dot (src/quant.cpp:266-363, dequant_q6_K_row :101-127 + dot_f32): the activation's
three signed-byte digit planes per 32-element block, and the Q8_0, Q4_0 and Q6_K unit sums as
the kernels form them (Q6_K with its word realignment, six-bit assembly and the -32 offset
through 16-element digit sums).  Pins the formulas on the CPU; the GPU tests check the kernels."""
import numpy as np
import pytest

import pyoracle as po
from tinferno_b200 import gguf, quants

fp = po._fp


def s8(v):
    v = np.asarray(v, np.int64) & 0xFF
    return np.where(v > 127, v - 256, v)


def digit_planes(x):
    """q8_build_planes / q4_build_planes: per 32-element block, 2^sh with the block maximum
    below 2^22, X = round-half-even(x * 2^sh), X = x0 + 2^8 x1 + 2^16 x2 in signed bytes."""
    xb = x.reshape(-1, 32)
    am = np.abs(xb).max(axis=1).astype(np.float32)
    e = ((am.view(np.uint32) >> 23) & 0xFF).astype(np.int64)
    sh = np.minimum(148 - e, 126)
    X = np.rint(xb.astype(np.float64) * np.exp2(sh)[:, None]).astype(np.int64).reshape(-1)
    Xu = X & 0xFFFFFFFF
    d = [s8(Xu), s8((Xu + 128) >> 8), s8((Xu + 32896) >> 16)]
    assert np.array_equal(d[0] + 256 * d[1] + 65536 * d[2], X)
    assert np.abs(X).max() < 1 << 22
    return d, np.exp2(-sh.astype(np.float64))


def combine(s):
    """tA = S2 * 2^16 + S1 * 2^8 + S0: the block (or sub-block) sum of q * X."""
    return s[2] * 65536 + s[1] * 256 + s[0]


def dot_q8_0(row, d, inv):
    blk = row.reshape(-1, 34)
    sc = blk[:, :2].copy().view(np.float16).astype(np.float64).reshape(-1)
    q = blk[:, 2:].view(np.int8).astype(np.int64)
    t = combine([(q * p.reshape(-1, 32)).sum(axis=1) for p in d])
    return float((sc * inv * t).sum())


def dot_q4_0(row, d, inv):
    blk = row.reshape(-1, 18)
    sc = blk[:, :2].copy().view(np.float16).astype(np.float64).reshape(-1)
    qs = blk[:, 2:].astype(np.int64)
    nib = np.concatenate([qs & 15, qs >> 4], axis=1)  # elements 0..15 low, 16..31 high nibbles
    # nibbles as non-negative bytes in dp4a, the -8 through the block's digit sums
    t = combine([(nib * p.reshape(-1, 32)).sum(axis=1) - 8 * p.reshape(-1, 32).sum(axis=1) for p in d])
    return float((sc * inv * t).sum())


def word(buf, off):
    return int(buf[off]) | int(buf[off + 1]) << 8 | int(buf[off + 2]) << 16 | int(buf[off + 3]) << 24


def byte_perm(x, y, sel):
    b = [(x >> (8 * i)) & 0xFF for i in range(4)] + [(y >> (8 * i)) & 0xFF for i in range(4)]
    return sum(b[(sel >> (4 * i)) & 7] << (8 * i) for i in range(4))


def dot_q6_k(row, d, inv):
    """unit_dot_q6k_int over the row's 64-element units (h, j) of each super-block, the row
    starting 4-byte aligned as in the kernel's stages, so odd super-blocks sit 2 bytes off."""
    total = 0.0
    for u in range(row.size // 210 * 4):
        sb, h, j = u >> 2, (u >> 1) & 1, u & 1
        base = 210 * sb
        m2 = base & 3
        assert m2 in (0, 2)
        aw = base - m2
        sel = 0x5432 if m2 else 0x3210
        blk_a = 8 * sb + 4 * h + j
        blk_b = blk_a + 2
        hw = lambda k: int(row[base + 2 * k]) | int(row[base + 2 * k + 1]) << 8  # noqa: E731
        sc_a, sc_b = hw(96 + 4 * h + j), hw(96 + 4 * h + j + 2)
        dd = float(np.uint16(hw(104)).view(np.float16))
        fa = fb = 0.0
        for half in range(2):
            acc = np.zeros((2, 3), np.int64)
            for k in range(4):
                i = 4 * half + k
                ql_off, qh_off = aw + 64 * h + 32 * j + 4 * i, aw + 128 + 32 * h + 4 * i
                lw = byte_perm(word(row, ql_off), word(row, ql_off + 4), sel)
                hq = byte_perm(word(row, qh_off), word(row, qh_off + 4), sel)
                ua = (lw & 0x0F0F0F0F) | ((hq << (4 - 2 * j)) & 0x30303030)
                ub = ((lw >> 4) & 0x0F0F0F0F) | ((hq >> (2 * j)) & 0x30303030)
                bytes_a = s8([(ua >> (8 * n)) & 0xFF for n in range(4)])
                bytes_b = s8([(ub >> (8 * n)) & 0xFF for n in range(4)])
                for p in range(3):
                    acc[0, p] += int((bytes_a * d[p][32 * blk_a + 4 * i:32 * blk_a + 4 * i + 4]).sum())
                    acc[1, p] += int((bytes_b * d[p][32 * blk_b + 4 * i:32 * blk_b + 4 * i + 4]).sum())
            for p in range(3):  # q = u - 32 through the 16-element digit sums
                acc[0, p] -= 32 * int(d[p][32 * blk_a + 16 * half:32 * blk_a + 16 * half + 16].sum())
                acc[1, p] -= 32 * int(d[p][32 * blk_b + 16 * half:32 * blk_b + 16 * half + 16].sum())
            fa += float(np.int8(np.uint8((sc_a >> (8 * half)) & 0xFF))) * combine(acc[0])
            fb += float(np.int8(np.uint8((sc_b >> (8 * half)) & 0xFF))) * combine(acc[1])
        total += dd * (inv[blk_a] * fa + inv[blk_b] * fb)
    return total


DOTS = {gguf.GGML_Q8_0: dot_q8_0, gguf.GGML_Q4_0: dot_q4_0, gguf.GGML_Q6_K: dot_q6_k}


@pytest.mark.parametrize("t", list(DOTS), ids=lambda t: gguf.TYPE_NAME[t])
@pytest.mark.parametrize("k", [512, 2048])
def test_integer_unit_sums_match_oracle(t, k):
    n = 6
    rng = np.random.default_rng(k + t)
    w = (rng.standard_normal((n, k)) * 0.02).astype(np.float32)
    raw = np.ascontiguousarray(quants.quantize(w, t))
    x = rng.standard_normal(k).astype(np.float32)
    x[:32] *= 1e-3  # blocks of very different magnitude take their own shifts
    x[32:64] = 0.0  # an all-zero block takes the largest shift
    want = np.zeros((1, n), np.float32)
    po.oracle_lib().tfo_matmul(fp(want), fp(x[None, :].copy()), t, raw.ctypes.data, n, k, 1, 1)
    d, inv = digit_planes(x)
    rows = raw.reshape(n, -1)
    deq = quants.dequant(raw, t, k).reshape(n, k).astype(np.float64)
    scale = np.abs(deq) @ np.abs(x.astype(np.float64))
    for r in range(n):
        got = DOTS[t](rows[r], d, inv)
        assert abs(got - want[0, r]) <= 4e-6 * scale[r] + 1e-7, (r, got, want[0, r])
