"""CPU restatement of the tensor-core GEMM's operand arithmetic (gemm.cuh, gemm.cu): the exact
f16 split of every Q8_0 / Q4_0 weight after the per-matrix power-of-two scale 2^sw
(q8_scale_exponent, gm_dequant16_r), and the f16 split of the activation rows after the per-row
scale 2^sx (tf_xprep_rows_kernel / tf_xprep_kernel).  Pins the precision the GEMM path claims:
Wh + Wl == q * d * 2^sw exactly, and Xh + Xl within 2^-22 of each row's maximum; the GPU tests
check the kernels themselves against the reference."""
import numpy as np
import pytest

from tinferno_b200 import gguf, quants


def scale_exponent(d_bits):
    """q8_exponent_from_dbits over the blocks' fp16 d bits (sign dropped): 2^(21 - E) for the
    largest biased exponent E (subnormals count as E = 1) maps every |q * d| below 2^14."""
    mx = int((d_bits & 0x7FFF).max())
    if mx == 0 or mx >= 0x7C00:
        return 0
    return 21 - max(mx >> 10, 1)


def weight_split(q, d_bits, sw):
    """gm_dequant16_r: dsc = f16(d * 2^sw), Wh = f16(q * dsc) (one rounding of the exact
    product), Wl = f16(q * dsc - Wh) (the remainder, exact in f16)."""
    d = d_bits.view(np.float16).astype(np.float32)
    dsc = (d * np.float32(2.0 ** sw)).astype(np.float16)
    prod = q.astype(np.float64) * dsc.astype(np.float64)[:, None]   # exact: 8 x 11 bits
    wh = prod.astype(np.float16)
    wl = (prod - wh.astype(np.float64)).astype(np.float16)
    return dsc, prod, wh, wl


def activation_split(x):
    """xprep: am = the row's largest |x|, 2^sx = 2^(140 - biased exponent of am) (|x| 2^sx <
    2^14), Xh = f16(x 2^sx), Xl = f16(x 2^sx - Xh) with the difference exact in fp32."""
    am = np.abs(x).max(axis=1).astype(np.float32)
    be = ((am.view(np.uint32) >> 23) & 0xFF).astype(np.int64)
    sx = np.clip(140 - be, -100, 100)
    S = np.exp2(sx.astype(np.float64)).astype(np.float32)[:, None]
    v = (x.astype(np.float32) * S).astype(np.float32)                # exact power-of-two scaling
    xh = v.astype(np.float16)
    xl = (v - xh.astype(np.float32)).astype(np.float16)
    return sx, v, xh, xl


def q8_blocks(w):
    """(quants [rows][K], fp16 d bits [rows * K/32]) of the reference quantiser's Q8_0 rows."""
    raw = np.ascontiguousarray(quants.quantize(w, gguf.GGML_Q8_0)).reshape(-1, 34)
    d_bits = raw[:, :2].copy().view(np.uint16).reshape(-1)
    q = raw[:, 2:].view(np.int8).astype(np.int64)
    return q, d_bits


@pytest.mark.parametrize("std,K", [(0.02, 1536), (0.02, 8960), (1.0, 2048), (1e-3, 896)])
def test_q8_weight_split_is_exact(std, K):
    rng = np.random.default_rng(11)
    w = (rng.standard_normal((64, K)) * std).astype(np.float32)
    q, d_bits = q8_blocks(w)
    sw = scale_exponent(d_bits)
    dsc, prod, wh, wl = weight_split(q, d_bits, sw)
    assert np.isfinite(wh).all() and np.isfinite(wl).all()
    assert np.abs(prod).max() < 2.0 ** 14
    # the blocks parse as Q8_0: q * d is w to within half a quantisation step plus the fp16
    # rounding of d (|q| <= 127 times half an ulp of d; small d are f16 subnormals)
    d = d_bits.view(np.float16).astype(np.float64)
    half_ulp = 0.5 * np.spacing(np.abs(d_bits.view(np.float16))).astype(np.float64)
    bound = (0.5 * np.abs(d) + 127 * half_ulp)[:, None]
    assert (np.abs(prod * 2.0 ** -sw - w.reshape(-1, 32)) <= bound).all()
    # the scaled block scale is d exactly (a power-of-two scaling of an f16 value)
    assert np.array_equal(dsc.astype(np.float64), d * 2.0 ** sw)
    # Wh + Wl is q * d * 2^sw with no rounding at all
    assert np.array_equal(wh.astype(np.float64) + wl.astype(np.float64), prod)


def test_q4_weight_split_is_exact():
    rng = np.random.default_rng(5)
    w = (rng.standard_normal((32, 2048)) * 0.02).astype(np.float32)
    raw = np.ascontiguousarray(quants.quantize(w, gguf.GGML_Q4_0)).reshape(-1, 18)
    d_bits = raw[:, :2].copy().view(np.uint16).reshape(-1)
    nib = raw[:, 2:]
    q = np.concatenate([(nib & 0x0F), (nib >> 4)], axis=1).astype(np.int64) - 8
    sw = scale_exponent(d_bits)
    _, prod, wh, wl = weight_split(q, d_bits, sw)
    assert np.array_equal(wh.astype(np.float64) + wl.astype(np.float64), prod)


@pytest.mark.parametrize("scale", [1.0, 1e-3, 300.0])
def test_activation_split_keeps_22_bits_of_the_row_maximum(scale):
    rng = np.random.default_rng(3)
    x = (rng.standard_normal((48, 1536)) * scale).astype(np.float32)
    x[5, :] = 0.0           # a zero row: the largest shift, halves all zero
    x[7, 100] = 1e4 * scale  # one large element: the rest of the row keeps 2^-22 of it
    sx, v, xh, xl = activation_split(x)
    am = np.abs(x).max(axis=1).astype(np.float64)
    assert np.isfinite(xh).all() and np.isfinite(xl).all()
    assert np.abs(v).max() < 2.0 ** 14
    back = (xh.astype(np.float64) + xl.astype(np.float64)) * np.exp2(-sx.astype(np.float64))[:, None]
    err = np.abs(back - x.astype(np.float64)).max(axis=1)
    assert (err <= am * 2.0 ** -22).all(), float((err / np.maximum(am, 1e-300)).max())
    assert np.array_equal(back[5], np.zeros(1536))


def test_split_product_against_exact_dot():
    """The three accumulated products (Wh Xh + Wh Xl + Wl Xh, the Wl Xl term dropped), scaled
    back by 2^-(sw+sx), against the exact dot of the dequantised weights with the fp32 row:
    within 2^-20 of sum |w| |x| per output."""
    rng = np.random.default_rng(9)
    K = 1536
    w = (rng.standard_normal((40, K)) * 0.02).astype(np.float32)
    x = rng.standard_normal((6, K)).astype(np.float32)
    q, d_bits = q8_blocks(w)
    sw = scale_exponent(d_bits)
    _, prod, wh, wl = weight_split(q, d_bits, sw)
    sx, v, xh, xl = activation_split(x)
    Wh, Wl = wh.reshape(40, K).astype(np.float64), wl.reshape(40, K).astype(np.float64)
    Xh, Xl = xh.astype(np.float64), xl.astype(np.float64)
    y = (Xh @ Wh.T + Xl @ Wh.T + Xh @ Wl.T) * np.exp2(-(sw + sx.astype(np.float64)))[:, None]
    wdq = prod.reshape(40, K) * 2.0 ** -sw            # q * d, the reference's dequantised weight
    exact = x.astype(np.float64) @ wdq.T
    bound = (np.abs(x).astype(np.float64) @ np.abs(wdq).T) * 2.0 ** -20
    assert (np.abs(y - exact) <= bound).all()
