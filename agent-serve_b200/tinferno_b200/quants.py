"""Block quantisers and dequantisers (numpy, host side) for the GGUF formats the engine reads.

Byte layouts are the reference's (src/quant.hpp:13-35 of RohanDisa/agent-serve):
  Q8_0  {fp16 d; int8 qs[32]}                                    34 B / 32 weights
  Q4_0  {fp16 d; uint8 qs[16]}  q = nibble - 8, low nibbles -> 0..15   18 B / 32
  Q4_1  {fp16 d; fp16 m; uint8 qs[16]}  x = q*d + m                    20 B / 32
  Q6_K  {uint8 ql[128]; uint8 qh[64]; int8 scales[16]; fp16 d}         210 B / 256

``quant_q8_0`` and ``quant_q4_0`` follow the reference quantisers (src/quant.cpp:147-183,
with the v2 build's round-to-nearest-even fp16 conversion and std::round's
half-away-from-zero rounding).  The reference has no Q4_1 or Q6_K quantiser; the ones
here are new and only need to produce valid encodings, since the reference, the oracle
and the CUDA path all read the same bytes.  ``dequant`` restates src/quant.cpp:66-145 for
host-side checks.
"""
from __future__ import annotations

import numpy as np

from .gguf import GGML_F16, GGML_F32, GGML_Q4_0, GGML_Q4_1, GGML_Q6_K, GGML_Q8_0


def _round_half_away(v: np.ndarray) -> np.ndarray:
    """std::round on float32 values, exactly (the sum is exact in float64)."""
    a = np.floor(np.abs(v).astype(np.float64) + 0.5)
    return np.copysign(a, v)


def _f16_bits(v: np.ndarray) -> np.ndarray:
    return v.astype(np.float32).astype(np.float16).view(np.uint16)  # numpy rounds to nearest even


def quant_q8_0(x: np.ndarray) -> np.ndarray:
    """x: float32 [rows, K] -> uint8 [rows, K/32*34].  src/quant.cpp:147-163."""
    rows, k = x.shape
    xb = x.reshape(rows, k // 32, 32).astype(np.float32, copy=False)
    amax = np.abs(xb).max(axis=2)
    d = (amax / np.float32(127.0)).astype(np.float32)
    with np.errstate(divide="ignore"):
        idv = np.where(d > 0, np.float32(1.0) / np.where(d > 0, d, 1), np.float32(0)).astype(np.float32)
    q = _round_half_away(xb * idv[:, :, None])
    q = np.clip(q, -127, 127).astype(np.int8)
    out = np.empty((rows, k // 32, 34), dtype=np.uint8)
    out[:, :, 0:2] = _f16_bits(d).view(np.uint8).reshape(rows, k // 32, 2)
    out[:, :, 2:] = q.view(np.uint8)
    return out.reshape(rows, -1)


def quant_q4_0(x: np.ndarray) -> np.ndarray:
    """x: float32 [rows, K] -> uint8 [rows, K/32*18].  src/quant.cpp:165-183."""
    rows, k = x.shape
    xb = x.reshape(rows, k // 32, 32).astype(np.float32, copy=False)
    amax = np.abs(xb).max(axis=2)
    d = (amax / np.float32(8.0)).astype(np.float32)
    idv = np.where(d > 0, np.float32(1.0) / np.where(d > 0, d, 1), np.float32(0)).astype(np.float32)
    q = np.clip(_round_half_away(xb * idv[:, :, None]), -8, 7).astype(np.int16) + 8
    out = np.empty((rows, k // 32, 18), dtype=np.uint8)
    out[:, :, 0:2] = _f16_bits(d).view(np.uint8).reshape(rows, k // 32, 2)
    out[:, :, 2:] = (q[:, :, :16] | (q[:, :, 16:] << 4)).astype(np.uint8)
    return out.reshape(rows, -1)


def quant_q4_1(x: np.ndarray) -> np.ndarray:
    """New quantiser (the reference has none): per 32-block min m and step d = (max-min)/15,
    q = round((x - m)/d) in [0, 15]; stores fp16 d and fp16 m."""
    rows, k = x.shape
    xb = x.reshape(rows, k // 32, 32).astype(np.float32, copy=False)
    mn = xb.min(axis=2)
    mx = xb.max(axis=2)
    d = ((mx - mn) / np.float32(15.0)).astype(np.float32)
    d16 = d.astype(np.float16)
    m16 = mn.astype(np.float16)
    dq = d16.astype(np.float32)
    idv = np.where(dq > 0, np.float32(1.0) / np.where(dq > 0, dq, 1), np.float32(0)).astype(np.float32)
    q = np.clip(_round_half_away((xb - m16.astype(np.float32)[:, :, None]) * idv[:, :, None]), 0, 15)
    q = q.astype(np.uint8)
    out = np.empty((rows, k // 32, 20), dtype=np.uint8)
    out[:, :, 0:2] = d16.view(np.uint16).view(np.uint8).reshape(rows, k // 32, 2)
    out[:, :, 2:4] = m16.view(np.uint16).view(np.uint8).reshape(rows, k // 32, 2)
    out[:, :, 4:] = q[:, :, :16] | (q[:, :, 16:] << 4)
    return out.reshape(rows, -1)


def quant_q6_k(x: np.ndarray) -> np.ndarray:
    """New quantiser (the reference has none).  Per 256-element super-block: 16 sub-blocks of
    16 elements with an int8 scale each and one fp16 super-scale d; q in [-32, 31] stored
    as q+32 split into 4 low bits (ql) and 2 high bits (qh) in the interleave that
    dequant_q6_K (src/quant.cpp:101-127) reads."""
    rows, k = x.shape
    nsb = k // 256
    xb = x.reshape(rows, nsb, 16, 16).astype(np.float32, copy=False)
    amax = np.abs(xb).max(axis=3)                              # [rows, nsb, 16]
    sub = (amax / np.float32(31.5)).astype(np.float32)         # per-sub-block step
    smax = sub.max(axis=2)                                     # [rows, nsb]
    d = (smax / np.float32(127.0)).astype(np.float32)
    d16 = d.astype(np.float16)
    dq = d16.astype(np.float32)
    idv = np.where(dq > 0, np.float32(1.0) / np.where(dq > 0, dq, 1), np.float32(0)).astype(np.float32)
    sc = np.clip(_round_half_away(sub * idv[:, :, None]), -127, 127).astype(np.int8)  # [rows,nsb,16]
    step = (dq[:, :, None] * sc.astype(np.float32)).astype(np.float32)
    istep = np.where(step > 0, np.float32(1.0) / np.where(step > 0, step, 1), np.float32(0))
    q = np.clip(_round_half_away(xb * istep[:, :, :, None].astype(np.float32)), -32, 31)
    u = (q.astype(np.int16) + 32).astype(np.uint8).reshape(rows, nsb, 2, 4, 32)  # [.., half, quarter, l]
    lo = u & 0x0F
    hi = u >> 4
    ql = np.empty((rows, nsb, 2, 64), dtype=np.uint8)
    ql[..., :32] = lo[:, :, :, 0, :] | (lo[:, :, :, 2, :] << 4)
    ql[..., 32:] = lo[:, :, :, 1, :] | (lo[:, :, :, 3, :] << 4)
    qh = (hi[:, :, :, 0, :] | (hi[:, :, :, 1, :] << 2) | (hi[:, :, :, 2, :] << 4)
          | (hi[:, :, :, 3, :] << 6)).astype(np.uint8)              # [rows, nsb, 2, 32]
    out = np.empty((rows, nsb, 210), dtype=np.uint8)
    out[:, :, 0:128] = ql.reshape(rows, nsb, 128)
    out[:, :, 128:192] = qh.reshape(rows, nsb, 64)
    out[:, :, 192:208] = sc.view(np.uint8)
    out[:, :, 208:210] = d16.view(np.uint16).view(np.uint8).reshape(rows, nsb, 2)
    return out.reshape(rows, -1)


def quantize(x: np.ndarray, ggml_type: int) -> np.ndarray:
    """float32 [rows, K] -> uint8 bytes of the tensor in the given type."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    if ggml_type == GGML_F32:
        return x.view(np.uint8).reshape(x.shape[0], -1)
    if ggml_type == GGML_F16:
        return x.astype(np.float16).view(np.uint8).reshape(x.shape[0], -1)
    if ggml_type == GGML_Q8_0:
        return quant_q8_0(x)
    if ggml_type == GGML_Q4_0:
        return quant_q4_0(x)
    if ggml_type == GGML_Q4_1:
        return quant_q4_1(x)
    if ggml_type == GGML_Q6_K:
        return quant_q6_k(x)
    raise ValueError(f"unsupported type {ggml_type}")


def dequant(raw: np.ndarray, ggml_type: int, k: int) -> np.ndarray:
    """uint8 [rows, rowbytes] -> float32 [rows, K]; restates src/quant.cpp:66-145."""
    raw = np.ascontiguousarray(raw, dtype=np.uint8)
    raw = raw.reshape(-1, raw.shape[-1]) if raw.ndim > 1 else raw.reshape(1, -1)
    rows = raw.shape[0]
    if ggml_type == GGML_F32:
        return raw.view(np.float32).reshape(rows, k).copy()
    if ggml_type == GGML_F16:
        return raw.view(np.float16).astype(np.float32).reshape(rows, k)
    if ggml_type == GGML_Q8_0:
        b = raw.reshape(rows, k // 32, 34)
        d = b[:, :, 0:2].copy().view(np.float16).astype(np.float32)
        q = b[:, :, 2:].view(np.int8).astype(np.float32)
        return (d * q).astype(np.float32).reshape(rows, k)
    if ggml_type == GGML_Q4_0:
        b = raw.reshape(rows, k // 32, 18)
        d = b[:, :, 0:2].copy().view(np.float16).astype(np.float32)
        qs = b[:, :, 2:]
        q = np.concatenate([(qs & 0x0F).astype(np.int16) - 8, (qs >> 4).astype(np.int16) - 8], axis=2)
        return (d * q.astype(np.float32)).astype(np.float32).reshape(rows, k)
    if ggml_type == GGML_Q4_1:
        b = raw.reshape(rows, k // 32, 20)
        d = b[:, :, 0:2].copy().view(np.float16).astype(np.float32)
        m = b[:, :, 2:4].copy().view(np.float16).astype(np.float32)
        qs = b[:, :, 4:]
        q = np.concatenate([qs & 0x0F, qs >> 4], axis=2).astype(np.float32)
        # the reference build contracts q*d + m to one FMA: compute in float64 and round once
        return (q.astype(np.float64) * d + m).astype(np.float32).reshape(rows, k)
    if ggml_type == GGML_Q6_K:
        nsb = k // 256
        b = raw.reshape(rows, nsb, 210)
        ql = b[:, :, 0:128].reshape(rows, nsb, 2, 64)
        qh = b[:, :, 128:192].reshape(rows, nsb, 2, 32)
        sc = b[:, :, 192:208].view(np.int8).astype(np.float32).reshape(rows, nsb, 2, 8)
        d = b[:, :, 208:210].copy().view(np.float16).astype(np.float32)  # [rows, nsb, 1]
        lo = np.stack([ql[..., :32] & 0xF, ql[..., 32:] & 0xF, ql[..., :32] >> 4, ql[..., 32:] >> 4], axis=3)
        hi = np.stack([(qh >> 0) & 3, (qh >> 2) & 3, (qh >> 4) & 3, (qh >> 6) & 3], axis=3)
        q = (lo | (hi << 4)).astype(np.int16) - 32                      # [rows, nsb, 2, 4, 32]
        scale = sc.reshape(rows, nsb, 2, 4, 2)                           # quarter t: sc[2t + l//16]
        s = np.repeat(scale, 16, axis=4)                                 # [rows, nsb, 2, 4, 32]
        y = (d[:, :, :, None, None] * s).astype(np.float32) * q.astype(np.float32)
        return y.astype(np.float32).reshape(rows, k)
    raise ValueError(f"unsupported type {ggml_type}")
