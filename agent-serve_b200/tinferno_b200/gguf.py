"""GGUF v2/v3 reader and v3 writer (host side, numpy).

The reader binds what the reference engine's loader binds (src/gguf.cpp:88-168 of
RohanDisa/agent-serve): the key/value metadata, then the tensor table with ggml type
ids and ne[] in ggml order (ne[0] innermost), data offsets relative to the aligned
data section (``general.alignment``, default 32).  Tensor bytes are exposed as
zero-copy views of a read-only memory map, in their native block layouts; the
device upload copies those bytes verbatim.

The writer emits what the reference's ``write_gguf`` emits (src/gguf.cpp:237-300):
version 3, string/u64/f32 metadata, tensor infos, 32-byte aligned payloads.  Payloads
are produced by callbacks so multi-GB synthetic models stream to disk.
"""
from __future__ import annotations

import mmap
import os
import struct
from dataclasses import dataclass, field
from typing import Callable, Dict, Iterable, List, Optional, Sequence, Tuple

import numpy as np

GGUF_MAGIC = 0x46554747

# ggml type id -> (block size in elements, block size in bytes); src/tensor.cpp:42-70
GGML_F32, GGML_F16, GGML_Q4_0, GGML_Q4_1, GGML_Q8_0, GGML_Q6_K = 0, 1, 2, 3, 8, 14
BLOCK = {
    GGML_F32: (1, 4),
    GGML_F16: (1, 2),
    GGML_Q4_0: (32, 18),
    GGML_Q4_1: (32, 20),
    GGML_Q8_0: (32, 34),
    GGML_Q6_K: (256, 210),
}
TYPE_NAME = {GGML_F32: "F32", GGML_F16: "F16", GGML_Q4_0: "Q4_0", GGML_Q4_1: "Q4_1",
             GGML_Q8_0: "Q8_0", GGML_Q6_K: "Q6_K"}
NAME_TYPE = {v: k for k, v in TYPE_NAME.items()}


def row_nbytes(ggml_type: int, ne0: int) -> int:
    bs, bb = BLOCK[ggml_type]
    if ne0 % bs:
        raise ValueError(f"row length {ne0} not divisible by block size {bs}")
    return (ne0 // bs) * bb


def tensor_nbytes(ggml_type: int, ne: Sequence[int]) -> int:
    rows = 1
    for d in ne[1:]:
        rows *= int(d)
    return rows * row_nbytes(ggml_type, int(ne[0]))


@dataclass
class TensorInfo:
    name: str
    ggml_type: int
    ne: Tuple[int, ...]
    offset: int = 0          # absolute file offset of the data
    nbytes: int = 0
    data: Optional[np.ndarray] = None  # uint8 view (reader) or None

    @property
    def cols(self) -> int:
        return int(self.ne[0])

    @property
    def rows(self) -> int:
        r = 1
        for d in self.ne[1:]:
            r *= int(d)
        return r


class GGUFReader:
    """Read-only GGUF view.  ``tensors`` maps name -> TensorInfo with ``data`` a uint8
    memmap slice; ``kv`` holds scalars, strings and lists."""

    def __init__(self, path: str):
        self.path = path
        self._f = open(path, "rb")
        self._mm = mmap.mmap(self._f.fileno(), 0, access=mmap.ACCESS_READ)
        self.buf = np.frombuffer(self._mm, dtype=np.uint8)
        self.kv: Dict[str, object] = {}
        self.tensors: Dict[str, TensorInfo] = {}
        self.order: List[str] = []
        self._parse()

    # -- cursor helpers
    def _rd(self, fmt: str):
        v = struct.unpack_from("<" + fmt, self._mm, self._p)
        self._p += struct.calcsize("<" + fmt)
        return v[0]

    def _rdstr(self) -> str:
        n = self._rd("Q")
        if self._p + n > len(self._mm):
            raise ValueError("GGUF string overflow")
        s = self._mm[self._p:self._p + n].decode("utf-8", errors="replace")
        self._p += n
        return s

    _SCALAR = {0: "B", 1: "b", 2: "H", 3: "h", 4: "I", 5: "i", 6: "f", 7: "?", 10: "Q", 11: "q", 12: "d"}

    def _value(self, t: int):
        if t in self._SCALAR:
            return self._rd(self._SCALAR[t])
        if t == 8:
            return self._rdstr()
        if t == 9:
            et = self._rd("I")
            n = self._rd("Q")
            return [self._value(et) for _ in range(n)]
        raise ValueError(f"unknown GGUF value type {t}")

    def _parse(self):
        self._p = 0
        if self._rd("I") != GGUF_MAGIC:
            raise ValueError(f"not a GGUF file: {self.path}")
        version = self._rd("I")
        if version not in (2, 3):
            raise ValueError("unsupported GGUF version")
        n_tensors = self._rd("Q")
        n_kv = self._rd("Q")
        for _ in range(n_kv):
            key = self._rdstr()
            t = self._rd("I")
            self.kv[key] = self._value(t)
        align = int(self.kv.get("general.alignment", 32)) or 32
        infos = []
        for _ in range(n_tensors):
            name = self._rdstr()
            nd = self._rd("I")
            if not 1 <= nd <= 4:
                raise ValueError(f"bad ndim for {name}")
            ne = tuple(self._rd("Q") for _ in range(nd))
            t = self._rd("I")
            if t not in BLOCK:
                raise ValueError(f"unsupported ggml type {t}")
            off = self._rd("Q")
            infos.append(TensorInfo(name, t, ne, off, tensor_nbytes(t, ne)))
        data_off = (self._p + align - 1) // align * align
        for ti in infos:
            ti.offset += data_off
            if ti.offset + ti.nbytes > len(self._mm):
                raise ValueError(f"tensor out of range: {ti.name}")
            ti.data = self.buf[ti.offset:ti.offset + ti.nbytes]
            self.tensors[ti.name] = ti
            self.order.append(ti.name)

    # reference accessors: src/gguf.hpp:10-31
    @property
    def arch(self) -> str:
        return str(self.kv.get("general.architecture", "llama"))

    def u64(self, key: str, default: int = 0) -> int:
        v = self.kv.get(key, default)
        return int(v) if isinstance(v, (int, np.integer, bool)) else default

    def f32(self, key: str, default: float = 0.0) -> float:
        v = self.kv.get(key, default)
        return float(np.float32(v)) if isinstance(v, (int, float)) else default

    def str(self, key: str, default: str = "") -> str:
        v = self.kv.get(key, default)
        return v if isinstance(v, str) else default

    def weight_bytes(self) -> int:
        """src/gguf.cpp:219-223: bytes of every tensor in the file."""
        return sum(t.nbytes for t in self.tensors.values())

    def close(self):
        self.buf = None
        for t in self.tensors.values():
            t.data = None
        try:
            self._mm.close()
        except BufferError:
            pass
        self._f.close()


# ---------------------------------------------------------------------------------------
# writer

def _wstr(f, s: str):
    b = s.encode("utf-8")
    f.write(struct.pack("<Q", len(b)))
    f.write(b)


@dataclass
class TensorSpec:
    name: str
    ggml_type: int
    ne: Tuple[int, ...]
    produce: Callable[[], Iterable[bytes]] = field(repr=False, default=None)

    @property
    def nbytes(self) -> int:
        return tensor_nbytes(self.ggml_type, self.ne)


def write_gguf(path: str, meta_str: Dict[str, str], meta_u64: Dict[str, int],
               meta_f32: Dict[str, float], tensors: Sequence[TensorSpec], align: int = 32):
    """Write a GGUF v3 file; each TensorSpec.produce() yields the tensor's bytes in order
    (any chunking) and must yield exactly ``nbytes``."""
    tmp = path + ".tmp"
    with open(tmp, "wb") as f:
        f.write(struct.pack("<IIQQ", GGUF_MAGIC, 3, len(tensors),
                            len(meta_str) + len(meta_u64) + len(meta_f32)))
        for k, v in meta_str.items():
            _wstr(f, k)
            f.write(struct.pack("<I", 8))
            _wstr(f, v)
        for k, v in meta_u64.items():
            _wstr(f, k)
            f.write(struct.pack("<IQ", 10, int(v)))
        for k, v in meta_f32.items():
            _wstr(f, k)
            f.write(struct.pack("<If", 6, float(v)))
        offs, acc = [], 0
        for t in tensors:
            offs.append(acc)
            acc += t.nbytes
            acc = (acc + align - 1) // align * align
        for t, off in zip(tensors, offs):
            _wstr(f, t.name)
            f.write(struct.pack("<I", len(t.ne)))
            for d in t.ne:
                f.write(struct.pack("<Q", int(d)))
            f.write(struct.pack("<IQ", t.ggml_type, off))
        pos = f.tell()
        f.write(b"\0" * ((align - pos % align) % align))
        for i, t in enumerate(tensors):
            n = 0
            for chunk in t.produce():
                f.write(chunk)
                n += len(chunk)
            if n != t.nbytes:
                raise ValueError(f"{t.name}: produced {n} bytes, expected {t.nbytes}")
            if i + 1 < len(tensors):
                f.write(b"\0" * ((align - n % align) % align))
    os.replace(tmp, path)
