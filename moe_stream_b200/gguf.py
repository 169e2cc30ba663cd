"""Minimal GGUF v3 writer and reader for native quantized block layouts.

The reader follows the header parse of moe-stream-core/src/gguf/reader.rs:259-368
(magic, version 2..3, metadata key/values, tensor infos, data start aligned to
``general.alignment`` or 32) and the per-expert slice arithmetic of
reader.rs:394-444 (expert e of a stacked ``[n_exp, rows, cols]`` tensor starts at
``data_offset + e * raw_size(rows * cols)``).  Block sizes follow
``GgmlQuantType::block_info`` (reader.rs:99-127).

The writer exists so that tests and the benchmark can build seeded synthetic
models; it stores every tensor in its native GGML block layout, untouched.
"""
from __future__ import annotations

import mmap
import struct
from dataclasses import dataclass, field
from typing import Dict, List, Tuple, Union

import numpy as np

GGUF_MAGIC = 0x46554747  # "GGUF" little-endian

# GGML type ids (reader.rs:38-65)
F32, F16, Q4_0, Q4_1, Q5_0, Q5_1, Q8_0, Q8_1 = 0, 1, 2, 3, 6, 7, 8, 9
Q2_K, Q3_K, Q4_K, Q5_K, Q6_K, Q8_K, BF16, MXFP4 = 10, 11, 12, 13, 14, 15, 30, 39

QTYPE_NAMES = {F32: "F32", F16: "F16", Q8_0: "Q8_0", Q4_K: "Q4_K", Q6_K: "Q6_K",
               MXFP4: "MXFP4", BF16: "BF16", Q4_0: "Q4_0", Q5_0: "Q5_0"}

# (block_bytes, block_elements) as in GgmlQuantType::block_info / element_size
BLOCK_INFO = {
    F32: (4, 1), F16: (2, 1), BF16: (2, 1),
    Q4_0: (18, 32), Q4_1: (20, 32), Q5_0: (22, 32), Q5_1: (24, 32),
    Q8_0: (34, 32), Q8_1: (36, 32),
    Q2_K: (84, 256), Q3_K: (110, 256), Q4_K: (144, 256), Q5_K: (176, 256),
    Q6_K: (210, 256), MXFP4: (17, 32),
}

# metadata value types
T_U8, T_I8, T_U16, T_I16, T_U32, T_I32, T_F32, T_BOOL, T_STR, T_ARR, T_U64, T_I64, T_F64 = range(13)
_SCALAR_FMT = {T_U8: "<B", T_I8: "<b", T_U16: "<H", T_I16: "<h", T_U32: "<I", T_I32: "<i",
               T_F32: "<f", T_BOOL: "<?", T_U64: "<Q", T_I64: "<q", T_F64: "<d"}


def raw_size(qtype: int, n_elements: int) -> int:
    """Bytes for ``n_elements`` of ``qtype`` (reader.rs ``raw_size``)."""
    bb, be = BLOCK_INFO[qtype]
    return ((n_elements + be - 1) // be) * bb


def row_bytes(qtype: int, cols: int) -> int:
    bb, be = BLOCK_INFO[qtype]
    if cols % be:
        raise ValueError(f"cols {cols} not a multiple of block size {be} for {QTYPE_NAMES.get(qtype, qtype)}")
    return cols // be * bb


@dataclass
class Tensor:
    name: str
    qtype: int
    shape: Tuple[int, ...]          # PyTorch order, e.g. [n_exp, rows, cols]
    data: np.ndarray                # raw bytes (uint8) or typed array for F32/F16

    @property
    def nbytes(self) -> int:
        return raw_size(self.qtype, int(np.prod(self.shape)))

    def raw(self) -> np.ndarray:
        b = np.ascontiguousarray(self.data).view(np.uint8).reshape(-1)
        if b.size != self.nbytes:
            raise ValueError(f"{self.name}: {b.size} bytes, expected {self.nbytes}")
        return b


MetaValue = Union[int, float, str, bool, List[int], List[float], List[str]]


@dataclass
class Model:
    metadata: Dict[str, Tuple[int, MetaValue]] = field(default_factory=dict)
    tensors: Dict[str, Tensor] = field(default_factory=dict)

    def add_meta(self, key: str, vtype: int, value: MetaValue) -> None:
        self.metadata[key] = (vtype, value)

    def add(self, name: str, qtype: int, shape, data) -> None:
        t = Tensor(name, qtype, tuple(int(s) for s in shape), data)
        t.raw()  # validate size
        self.tensors[name] = t


def _w_str(f, s: str) -> None:
    b = s.encode("utf-8")
    f.write(struct.pack("<Q", len(b)))
    f.write(b)


def _w_value(f, vtype: int, v) -> None:
    if vtype == T_STR:
        _w_str(f, v)
    elif vtype == T_ARR:
        etype, items = v
        f.write(struct.pack("<IQ", etype, len(items)))
        for it in items:
            _w_value(f, etype, it)
    else:
        f.write(struct.pack(_SCALAR_FMT[vtype], v))


def write_gguf(path: str, model: Model, alignment: int = 32) -> None:
    """Write ``model`` as a GGUF v3 file with every tensor in native block layout."""
    names = list(model.tensors)
    offsets, off = [], 0
    for n in names:
        off = (off + alignment - 1) // alignment * alignment
        offsets.append(off)
        off += model.tensors[n].nbytes
    with open(path, "wb") as f:
        f.write(struct.pack("<IIQQ", GGUF_MAGIC, 3, len(names), len(model.metadata)))
        for k, (vt, v) in model.metadata.items():
            _w_str(f, k)
            f.write(struct.pack("<I", vt))
            _w_value(f, vt, v)
        for n, o in zip(names, offsets):
            t = model.tensors[n]
            _w_str(f, n)
            dims = list(reversed(t.shape))  # GGUF order: innermost first
            f.write(struct.pack("<I", len(dims)))
            for d in dims:
                f.write(struct.pack("<Q", d))
            f.write(struct.pack("<IQ", t.qtype, o))
        pos = f.tell()
        start = (pos + alignment - 1) // alignment * alignment
        f.write(b"\0" * (start - pos))
        for n, o in zip(names, offsets):
            cur = f.tell() - start
            f.write(b"\0" * (o - cur))
            f.write(model.tensors[n].raw().tobytes())


class _Buf:
    def __init__(self, mm):
        self.mm, self.pos = mm, 0

    def read(self, fmt: str):
        v = struct.unpack_from(fmt, self.mm, self.pos)
        self.pos += struct.calcsize(fmt)
        return v[0] if len(v) == 1 else v

    def string(self) -> str:
        n = self.read("<Q")
        s = bytes(self.mm[self.pos:self.pos + n]).decode("utf-8")
        self.pos += n
        return s

    def value(self, vtype: int):
        if vtype == T_STR:
            return self.string()
        if vtype == T_ARR:
            et, n = self.read("<I"), self.read("<Q")
            return [self.value(et) for _ in range(n)]
        return self.read(_SCALAR_FMT[vtype])


@dataclass
class TensorInfo:
    name: str
    qtype: int
    shape: Tuple[int, ...]
    offset: int   # absolute file offset

    @property
    def nbytes(self) -> int:
        return raw_size(self.qtype, int(np.prod(self.shape)))


class GgufFile:
    """Read-only mmap view (reader.rs ``GgufReader::open`` / ``tensor_data``)."""

    def __init__(self, path: str):
        self._f = open(path, "rb")
        self.mm = mmap.mmap(self._f.fileno(), 0, access=mmap.ACCESS_READ)
        b = _Buf(self.mm)
        if b.read("<I") != GGUF_MAGIC:
            raise ValueError("invalid GGUF magic")
        ver = b.read("<I")
        if ver not in (2, 3):
            raise ValueError(f"unsupported GGUF version {ver}")
        nt, nm = b.read("<Q"), b.read("<Q")
        self.metadata: Dict[str, MetaValue] = {}
        for _ in range(nm):
            k = b.string()
            self.metadata[k] = b.value(b.read("<I"))
        infos = []
        for _ in range(nt):
            name = b.string()
            nd = b.read("<I")
            dims = [b.read("<Q") for _ in range(nd)]
            qt, off = b.read("<I"), b.read("<Q")
            infos.append((name, qt, tuple(reversed(dims)), off))
        align = int(self.metadata.get("general.alignment", 32))
        start = (b.pos + align - 1) // align * align
        self.tensors = {n: TensorInfo(n, qt, shp, start + off) for n, qt, shp, off in infos}

    def data(self, name: str) -> np.ndarray:
        t = self.tensors[name]
        end = t.offset + t.nbytes
        if end > len(self.mm):
            raise ValueError(f"{name}: out of bounds")
        return np.frombuffer(self.mm, dtype=np.uint8, count=t.nbytes, offset=t.offset)

    def expert_slice(self, name: str, e: int) -> np.ndarray:
        t = self.tensors[name]
        if e >= t.shape[0]:
            raise IndexError(f"expert {e} out of range {t.shape[0]}")
        per = raw_size(t.qtype, int(np.prod(t.shape[1:])))
        return np.frombuffer(self.mm, dtype=np.uint8, count=per, offset=t.offset + e * per)

    def close(self) -> None:
        try:
            self.mm.close()
        except BufferError:   # numpy views still alive; the map is released with them
            pass
        self._f.close()
