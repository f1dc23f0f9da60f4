"""GGUF model files: reader (and a writer for synthetic test files).

The container format ggml-based applications (llama.cpp, Ollama) load their
quantised weights from, written here from its published description
(version 3, little endian):

    header   : magic "GGUF" (u32), version (u32), tensor count (u64),
               metadata entry count (u64)
    metadata : key (string), value type (u32), value
    tensors  : name (string), n_dims (u32), dims (u64 each, innermost
               first), ggml type (u32), offset (u64, from the data section)
    data     : starts at the first multiple of `general.alignment` (default
               32) after the tensor table; each tensor at its offset

Strings are a u64 byte length and UTF-8 bytes; arrays a u32 element type, a
u64 count and the elements.  A weight of ggml shape [ne0, ne1] (ne0 = K, the
innermost, contiguous dimension) is ne1 rows of ne0 values, i.e. the N x K
row-per-output-channel layout the kernels take, block-quantised along K.

The reader memory-maps the file and hands out numpy views of tensor bytes;
no reference code exists for this (the reference only sketches a GGUF-driven
runner in its notes), so the format follows the public specification.
"""
from __future__ import annotations

import mmap
import struct
from dataclasses import dataclass, field
from pathlib import Path

import numpy as np

from . import synth as S

MAGIC = 0x46554747  # "GGUF" little endian
DEFAULT_ALIGNMENT = 32

# metadata value types
U8, I8, U16, I16, U32, I32, F32, BOOL, STRING, ARRAY, U64, I64, F64 = range(13)
_SCALAR = {U8: "<B", I8: "<b", U16: "<H", I16: "<h", U32: "<I", I32: "<i", F32: "<f", BOOL: "<?", U64: "<Q",
           I64: "<q", F64: "<d"}

# ggml tensor types used here -> (this library's VKF_DEQUANT_* code or a
# plain dtype, values per block, bytes per block)
GGML_F32, GGML_F16, GGML_Q4_0, GGML_Q4_1, GGML_Q5_0, GGML_Q8_0, GGML_Q8_1 = 0, 1, 2, 3, 6, 8, 9
GGML_Q4_K, GGML_Q5_K, GGML_Q6_K = 12, 13, 14
GGML_TO_VKF = {GGML_Q4_0: S.Q4_0, GGML_Q4_1: S.Q4_1, GGML_Q5_0: S.Q5_0, GGML_Q8_0: S.Q8_0, GGML_Q8_1: S.Q8_1,
               GGML_Q4_K: S.Q4_K, GGML_Q5_K: S.Q5_K, GGML_Q6_K: S.Q6_K}
VKF_TO_GGML = {v: k for k, v in GGML_TO_VKF.items()}


def type_size(ggml_type: int) -> tuple[int, int]:
    """(values per block, bytes per block) of a ggml tensor type."""
    if ggml_type == GGML_F32:
        return 1, 4
    if ggml_type == GGML_F16:
        return 1, 2
    if ggml_type in GGML_TO_VKF:
        q = GGML_TO_VKF[ggml_type]
        return S.BLOCK_VALUES[q], S.BLOCK_BYTES[q]
    raise ValueError(f"ggml type {ggml_type} not supported")


@dataclass
class TensorInfo:
    name: str
    dims: tuple            # innermost first (ne0, ne1, ...)
    ggml_type: int
    offset: int            # from the start of the data section

    @property
    def n_values(self) -> int:
        return int(np.prod(self.dims, dtype=np.int64))

    @property
    def nbytes(self) -> int:
        qk, bb = type_size(self.ggml_type)
        if self.dims[0] % qk:
            raise ValueError(f"{self.name}: row of {self.dims[0]} values is not whole blocks of {qk}")
        return self.n_values // qk * bb


class _Reader:
    def __init__(self, buf):
        self.b, self.p = buf, 0

    def take(self, fmt):
        v = struct.unpack_from(fmt, self.b, self.p)[0]
        self.p += struct.calcsize(fmt)
        return v

    def string(self) -> str:
        n = self.take("<Q")
        s = bytes(self.b[self.p:self.p + n]).decode("utf-8")
        self.p += n
        return s

    def value(self, t):
        if t in _SCALAR:
            return self.take(_SCALAR[t])
        if t == STRING:
            return self.string()
        if t == ARRAY:
            et, n = self.take("<I"), self.take("<Q")
            return [self.value(et) for _ in range(n)]
        raise ValueError(f"unknown GGUF value type {t}")


@dataclass
class GGUFFile:
    path: Path
    version: int
    metadata: dict
    tensors: dict = field(default_factory=dict)   # name -> TensorInfo
    data_offset: int = 0
    _mm: object = None

    def tensor_bytes(self, name: str) -> np.ndarray:
        """The tensor's bytes (a read-only view into the mapped file)."""
        t = self.tensors[name]
        start = self.data_offset + t.offset
        return np.frombuffer(self._mm, np.uint8, t.nbytes, start)

    def weight(self, name: str):
        """(VKF_DEQUANT_* code or "f32"/"f16", K, N, bytes [N x row bytes])."""
        t = self.tensors[name]
        if len(t.dims) != 2:
            raise ValueError(f"{name}: not a matrix ({t.dims})")
        K, N = int(t.dims[0]), int(t.dims[1])
        kind = GGML_TO_VKF.get(t.ggml_type, {GGML_F32: "f32", GGML_F16: "f16"}.get(t.ggml_type))
        return kind, K, N, self.tensor_bytes(name).reshape(N, -1)

    def close(self):
        """Unmaps the file; while views from tensor_bytes are alive the
        mapping stays until they are gone."""
        if self._mm is not None:
            try:
                self._mm.close()
            except BufferError:
                pass
            self._mm = None


def read(path) -> GGUFFile:
    path = Path(path)
    f = open(path, "rb")
    mm = mmap.mmap(f.fileno(), 0, access=mmap.ACCESS_READ)
    f.close()
    r = _Reader(mm)
    if r.take("<I") != MAGIC:
        mm.close()
        raise ValueError(f"{path}: not a GGUF file")
    version = r.take("<I")
    if version not in (2, 3):
        mm.close()
        raise ValueError(f"{path}: GGUF version {version} not supported")
    n_tensors, n_kv = r.take("<Q"), r.take("<Q")
    meta = {}
    for _ in range(n_kv):
        k = r.string()
        meta[k] = r.value(r.take("<I"))
    tensors = {}
    for _ in range(n_tensors):
        name = r.string()
        nd = r.take("<I")
        dims = tuple(r.take("<Q") for _ in range(nd))
        tensors[name] = TensorInfo(name, dims, r.take("<I"), r.take("<Q"))
    align = int(meta.get("general.alignment", DEFAULT_ALIGNMENT))
    data = (r.p + align - 1) // align * align
    g = GGUFFile(path, version, meta, tensors, data, mm)
    for t in tensors.values():
        if t.offset % align or data + t.offset + t.nbytes > len(mm):
            g.close()
            raise ValueError(f"{path}: tensor {t.name} outside the file or misaligned")
    return g


def _w_string(out: bytearray, s: str):
    b = s.encode("utf-8")
    out += struct.pack("<Q", len(b)) + b


def _w_value(out: bytearray, v):
    if isinstance(v, bool):
        out += struct.pack("<I?", BOOL, v)
    elif isinstance(v, int):
        out += struct.pack("<Iq", I64, v) if v < 0 else struct.pack("<IQ", U64, v) if v >= 2 ** 32 else \
            struct.pack("<II", U32, v)
    elif isinstance(v, float):
        out += struct.pack("<If", F32, v)
    elif isinstance(v, str):
        out += struct.pack("<I", STRING)
        _w_string(out, v)
    elif isinstance(v, (list, tuple)):
        if not v:
            out += struct.pack("<IIQ", ARRAY, U32, 0)
            return
        et = STRING if isinstance(v[0], str) else F32 if isinstance(v[0], float) else I32
        out += struct.pack("<IIQ", ARRAY, et, len(v))
        for e in v:
            if et == STRING:
                _w_string(out, e)
            else:
                out += struct.pack(_SCALAR[et], e)
    else:
        raise TypeError(f"metadata value {v!r}")


def write(path, metadata: dict, tensors: list, alignment: int = DEFAULT_ALIGNMENT) -> None:
    """Writes a GGUF v3 file.  tensors: (name, dims innermost first, ggml
    type, bytes) in file order."""
    meta = dict(metadata)
    if alignment != DEFAULT_ALIGNMENT:
        meta["general.alignment"] = alignment
    out = bytearray(struct.pack("<IIQQ", MAGIC, 3, len(tensors), len(meta)))
    for k, v in meta.items():
        _w_string(out, k)
        _w_value(out, v)
    off = 0
    for name, dims, gt, data in tensors:
        _w_string(out, name)
        out += struct.pack("<I", len(dims)) + b"".join(struct.pack("<Q", d) for d in dims)
        out += struct.pack("<IQ", gt, off)
        off += (len(memoryview(data).cast("B")) + alignment - 1) // alignment * alignment
    out += b"\0" * ((-len(out)) % alignment)
    with open(path, "wb") as f:
        f.write(out)
        for _, _, _, data in tensors:
            b = memoryview(np.ascontiguousarray(data)).cast("B")
            f.write(b)
            f.write(b"\0" * ((-len(b)) % alignment))
