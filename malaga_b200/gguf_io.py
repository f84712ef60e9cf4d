"""Minimal GGUF v3 writer and metadata reader.

The container format written by the reference's converter through candle's
``gguf_file::write`` (crates/malaga-core/src/convert.rs:311-317): a header, the
metadata key/values, the tensor infos (dims in GGML order, i.e. innermost
first), then the tensor data, each tensor aligned to 32 bytes.

The writer streams: tensor infos are planned first (shape + type fix the byte
size), then each tensor's bytes are produced by a callback and written in
order, so a multi-GB model never has to be held in memory.
"""
from __future__ import annotations

import struct
from dataclasses import dataclass
from typing import Callable, Iterable

import numpy as np

GGUF_MAGIC = 0x46554747
ALIGN = 32

# GGML tensor types used by the NLLB presets.
F32, F16, Q8_0, Q4_K, Q6_K = 0, 1, 8, 12, 14
TYPE_NAMES = {F32: "F32", F16: "F16", Q8_0: "Q8_0", Q4_K: "Q4_K", Q6_K: "Q6_K"}
BLOCK = {F32: (1, 4), F16: (1, 2), Q8_0: (32, 34), Q4_K: (256, 144), Q6_K: (256, 210)}

# GGUF metadata value types.
T_U8, T_I8, T_U16, T_I16, T_U32, T_I32, T_F32, T_BOOL, T_STR, T_ARR, T_U64, T_I64, T_F64 = range(13)


def row_bytes(ggml_type: int, n: int) -> int:
    blk, size = BLOCK[ggml_type]
    if n % blk:
        raise ValueError(f"row of {n} values is not a whole number of {TYPE_NAMES[ggml_type]} blocks")
    return n // blk * size


def tensor_bytes(ggml_type: int, shape: tuple[int, ...]) -> int:
    rows = int(np.prod(shape[:-1])) if len(shape) > 1 else 1
    return rows * row_bytes(ggml_type, shape[-1])


@dataclass
class U32:
    v: int


@dataclass
class Bool:
    v: bool


def _str(s: str) -> bytes:
    b = s.encode("utf-8")
    return struct.pack("<Q", len(b)) + b


def _value(v) -> bytes:
    if isinstance(v, U32):
        return struct.pack("<I", T_U32) + struct.pack("<I", v.v)
    if isinstance(v, Bool):
        return struct.pack("<I", T_BOOL) + struct.pack("<B", int(v.v))
    if isinstance(v, str):
        return struct.pack("<I", T_STR) + _str(v)
    if isinstance(v, list):  # arrays of u32 (shortlists)
        return struct.pack("<I", T_ARR) + struct.pack("<IQ", T_U32, len(v)) + struct.pack(f"<{len(v)}I", *v)
    raise TypeError(f"unsupported metadata value {v!r}")


@dataclass
class TensorPlan:
    name: str
    shape: tuple[int, ...]  # row-major, last dim innermost (the reference's Tensor dims)
    ggml_type: int
    produce: Callable[[], bytes | np.ndarray]


def write_gguf(path: str, metadata: Iterable[tuple[str, object]], tensors: list[TensorPlan]) -> None:
    metadata = list(metadata)
    head = bytearray()
    head += struct.pack("<IIQQ", GGUF_MAGIC, 3, len(tensors), len(metadata))
    for k, v in metadata:
        head += _str(k) + _value(v)
    offset = 0
    offsets = []
    for t in tensors:
        dims = list(reversed(t.shape))
        head += _str(t.name) + struct.pack("<I", len(dims)) + struct.pack(f"<{len(dims)}Q", *dims)
        head += struct.pack("<IQ", t.ggml_type, offset)
        offsets.append(offset)
        offset += tensor_bytes(t.ggml_type, t.shape)
        offset = (offset + ALIGN - 1) // ALIGN * ALIGN
    pad = (-len(head)) % ALIGN
    head += b"\0" * pad
    with open(path, "wb") as f:
        f.write(head)
        pos = 0
        for t, off in zip(tensors, offsets):
            if pos < off:
                f.write(b"\0" * (off - pos))
                pos = off
            data = t.produce()
            if isinstance(data, np.ndarray):
                data = data.tobytes()
            want = tensor_bytes(t.ggml_type, t.shape)
            if len(data) != want:
                raise ValueError(f"{t.name}: produced {len(data)} bytes, expected {want}")
            f.write(data)
            pos += len(data)


def read_metadata(path: str) -> tuple[dict, dict]:
    """Returns (metadata, tensor_infos) of a GGUF file; infos map name -> (shape, type, offset)."""
    with open(path, "rb") as f:
        buf = f.read(1 << 20)
        need = len(buf)
        while True:
            try:
                return _parse(buf)
            except (struct.error, IndexError):
                more = f.read(need)
                if not more:
                    raise
                buf += more
                need *= 2


def _parse(buf: bytes) -> tuple[dict, dict]:
    p = 0

    def rd(fmt):
        nonlocal p
        vals = struct.unpack_from(fmt, buf, p)
        p += struct.calcsize(fmt)
        return vals

    def rstr():
        nonlocal p
        (n,) = rd("<Q")
        s = buf[p : p + n].decode("utf-8")
        if p + n > len(buf):
            raise struct.error("truncated")
        p += n
        return s

    scalar = {T_U8: "<B", T_I8: "<b", T_U16: "<H", T_I16: "<h", T_U32: "<I", T_I32: "<i", T_F32: "<f",
              T_BOOL: "<B", T_U64: "<Q", T_I64: "<q", T_F64: "<d"}

    def rval(t):
        if t == T_STR:
            return rstr()
        if t == T_ARR:
            et, n = rd("<IQ")
            return [rval(et) for _ in range(n)]
        (v,) = rd(scalar[t])
        return bool(v) if t == T_BOOL else v

    magic, version, nt, nkv = rd("<IIQQ")
    if magic != GGUF_MAGIC:
        raise ValueError("not a GGUF file")
    meta = {}
    for _ in range(nkv):
        k = rstr()
        (t,) = rd("<I")
        meta[k] = rval(t)
    infos = {}
    for _ in range(nt):
        name = rstr()
        (nd,) = rd("<I")
        dims = rd(f"<{nd}Q")
        t, off = rd("<IQ")
        infos[name] = (tuple(reversed(dims)), t, off)
    return meta, infos
