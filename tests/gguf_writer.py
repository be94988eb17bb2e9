"""A small GGUF (v3) writer for the GGUF ingestion tests (test
infrastructure): builds files with chosen metadata, tensors and alignment,
including deliberately malformed ones.  The layout follows the GGUF v3
format as the reference's reader parses it (src/gguf.cc:396-575)."""
from __future__ import annotations

import struct

import numpy as np

# GGUF value types
U8, I8, U16, I16, U32, I32, F32, BOOL, STRING, ARRAY, U64, I64, F64 = range(13)
_SCALAR = {U8: "<B", I8: "<b", U16: "<H", I16: "<h", U32: "<I", I32: "<i", F32: "<f", BOOL: "<B",
           U64: "<Q", I64: "<q", F64: "<d"}


def _str(s: str | bytes) -> bytes:
    b = s.encode() if isinstance(s, str) else s
    return struct.pack("<Q", len(b)) + b


def _value(vtype: int, v) -> bytes:
    if vtype == STRING:
        return _str(v)
    if vtype == ARRAY:
        et, items = v
        return struct.pack("<IQ", et, len(items)) + b"".join(_value(et, it) for it in items)
    return struct.pack(_SCALAR[vtype], v)


def build(metadata, tensors, alignment=None, version=3, magic=b"GGUF", pad_data=True, truncate=0):
    """metadata: [(key, vtype, value)]; tensors: [(name, dims (fastest
    first), ggml type, data bytes)].  Tensor data is laid out in order, each
    at a multiple of the alignment.  Returns the file bytes."""
    align = alignment if alignment and alignment & (alignment - 1) == 0 else 32  # layout (value as given)
    meta = list(metadata)
    if alignment is not None:
        meta = [("general.alignment", U32, alignment)] + meta
    head = magic + struct.pack("<IQQ", version, len(tensors), len(meta))
    for key, vt, v in meta:
        head += _str(key) + struct.pack("<I", vt) + _value(vt, v)
    offsets, off = [], 0
    for _, _, _, data in tensors:
        offsets.append(off)
        off += len(data)
        off += (-off) % align
    for (name, dims, gtype, _), o in zip(tensors, offsets):
        head += _str(name) + struct.pack("<I", len(dims)) + b"".join(struct.pack("<Q", d) for d in dims)
        head += struct.pack("<IQ", gtype, o)
    head += b"\0" * ((-len(head)) % align)
    body = bytearray()
    for (_, _, _, data), o in zip(tensors, offsets):
        body += b"\0" * (o - len(body))
        body += data
    if pad_data:
        body += b"\0" * ((-len(body)) % align)
    out = bytes(head + body)
    return out[:len(out) - truncate] if truncate else out


def quantized(oracle, fmt: str, out_f: int, in_f: int, seed: int, synth) -> bytes:
    """Blocks of a seeded N(0, 0.02) [out, in] matrix (the reference's
    quantizers, through the oracle)."""
    w = synth.normal((out_f, in_f), seed=seed, std=0.02)
    return np.ascontiguousarray(oracle.quantize(fmt, w)).tobytes()
