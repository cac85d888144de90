"""Minimal GGUF v3 writer for tests (test infrastructure): metadata scalars,
strings and arrays, and tensors given as raw block bytes with their GGML
type. Layout per the GGUF specification: header, key/value pairs, tensor
table, data section aligned to ``general.alignment`` (32)."""

from __future__ import annotations

import struct

import numpy as np

ALIGN = 32


def _s(x: str) -> bytes:
    b = x.encode("utf-8")
    return struct.pack("<Q", len(b)) + b


def _val(v):
    if isinstance(v, bool):
        return struct.pack("<I", 7) + struct.pack("<?", v)
    if isinstance(v, int):
        return struct.pack("<I", 4) + struct.pack("<I", v)   # uint32
    if isinstance(v, float):
        return struct.pack("<I", 6) + struct.pack("<f", v)
    if isinstance(v, str):
        return struct.pack("<I", 8) + _s(v)
    if isinstance(v, list):  # array of uint32
        return struct.pack("<I", 9) + struct.pack("<IQ", 4, len(v)) + b"".join(struct.pack("<I", x) for x in v)
    raise TypeError(type(v))


def write_gguf(path, metadata: dict, tensors: list) -> None:
    """tensors: list of (name, dims_innermost_first, ggml_type, raw_bytes)."""
    head = b"GGUF" + struct.pack("<IQQ", 3, len(tensors), len(metadata))
    kv = b"".join(_s(k) + _val(v) for k, v in metadata.items())
    infos, data, off = b"", b"", 0
    for name, dims, gtype, raw in tensors:
        infos += _s(name) + struct.pack("<I", len(dims)) + struct.pack(f"<{len(dims)}Q", *dims)
        infos += struct.pack("<IQ", gtype, off)
        pad = (-len(raw)) % ALIGN
        data += bytes(raw) + b"\0" * pad
        off += len(raw) + pad
    body = head + kv + infos
    body += b"\0" * ((-len(body)) % ALIGN)
    with open(path, "wb") as f:
        f.write(body + data)


def random_q4_0(rng: np.random.Generator, rows: int, K: int, scale: float = 0.01) -> bytes:
    nb = rows * K // 32
    d = (rng.standard_normal(nb) * scale).astype(np.float16)
    qs = rng.integers(0, 256, size=(nb, 16), dtype=np.uint8)
    blk = np.concatenate([d.view(np.uint8).reshape(nb, 2), qs], axis=1)
    return blk.tobytes()


def random_q4_k(rng: np.random.Generator, rows: int, K: int, scale: float = 2e-3) -> bytes:
    nb = rows * K // 256
    d = (np.abs(rng.standard_normal(nb)) * scale).astype(np.float16)
    dmin = (np.abs(rng.standard_normal(nb)) * scale).astype(np.float16)
    sc = rng.integers(0, 256, size=(nb, 12), dtype=np.uint8)
    qs = rng.integers(0, 256, size=(nb, 128), dtype=np.uint8)
    blk = np.concatenate([d.view(np.uint8).reshape(nb, 2), dmin.view(np.uint8).reshape(nb, 2), sc, qs], axis=1)
    return blk.tobytes()
