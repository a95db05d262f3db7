"""Host-side packing of logical values into the device byte image (`Scalar::to_buf` / `load`,
furiosa-opt-std/src/scalar.rs:45-94,657-680): byte-multiple types are their little-endian bytes,
4-bit types pack two per byte with the low element in the low nibble, i5 / i9 stage in the i8 / i16
that backs them. bf16 values travel as their raw uint16 bit patterns.
"""
from __future__ import annotations

import numpy as np

NP = {"i8": np.int8, "i16": np.int16, "i32": np.int32, "bf16": np.uint16, "f32": np.float32, "i5": np.int8,
      "i9": np.int16, "f8e4m3": np.uint8, "f8e5m2": np.uint8, "i4": np.int8, "f4e2m1": np.uint8}
BITS = {"i8": 8, "i16": 16, "i32": 32, "bf16": 16, "f32": 32, "i4": 4, "f8e4m3": 8, "f8e5m2": 8, "f4e2m1": 4,
        "i5": 8, "i9": 16}


def nbytes(dtype: str, n: int) -> int:
    bits = BITS[dtype] * n
    if bits % 8:
        raise ValueError(f"a sub-byte element count must be byte-aligned (got {n} elements at {BITS[dtype]} bits)")
    return bits // 8


def f32_to_bf16_bits(x) -> np.ndarray:
    """Plain IEEE round-to-nearest-even f32 -> bf16 bits (`half::bf16::from_f32`)."""
    u = np.asarray(x, dtype=np.float32).view(np.uint32).astype(np.uint64)
    nan = (u & 0x7FFFFFFF) > 0x7F800000
    hi = (u >> 16) & 0xFFFF
    up = ((u & 0x8000) != 0) & ((u & 0x17FFF) != 0)
    out = np.where(nan, hi | 0x40, hi + up.astype(np.uint64))
    return (out & 0xFFFF).astype(np.uint16)


def bf16_bits_to_f32(b) -> np.ndarray:
    return (np.asarray(b, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


def to_bytes(values, dtype: str) -> bytes:
    v = np.asarray(values)
    if dtype in ("i4", "f4e2m1"):
        codes = (v.astype(np.int64) & 0xF).astype(np.uint8)
        if codes.size % 2:
            raise ValueError("a sub-byte element count must be byte-aligned")
        return (codes[0::2] | (codes[1::2] << 4)).astype(np.uint8).tobytes()
    if dtype == "bf16" and v.dtype != np.uint16:
        v = f32_to_bf16_bits(v.astype(np.float32))
    return np.ascontiguousarray(v.astype(NP[dtype])).tobytes()


def from_bytes(buf: bytes, dtype: str, n: int) -> np.ndarray:
    raw = np.frombuffer(buf, dtype=np.uint8)
    if dtype in ("i4", "f4e2m1"):
        lo, hi = raw & 0xF, raw >> 4
        codes = np.empty(raw.size * 2, dtype=np.uint8)
        codes[0::2], codes[1::2] = lo, hi
        codes = codes[:n]
        if dtype == "i4":
            return ((codes.astype(np.int8) << 4) >> 4).astype(np.int8)
        return codes
    return np.frombuffer(buf, dtype=NP[dtype], count=n).copy()
