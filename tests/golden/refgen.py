"""Seeded input generators restated from the reference's own XCTests.

These reproduce, value for value, the synthetic inputs Siliconed's tests build for this path, so
that the oracle and the CUDA path are checked on the very inputs the reference checks itself on:

* ``SplitMix`` -- the generator of DequantizeTests (Tests/SiliconedTests/DequantizeTests.swift:10-18),
  SplitMix64 (Steele, Lea, Flood 2014) with the test's seed 0x4D31_3432; ``codes`` and ``scales``
  restate its ``codes(_:)`` (:20-21) and ``scales(_:_:)`` (:23-42).
* ``XorShift`` -- the ``Random`` of Qwen3VLDecoderTests (Tests/SiliconedTests/Qwen3VLDecoderTests.swift:25-35),
  Marsaglia's xorshift64 (13, 7, 17) seeded ``seed * 0x9E3779B97F4A7C15 + 1``; ``int8_matrix`` restates
  its byte pool (:57-62), ``fillBytes`` (:90-102) and ``int8Matrix`` (:118-145).

Pure numpy; no part of the product or of the oracle is used here.
"""
from __future__ import annotations

import numpy as np

M64 = (1 << 64) - 1


class SplitMix:
    """DequantizeTests.swift:10-18."""

    def __init__(self, seed: int = 0x4D313432):
        self.state = seed & M64

    def next(self) -> int:
        self.state = (self.state + 0x9E3779B97F4A7C15) & M64
        z = self.state
        z = ((z ^ (z >> 30)) * 0xBF58476D1CE4E5B9) & M64
        z = ((z ^ (z >> 27)) * 0x94D049BB133111EB) & M64
        return z ^ (z >> 31)

    def codes(self, count: int) -> np.ndarray:
        """Every one of the 256 codes first, then truncated draws (DequantizeTests.swift:20-21)."""
        out = np.empty(count, np.uint8)
        n = min(count, 256)
        out[:n] = np.arange(n, dtype=np.uint8)
        for i in range(256, count):
            out[i] = self.next() & 0xFF
        return out

    def scales(self, count: int, kind: str):
        """(bytes, fp32 values) of ``count`` scales of ``kind`` in {"f16", "bf16", "f32"}:
        full fp32 mantissas, one negative (index 1) and one zero (index 2) (DequantizeTests.swift:23-42)."""
        base = np.float32(1.37e-9)
        xs = np.empty(count, np.float32)
        for i in range(count):
            x = np.float32(self.next() % 1_000_000 + 1) * base
            if i == 1:
                x = -x
            elif i == 2:
                x = np.float32(0)
            xs[i] = x
        if kind == "f16":
            h = xs.astype(np.float16)                       # Float16(x): nearest-even
            return h.view(np.uint8).copy(), h.astype(np.float32)
        if kind == "bf16":
            b = (xs.view(np.uint32) >> 16).astype(np.uint16)  # UInt16(x.bitPattern >> 16): truncation
            return b.view(np.uint8).copy(), (b.astype(np.uint32) << 16).view(np.float32)
        return xs.view(np.uint8).copy(), xs.copy()


class XorShift:
    """Qwen3VLDecoderTests.swift:25-35."""

    def __init__(self, seed: int):
        self.state = (seed * 0x9E3779B97F4A7C15 + 1) & M64

    def next(self) -> int:
        s = self.state
        s ^= (s << 13) & M64
        s ^= s >> 7
        s ^= (s << 17) & M64
        self.state = s
        return s

    def unit(self) -> np.float32:
        """Uniform in [-1, 1): Float(Int32(truncatingIfNeeded: next() >> 33)) / 2^30 - 1."""
        v = (self.next() >> 33) & 0xFFFFFFFF
        if v >= 1 << 31:
            v -= 1 << 32
        return np.float32(np.float32(v) / np.float32(1 << 30)) - np.float32(1)

    def floats(self, count: int, scale: float = 1.0) -> np.ndarray:
        sc = np.float32(scale)
        return np.array([self.unit() * sc for _ in range(count)], np.float32)


_POOL = None


def byte_pool() -> np.ndarray:
    """1 MiB of bytes ``UInt8(truncatingIfNeeded: next() >> 40)`` from XorShift(0x5EED) (:59-62)."""
    global _POOL
    if _POOL is None:
        r = XorShift(0x5EED)
        _POOL = np.array([(r.next() >> 40) & 0xFF for _ in range(1 << 20)], np.uint8)
    return _POOL


def fill_bytes(count: int, seed: int) -> np.ndarray:
    """Blocks of 4096 bytes copied from the pool at seeded offsets (:90-102)."""
    pool = byte_pool()
    r = XorShift(seed)
    out = np.empty(count, np.uint8)
    at = 0
    while at < count:
        frm = (r.next() >> 33) % (pool.size - 4096)
        n = min(4096, count - at)
        out[at:at + n] = pool[frm:frm + n]
        at += 4096
    return out


def int8_matrix(k: int, n: int, seed: int, kind: str = "f32"):
    """int8 [k, n] (the map's layout) and its per-column scales as the kernel reads them (:118-145).
    Returns (q int8 [k, n], scale bytes, scale fp32 values)."""
    q = fill_bytes(k * n, seed).view(np.int8).reshape(k, n)
    r = XorShift(seed ^ 0xABCDEF)
    nominal = np.float32(1) / (np.float32(64) * np.float32(np.sqrt(np.float32(k))))
    s = np.empty(n, np.float32)
    for c in range(n):
        s[c] = nominal * (np.float32(1.2) + r.unit() * np.float32(0.8))
    if kind == "bf16":
        b = (s.view(np.uint32) >> 16).astype(np.uint16)
        return q, b.view(np.uint8).copy(), (b.astype(np.uint32) << 16).view(np.float32)
    if kind == "f16":
        h = s.astype(np.float16)
        return q, h.view(np.uint8).copy(), h.astype(np.float32)
    return q, s.view(np.uint8).copy(), s.copy()
