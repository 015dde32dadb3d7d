"""Seeded synthetic workloads with the shapes and value distributions of the benchmark configs.

No dataset or checkpoint is involved anywhere on this path: every input is drawn here, from
numpy's PCG64 generator (``numpy.random.default_rng(seed)``), host side, in the published
nn.Linear layout [N out, K in].  Weights are registered with ``published_nk=True`` (the forge
transposes them to the map's [K, N]; the library does the same when it re-tiles).
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np


def to_bf16_bits(a: np.ndarray) -> np.ndarray:
    """fp32 -> bf16 bit patterns, nearest-even (finite inputs)."""
    u = np.ascontiguousarray(a, np.float32).view(np.uint32)
    return ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)


def to_e4m3_codes(a: np.ndarray) -> np.ndarray:
    """fp32 -> e4m3fn codes, nearest-even, clipped to +-448 (ml_dtypes' conversion)."""
    import ml_dtypes
    return np.clip(a, -448.0, 448.0).astype(ml_dtypes.float8_e4m3fn).view(np.uint8)


@dataclass
class LinearCase:
    name: str
    kind: int                 # 1 int8, 2 e4m3
    x: np.ndarray             # bf16 bits [M, K]
    codes_nk: np.ndarray      # uint8 [N, K] (published layout)
    scales: np.ndarray        # fp32 [N]
    bias: np.ndarray | None   # bf16 bits [N]

    @property
    def m(self): return self.x.shape[0]

    @property
    def k(self): return self.x.shape[1]

    @property
    def n(self): return self.codes_nk.shape[0]

    @property
    def flops(self) -> float: return 2.0 * self.m * self.k * self.n

    def bytes_moved(self, out_bytes: int = 2) -> float:
        """Algorithmic bytes of one product: x, weight codes, scales, bias, y."""
        b = self.m * self.k * 2 + self.n * self.k + self.n * 4 + self.m * self.n * out_bytes
        return float(b + (self.n * 2 if self.bias is not None else 0))


def config1(m: int = 4096, k: int = 3072, n: int = 3072, seed: int = 0) -> LinearCase:
    """Config 1: int8 weight-only linear, x ~ N(0,1) bf16, q uniform in [-127, 127],
    s = |N(0, 0.02)| / 127 per output, bias ~ N(0, 0.01) bf16."""
    g = np.random.default_rng(seed)
    x = to_bf16_bits(g.standard_normal((m, k), dtype=np.float32))
    q = g.integers(-127, 128, size=(n, k), dtype=np.int16).astype(np.int8).view(np.uint8)
    s = (np.abs(g.standard_normal(n, dtype=np.float32)) * np.float32(0.02) / np.float32(127)).astype(np.float32)
    b = to_bf16_bits(g.standard_normal(n, dtype=np.float32) * np.float32(0.01))
    return LinearCase("cfg1-int8", 1, x, q, s, b)


def config2(m: int = 4096, k: int = 3840, n: int = 10240, seed: int = 0) -> LinearCase:
    """Config 2: fp8 e4m3 weight-only linear, W = e4m3(clip(N(0,1), +-448)), s = |N(0, 0.02)| / 448, no bias."""
    g = np.random.default_rng(seed)
    x = to_bf16_bits(g.standard_normal((m, k), dtype=np.float32))
    q = to_e4m3_codes(g.standard_normal((n, k), dtype=np.float32))
    s = (np.abs(g.standard_normal(n, dtype=np.float32)) * np.float32(0.02) / np.float32(448)).astype(np.float32)
    return LinearCase("cfg2-e4m3", 2, x, q, s, None)


def encoder_prefill(m: int = 128, n: int = 9728, k: int = 2560, seed: int = 0) -> LinearCase:
    """A text encoder's prefill product (32 < M <= 128 rows, the single-CTA tensor-core GEMM's range): the
    gate / up shape of the Z-Image encoder's MLP as its published int8 checkpoint stores it ([9728, 2560],
    recorded in tests/golden/quant_fixture_pins.json), x ~ N(0,1) bf16, per-channel scales, no bias."""
    g = np.random.default_rng(seed)
    x = to_bf16_bits(g.standard_normal((m, k), dtype=np.float32))
    q = g.integers(-127, 128, size=(n, k), dtype=np.int16).astype(np.int8).view(np.uint8)
    s = (np.abs(g.standard_normal(n, dtype=np.float32)) * np.float32(0.02) / np.float32(127)).astype(np.float32)
    return LinearCase(f"encoder-prefill-m{m}-{n}x{k}", 1, x, q, s, None)


def config4(m: int, n: int, k: int, seed: int = 0) -> LinearCase:
    """Config 4: decode-shape GEMV, int8 per-channel weight [n out, k in], x ~ N(0,1) bf16, M <= 32."""
    g = np.random.default_rng(seed)
    x = to_bf16_bits(g.standard_normal((m, k), dtype=np.float32))
    q = g.integers(-127, 128, size=(n, k), dtype=np.int16).astype(np.int8).view(np.uint8)
    s = (np.abs(g.standard_normal(n, dtype=np.float32)) * np.float32(0.02) / np.float32(127)).astype(np.float32)
    return LinearCase(f"cfg4-gemv-m{m}-{n}x{k}", 1, x, q, s, None)
