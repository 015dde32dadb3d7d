"""CPU oracle for the quantized-linear path -- TEST INFRASTRUCTURE ONLY.

A ctypes wrapper over ``oracle/liboracle.so`` (built from ``oracle/oracle.c`` by
``oracle/Makefile``), the plain-C restatement of Siliconed's CPU arithmetic for the int8 / fp8
weight-only linear:

* ``dequantize``      -- ``Widen.dequantize`` (Sources/Siliconed/Widen.swift:129-271):
                         ``float(q) * s``, one rounded fp32 multiply, no FMA.
* ``e4m3_table``      -- ``Numerics.e4m3`` (Sources/Siliconed/Forge/Numerics.swift:49-55).
* ``f32_to_bf16``     -- the bf16 rounding rule (Sources/Siliconed/TensorGEMMBF16.swift:43-47).
* ``linear_int8``     -- ``linear_int8`` + ``scale_columns`` (Sources/Siliconed/TensorGEMM.swift:125-179)
                         then the bias (Sources/Siliconed/DiT.swift:410-413).
* ``linear_widened``  -- the widened / fp8 route (Sources/Siliconed/WeightProducts.swift:995-1001,
                         Sources/Siliconed/GEMM.swift:297-345).
* ``linear_fp64``     -- the fp64 witness (Sources/Siliconed/DiagnosticProbes.swift:86-94).
* ``gemv_int8_splits``-- the decode GEMV's split partials (Sources/Siliconed/DecodeKernels.swift:67-109).

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU legs may import this package,
and only as the checker or the timed CPU baseline.  The product library never calls it.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "liboracle.so")

INT8, E4M3 = 1, 2
SCALE_NONE, SCALE_F32, SCALE_BF16, SCALE_F16 = 0, 1, 2, 3
LAYOUT_TENSOR, LAYOUT_COLUMNS, LAYOUT_BLOCKS, LAYOUT_ROWS = 0, 1, 2, 3

_lib = None


def build(force: bool = False) -> str:
    """Compiles the oracle with its Makefile (gcc, -ffp-contract=off, OpenMP)."""
    src = os.path.join(HERE, "oracle.c")
    if force or not os.path.exists(LIB_PATH) or os.path.getmtime(LIB_PATH) < os.path.getmtime(src):
        subprocess.run(["make", "-s", "-C", HERE], check=True)
    return LIB_PATH


def lib() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        build()
        L = ctypes.CDLL(LIB_PATH)
        P, I64, I = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int
        L.orc_e4m3_table.argtypes = [P]
        L.orc_f32_to_bf16_array.argtypes = [P, P, I64]
        L.orc_dequantize.argtypes = [P, I, I64, P, I, I, I64, I64, I64, P]
        L.orc_linear_int8.argtypes = [P, I64, I64, I64, P, P, P, P, P]
        L.orc_linear_widened.argtypes = [P, I64, I64, I64, P, P, P, P]
        L.orc_linear_fp64.argtypes = [P, I64, I64, I64, P, P, P]
        L.orc_gemv_int8_splits.argtypes = [P, I64, I64, P, P, I64, P, P]
        L.orc_set_threads.argtypes = [I]
        L.orc_rotate_groups_bf16.argtypes = [P, I64, I64, I, P]
        L.orc_dequantize_rotated.argtypes = [P, I64, I64, I, P, P]
        L.orc_w8a8_quantize.argtypes = [P, I64, I64, I, P, P]
        L.orc_linear_w8a8.argtypes = [P, P, I64, I64, I64, P, P, P, P, P]
        L.orc_max_threads.restype = I
        _lib = L
    return _lib


def _p(a):
    return None if a is None else a.ctypes.data_as(ctypes.c_void_p)


def set_threads(n: int) -> None:
    lib().orc_set_threads(int(n))


def max_threads() -> int:
    return int(lib().orc_max_threads())


def e4m3_table() -> np.ndarray:
    out = np.empty(256, np.float32)
    lib().orc_e4m3_table(_p(out))
    return out


def f32_to_bf16(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, np.float32)
    out = np.empty(x.shape, np.uint16)
    lib().orc_f32_to_bf16_array(_p(x), _p(out), x.size)
    return out


def bf16_to_f32(b: np.ndarray) -> np.ndarray:
    return (np.ascontiguousarray(b, np.uint16).astype(np.uint32) << 16).view(np.float32)


def dequantize(values: np.ndarray, kind: int, scales: np.ndarray | None, scale_dtype: int,
               layout: int, width: int = 1, block: int = 1, first_row: int = 0,
               count: int | None = None) -> np.ndarray:
    """``Widen.dequantize``: fp32 ``float(q) * s`` for ``count`` values (default: all of ``values``)."""
    v = np.ascontiguousarray(values).view(np.uint8).reshape(-1)
    n = v.size if count is None else int(count)
    out = np.empty(n, np.float32)
    s = None if scales is None else np.ascontiguousarray(scales)
    lib().orc_dequantize(_p(v), kind, n, _p(s), scale_dtype if s is not None else SCALE_NONE,
                         layout, width, block, first_row, _p(out))
    return out


def linear_int8(x_bf16: np.ndarray, q_kn: np.ndarray, s: np.ndarray, bias_bf16: np.ndarray | None = None):
    """Native int8 route: returns (c fp32 [m, n], y bf16 [m, n])."""
    x = np.ascontiguousarray(x_bf16, np.uint16)
    q = np.ascontiguousarray(q_kn, np.int8)
    m, k = x.shape
    k2, n = q.shape
    assert k == k2
    s = np.ascontiguousarray(s, np.float32)
    b = None if bias_bf16 is None else np.ascontiguousarray(bias_bf16, np.uint16)
    c = np.empty((m, n), np.float32)
    y = np.empty((m, n), np.uint16)
    lib().orc_linear_int8(_p(x), m, k, n, _p(q), _p(s), _p(b), _p(c), _p(y))
    return c, y


def linear_widened(x_bf16: np.ndarray, w_kn: np.ndarray, bias_bf16: np.ndarray | None = None):
    """Widened route on an fp32 weight [k, n]: returns (c fp32, y bf16)."""
    x = np.ascontiguousarray(x_bf16, np.uint16)
    w = np.ascontiguousarray(w_kn, np.float32)
    m, k = x.shape
    n = w.shape[1]
    b = None if bias_bf16 is None else np.ascontiguousarray(bias_bf16, np.uint16)
    c = np.empty((m, n), np.float32)
    y = np.empty((m, n), np.uint16)
    lib().orc_linear_widened(_p(x), m, k, n, _p(w), _p(b), _p(c), _p(y))
    return c, y


def linear_fp64(x_bf16: np.ndarray, w_kn: np.ndarray, bias_bf16: np.ndarray | None = None) -> np.ndarray:
    x = np.ascontiguousarray(x_bf16, np.uint16)
    w = np.ascontiguousarray(w_kn, np.float32)
    m, k = x.shape
    n = w.shape[1]
    b = None if bias_bf16 is None else np.ascontiguousarray(bias_bf16, np.uint16)
    c = np.empty((m, n), np.float64)
    lib().orc_linear_fp64(_p(x), m, k, n, _p(w), _p(b), _p(c))
    return c


def gemv_int8_splits(x: np.ndarray, q_kn: np.ndarray, s: np.ndarray, splits: int):
    x = np.ascontiguousarray(x, np.float32).reshape(-1)
    q = np.ascontiguousarray(q_kn, np.int8)
    k, n = q.shape
    s = np.ascontiguousarray(s, np.float32)
    parts = np.empty((splits, n), np.float32)
    out = np.empty(n, np.float32)
    lib().orc_gemv_int8_splits(_p(x), k, n, _p(q), _p(s), splits, _p(parts), _p(out))
    return parts, out


def rotate_groups_bf16(x_bf16: np.ndarray, group: int) -> np.ndarray:
    """convrot on the activation (rotate_groups, TensorGEMM.swift:183-201): bf16 [m, k] -> bf16 [m, k]."""
    x = np.ascontiguousarray(x_bf16, np.uint16)
    m, k = x.shape
    assert k % group == 0
    out = np.empty_like(x)
    lib().orc_rotate_groups_bf16(_p(x), m, k, group, _p(out))
    return out


def dequantize_rotated(q_kn: np.ndarray, group: int, s: np.ndarray) -> np.ndarray:
    """Widen.dequantizeRotated (Widen.swift:374-428): fp32 [k, n] = float(H q) * (s / sqrt(G))."""
    q = np.ascontiguousarray(q_kn, np.int8)
    k, n = q.shape
    assert k % group == 0
    s = np.ascontiguousarray(np.broadcast_to(np.asarray(s, np.float32), (n,)), np.float32)
    out = np.empty((k, n), np.float32)
    lib().orc_dequantize_rotated(_p(q), k, n, group, _p(s), _p(out))
    return out


def w8a8_quantize(x: np.ndarray, group: int = 0):
    """W8A8.quantize (TensorGEMMInt8.swift:198-221) per row of fp32 x [m, k]: (codes int8 [m, k], scales fp32 [m])."""
    x = np.ascontiguousarray(x, np.float32)
    m, k = x.shape
    assert group == 0 or k % group == 0
    codes = np.empty((m, k), np.int8)
    scales = np.empty(m, np.float32)
    lib().orc_w8a8_quantize(_p(x), m, k, group, _p(codes), _p(scales))
    return codes, scales


def linear_w8a8(codes: np.ndarray, sx: np.ndarray, q_kn: np.ndarray, sw: np.ndarray, bias_bf16: np.ndarray | None = None):
    """float(codes . q) * (s_x * s_w) (+ bias): returns (c fp32 [m, n], y bf16 [m, n])."""
    codes = np.ascontiguousarray(codes, np.int8)
    q = np.ascontiguousarray(q_kn, np.int8)
    m, k = codes.shape
    n = q.shape[1]
    sx = np.ascontiguousarray(sx, np.float32)
    sw = np.ascontiguousarray(np.broadcast_to(np.asarray(sw, np.float32), (n,)), np.float32)
    b = None if bias_bf16 is None else np.ascontiguousarray(bias_bf16, np.uint16)
    c = np.empty((m, n), np.float32)
    y = np.empty((m, n), np.uint16)
    lib().orc_linear_w8a8(_p(codes), _p(sx), m, k, n, _p(q), _p(sw), _p(b), _p(c), _p(y))
    return c, y
