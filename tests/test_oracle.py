"""The oracle pinned before it is trusted (CPU only).

The oracle (oracle/oracle.c) restates Siliconed's CPU arithmetic.  Here it is checked against the
golden fixtures of tests/golden/, whose expected values come from independent implementations
(numpy IEEE fp32, ml_dtypes e4m3fn / bf16, numpy fp64) on the reference's own test inputs:

* DequantizeTests.swift:79-133   -- bit-exact ``float(q) * s`` for int8 and e4m3, every layout and scale type,
                                    all 256 codes, counts that are not multiples of 16, a guard value past the end.
* QuantizedMapTests.swift:132-143 -- the e4m3fn table on all 256 codes, NaN included.
* TensorGEMMBF16.swift:43-47     -- nearest-even bf16 rounding.
* Qwen3VLDecoderTests.swift:250-263 -- the GEMV's per-channel bar against fp64 (worst < 5e-6).
"""
import ctypes
import hashlib
import json
import os

import numpy as np
import pytest

import oracle
import refgen
from conftest import GOLDEN

SCALE = {"f32": oracle.SCALE_F32, "bf16": oracle.SCALE_BF16, "f16": oracle.SCALE_F16, "none": oracle.SCALE_NONE}
LAYOUT = {"tensor": oracle.LAYOUT_TENSOR, "columns": oracle.LAYOUT_COLUMNS, "blocks": oracle.LAYOUT_BLOCKS,
          "rows": oracle.LAYOUT_ROWS}
KIND = {"int8": oracle.INT8, "e4m3": oracle.E4M3}


def canonical_sha(out: np.ndarray) -> str:
    bits = out.view(np.uint32).copy()
    bits[np.isnan(out)] = 0x7FC00000
    return hashlib.sha256(bits.tobytes()).hexdigest()


def channel_error(got: np.ndarray, exact: np.ndarray):
    """Per-output-channel relative L2 (docs/VERIFY.md:223-232): (median, worst) over columns."""
    d = np.linalg.norm(got.astype(np.float64) - exact, axis=0)
    r = np.linalg.norm(exact, axis=0)
    e = d / np.maximum(r, 1e-300)
    return float(np.median(e)), float(e.max())


def regenerate(case):
    """The inputs of one DequantizeTests case, drawn in the test's own order."""
    g = refgen.SplitMix()
    q = g.codes(case["codes"])
    test = case["test"]
    if test in ("blocks", "blocks_rows"):
        k, n, b = 100, 2052, 32
        for st in ("f16", "bf16", "f32"):
            sb, sv = g.scales((k + b - 1) // b * n, st)
            if st == case["scale"]:
                return q, sb
    if test in ("columns", "columns_one_row"):
        for st in ("bf16", "f32"):
            sb, sv = g.scales(500, st)
            if st == case["scale"]:
                return q, sb
    if test in ("tensor", "fp8_cast"):
        sb, _ = g.scales(4, "f32")
        return q, sb[:4]
    if test == "rows":
        sb, _ = g.scales(case["scale_count"], "bf16")
        return q, sb
    raise AssertionError(test)


def test_e4m3_table_is_the_fixture():
    ref = json.load(open(os.path.join(GOLDEN, "e4m3_table.json")))["bits"]
    t = oracle.e4m3_table()
    bits = t.view(np.uint32).copy()
    bits[np.isnan(t)] = 0x7FC00000
    assert bits.tolist() == ref
    assert np.isnan(t[0x7F]) and np.isnan(t[0xFF]) and t[0x7E] == 448.0 and t[0x01] == 2.0 ** -9


def test_bf16_rounding_is_nearest_even():
    pairs = np.array(json.load(open(os.path.join(GOLDEN, "bf16_round.json")))["pairs"], np.uint64)
    f = pairs[:, 0].astype(np.uint32).view(np.float32)
    got = oracle.f32_to_bf16(f)
    assert np.array_equal(got, pairs[:, 1].astype(np.uint16))
    nan = np.array([0x7FC00001, 0xFF800001, 0x7F800001], np.uint32).view(np.float32)
    out = oracle.f32_to_bf16(nan)
    assert all(((int(o) & 0x7F80) == 0x7F80) and (int(o) & 0x7F) for o in out), "a NaN stays a NaN"


@pytest.mark.parametrize("case", json.load(open(os.path.join(GOLDEN, "dequant_kats.json")))["cases"],
                         ids=lambda c: f"{c['test']}-{c['kind']}-{c['scale']}")
def test_dequantize_known_answers(case):
    q, sb = regenerate(case)
    count = case["count"]
    out = np.full(count + 1, -7.0, np.float32)               # one guard value past the end
    vals = np.ascontiguousarray(q[case["offset"]:])
    s = None if case["scale"] == "none" else np.ascontiguousarray(sb)
    L = oracle.lib()
    L.orc_dequantize(vals.ctypes.data_as(ctypes.c_void_p), KIND[case["kind"]], count,
                     None if s is None else s.ctypes.data_as(ctypes.c_void_p), SCALE[case["scale"]],
                     LAYOUT[case["layout"]], case["width"], case["block"], case["first_row"],
                     out.ctypes.data_as(ctypes.c_void_p))
    assert out[count] == -7.0, "written past the end"
    assert canonical_sha(out[:count]) == case["sha256"]
    assert int(np.isnan(out[:count]).sum()) == case["nan"]


def test_a_planted_mistake_is_caught():
    """The comparison above is not vacuous: one value off by one ulp changes the digest."""
    case = json.load(open(os.path.join(GOLDEN, "dequant_kats.json")))["cases"][0]
    q, sb = regenerate(case)
    out = oracle.dequantize(q, KIND[case["kind"]], sb, SCALE[case["scale"]], LAYOUT[case["layout"]],
                            case["width"], case["block"], case["first_row"], count=case["count"])
    assert canonical_sha(out) == case["sha256"]
    bad = out.copy()
    i = int(np.flatnonzero(np.isfinite(bad) & (bad != 0))[1000])
    bad.view(np.uint32)[i] ^= 1
    assert canonical_sha(bad) != case["sha256"]


def test_gemv_splits_meet_the_reference_bar():
    """Qwen3VLDecoderTests.swift:250-263: every scale type, 5 splits, worst channel < 5e-6 vs fp64."""
    g = np.load(os.path.join(GOLDEN, "gemv_scale_types.npz"))
    x = g["x"]
    for st in ("bf16", "f16", "f32"):
        q, sb, sv = refgen.int8_matrix(1024, 1040, 77, st)
        if st == "f32":
            assert hashlib.sha256(q.tobytes()).digest() == g["q_sha256"].tobytes(), "generator restatement drifted"
        assert np.array_equal(sb, g[f"scale_bytes_{st}"])
        rows = [oracle.gemv_int8_splits(x[r], q, sv, 5)[1] for r in range(3)]
        med, worst = channel_error(np.stack(rows), g[f"exact_{st}"])
        assert med < 1e-6 and worst < 5e-6, (st, med, worst)


def test_linear_routes_against_fp64():
    g = np.load(os.path.join(GOLDEN, "linear_small.npz"))
    x, codes, s, b = g["int8_x"], g["int8_codes"], g["int8_s"], g["int8_bias"]
    c, y = oracle.linear_int8(x, codes.view(np.int8), s, b)
    med, worst = channel_error(c, g["int8_exact"])
    assert worst < 1e-5, worst
    assert np.array_equal(y, oracle.f32_to_bf16(c))
    # e4m3 through the widened route: the dequantized weight is the fixture's float(q) * s, bit for bit.
    x, codes, s, b = g["e4m3_x"], g["e4m3_codes"], g["e4m3_s"], g["e4m3_bias"]
    k, n = codes.shape
    w = oracle.dequantize(codes, oracle.E4M3, s, oracle.SCALE_F32, oracle.LAYOUT_COLUMNS, n).reshape(k, n)
    assert np.array_equal(w.view(np.uint32), g["e4m3_w"].view(np.uint32))
    c, y = oracle.linear_widened(x, w, b)
    med, worst = channel_error(c, g["e4m3_exact"])
    assert worst < 1e-5, worst
    c64 = oracle.linear_fp64(x, w, b)
    assert np.allclose(c64, g["e4m3_exact"], rtol=1e-12, atol=1e-12)


# ---------------------------------------------------------------------------------------------
# convrot (ComfyUI's rotated int8 maps): DequantizeTests.swift:159-214 restated


def regular_hadamard(g: int) -> np.ndarray:
    """The unnormalized regular Hadamard of size g by Kronecker powers of H4, built independently of
    the butterflies (as comfy_kitchen's _build_hadamard; DequantizeTests.swift:159-172)."""
    h4 = np.array([[1, 1, 1, -1], [1, 1, -1, 1], [1, -1, 1, 1], [-1, 1, 1, 1]], np.int64)
    h = h4
    while h.shape[0] < g:
        h = np.kron(h, h4)
    return h


@pytest.mark.parametrize("g,k,n", [(256, 768, 328), (256, 256, 12), (64, 192, 136), (16, 64, 40), (4, 8, 20),
                                   (16, 32, 8200), (4, 8, 4100)])
def test_dequantize_rotated_is_exactly_rotated(g, k, n):
    """Float(H q) * (s / sqrt(G)) at the bit (Widen.dequantizeRotated), with columns of +-127 / -128
    following H's first row (the extremes of m), bf16- and fp32-valued scales, one scale for the tensor."""
    rng = np.random.default_rng(g * 1000 + n)
    q = rng.integers(-128, 128, (k, n), dtype=np.int16).astype(np.int8)
    h = regular_hadamard(g)
    q[:g, 0] = np.where(h[0] > 0, 127, -128)
    q[:g, 1] = np.where(h[0] > 0, -128, 127)
    m = np.empty((k, n), np.int64)
    for g0 in range(0, k, g):
        m[g0:g0 + g] = h @ q[g0:g0 + g].astype(np.int64)
    assert np.abs(m).max() <= 32648
    norm = np.float32(1.0 / np.sqrt(g))
    s32 = (np.abs(rng.standard_normal(n)) * 1e-3 + 1e-6).astype(np.float32)
    for s in (s32, oracle.bf16_to_f32(oracle.f32_to_bf16(s32)), np.full(n, s32[0], np.float32)):
        got = oracle.dequantize_rotated(q, g, s)
        want = m.astype(np.float32) * (s * norm)          # one fp32 multiply (s * norm is exact)
        assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), f"G {g}, [{k}, {n}]"


def test_rotate_groups_is_the_orthogonal_rotation():
    """The fp32 butterflies of rotate_groups against x . H / sqrt(G) in fp64: the bf16 results agree
    except where the fp32 sum sits within its rounding error of a bf16 tie; rotating twice gives x back
    (H / sqrt(G) is symmetric and orthogonal) to within two bf16 roundings."""
    rng = np.random.default_rng(7)
    for g, k in ((256, 768), (64, 192), (16, 48), (4, 8)):
        x = oracle.f32_to_bf16(rng.standard_normal((64, k), dtype=np.float32))
        got = oracle.rotate_groups_bf16(x, g)
        xf = oracle.bf16_to_f32(x).astype(np.float64)
        h = regular_hadamard(g).astype(np.float64) / np.sqrt(g)
        ref = np.concatenate([xf[:, g0:g0 + g] @ h for g0 in range(0, k, g)], axis=1)
        want = oracle.f32_to_bf16(ref.astype(np.float32))
        assert np.mean(got == want) > 0.995, g
        gf = oracle.bf16_to_f32(got).astype(np.float64)
        assert np.all(np.abs(gf - ref) <= 2.0 ** -8 * np.abs(ref) + 1e-6 * np.abs(xf).max()), g
        back = oracle.bf16_to_f32(oracle.rotate_groups_bf16(got, g)).astype(np.float64)
        assert np.all(np.abs(back - xf) <= 2.0 ** -6 * np.abs(xf).max()), g


# ---------------------------------------------------------------------------------------------
# W8A8 (TensorGEMMInt8.swift): the oracle against an independent numpy restatement of the recipe


def numpy_w8a8_quantize(x: np.ndarray, group: int):
    """W8A8.quantize restated on whole columns of rows at once in numpy fp32 (IEEE adds, an IEEE
    division, np.rint half to even)."""
    y = x.astype(np.float32).copy()
    if group:
        norm = np.float32(1.0 / np.sqrt(group))
        m, k = y.shape
        v = y.reshape(m, k // group, group)
        span = 1
        while span < group:
            w = v.reshape(m, k // group, group // (4 * span), 4, span)
            a, b, c, d = w[:, :, :, 0].copy(), w[:, :, :, 1].copy(), w[:, :, :, 2].copy(), w[:, :, :, 3].copy()
            p, mm, u, ww = a + b, a - b, c + d, c - d
            w[:, :, :, 0], w[:, :, :, 1], w[:, :, :, 2], w[:, :, :, 3] = p + ww, p - ww, mm + u, u - mm
            span *= 4
        y = v.reshape(m, k) * norm
    top = np.abs(y).max(axis=1)
    scale = np.maximum(top / np.float32(127), np.float32(1e-30)).astype(np.float32)
    codes = np.clip(np.rint(y / scale[:, None]), -128, 127).astype(np.int8)
    return codes, scale


@pytest.mark.parametrize("m,k,group", [(150, 768, 256), (70, 10240, 256), (65, 448, 64), (33, 520, 0), (9, 16, 4)])
def test_w8a8_is_the_recipe(m, k, group):
    """The cases of W8A8KernelTests.swift:71-78 (rows of values in +-3, a row of zeros whose scale is the
    recipe's floor 1e-30, a massive column); codes, scales and the product at the bit."""
    rng = np.random.default_rng(m * k + group)
    a = ((rng.random((m, k), dtype=np.float32) - 0.5) * 6).astype(np.float32)
    a[3 % m] = 0
    a[:, k // 3] *= 300
    codes, sx = oracle.w8a8_quantize(a, group)
    ref_codes, ref_sx = numpy_w8a8_quantize(a, group)
    assert np.array_equal(sx.view(np.uint32), ref_sx.view(np.uint32))
    assert np.array_equal(codes, ref_codes)
    assert sx[3 % m] == np.float32(1e-30) and not codes[3 % m].any()
    n = 40
    q = rng.integers(-127, 128, (k, n), dtype=np.int16).astype(np.int8)
    sw = ((np.abs(rng.random(n, dtype=np.float32) - 0.5) + 0.01) / 64).astype(np.float32)
    c, _ = oracle.linear_w8a8(codes, sx, q, sw)
    acc = codes.astype(np.int64) @ q.astype(np.int64)
    assert np.abs(acc).max() < 2 ** 31
    want = acc.astype(np.int32).astype(np.float32) * (sx[:, None] * sw[None, :])
    assert np.array_equal(c.view(np.uint32), want.view(np.uint32))
    b = oracle.f32_to_bf16(rng.standard_normal(n, dtype=np.float32))
    cb, yb = oracle.linear_w8a8(codes, sx, q, sw, b)
    assert np.array_equal(cb.view(np.uint32), (want + oracle.bf16_to_f32(b)).view(np.uint32))
    assert np.array_equal(yb, oracle.f32_to_bf16(cb))
