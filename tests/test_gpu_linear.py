"""Parity of the CUDA path with the oracle, through the C ABI, on a B200.

Bars (stated here, used throughout):
* dequantized weights: bit-exact (NaN codes: NaN in the same places);
* fp32 outputs (sc_linear_ex, SC_OUT_F32) against the oracle's fp32 result: relative L2 <= 1e-5
  (only the summation order differs), and the reference's own per-channel bar against fp64 where the
  reference states one (Qwen3VLDecoderTests.swift:250-263: median < 1e-6, worst < 5e-6);
* bf16 outputs against the oracle's bf16 result of the same path: relative L2 <= 1e-3 and
  max-abs <= 2e-2 (the north star's GEMM bar), plus at most one bf16 ulp per value against the
  oracle's fp32 result.
"""
import ctypes

import numpy as np
import pytest

import oracle
import refgen
from siliconed_b200 import abi, configs

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

if not torch.cuda.is_available():  # collected on CPU boxes, skipped there
    pytest.skip("needs a CUDA device", allow_module_level=True)

from siliconed_b200.products import Context, QuantizedWeight  # noqa: E402

REL_L2_BF16, MAX_ABS_BF16, REL_L2_F32 = 1e-3, 2e-2, 1e-5


@pytest.fixture(scope="module")
def ctx():
    c = Context(0)
    yield c
    c.close()


def dev(a: np.ndarray):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def host(t) -> np.ndarray:
    return t.cpu().numpy()


def bf16_dev(bits: np.ndarray):
    return dev(bits.astype(np.uint16).view(np.int16)).view(torch.bfloat16)


def bf16_host(t) -> np.ndarray:
    return host(t.view(torch.int16)).view(np.uint16)


def f32_of_bf16(bits: np.ndarray) -> np.ndarray:
    return (bits.astype(np.uint32) << 16).view(np.float32)


def rel_l2(got, ref) -> float:
    got, ref = np.asarray(got, np.float64), np.asarray(ref, np.float64)
    return float(np.linalg.norm(got - ref) / max(np.linalg.norm(ref), 1e-300))


def linear_ex(ctx, w, x_dev, m, bias_dev, f32: bool, workspace: bool = True):
    """sc_linear_ex through ctypes, with a workspace of the reported size (workspace=True) or none
    (for m > 128: the fused pair kernel instead of the widened route)."""
    out = torch.empty((m, w.n), dtype=torch.float32 if f32 else torch.bfloat16, device="cuda")
    need = w.workspace_bytes(m) if workspace else 0
    ws = torch.empty(need, dtype=torch.uint8, device="cuda") if need else None
    ws_ptr = ws.data_ptr() if ws is not None else 0
    st = torch.cuda.current_stream().cuda_stream
    status = ctx.lib.sc_linear_ex(ctx.ptr, w.ptr, ctypes.c_void_p(x_dev.data_ptr()), m,
                                  ctypes.c_void_p(bias_dev.data_ptr() if bias_dev is not None else 0),
                                  ctypes.c_void_p(out.data_ptr()), abi.OUT_F32 if f32 else abi.OUT_BF16,
                                  ctypes.c_void_p(ws_ptr), need, ctypes.c_void_p(st))
    ctx.check(status)
    ctx.poll_errors()
    return out


def check_against_oracle(ctx, kind, x_bits, codes_kn, s, bias_bits, label, workspace=True):
    """Runs bf16 and fp32 outputs through the ABI and compares them with the oracle's route."""
    m, k = x_bits.shape
    n = codes_kn.shape[1]
    w = QuantizedWeight(ctx, codes_kn, kind, s)
    xd = bf16_dev(x_bits)
    bd = bf16_dev(bias_bits) if bias_bits is not None else None
    if kind == abi.WEIGHT_INT8:
        c_ref, y_ref = oracle.linear_int8(x_bits, codes_kn.view(np.int8), s, bias_bits)
    else:
        wf = oracle.dequantize(codes_kn, oracle.E4M3, s, oracle.SCALE_F32, oracle.LAYOUT_COLUMNS, n).reshape(k, n)
        c_ref, y_ref = oracle.linear_widened(x_bits, wf, bias_bits)
    y32 = host(linear_ex(ctx, w, xd, m, bd, True, workspace))
    e32 = rel_l2(y32, c_ref)
    assert e32 <= REL_L2_F32, f"{label}: fp32 rel-L2 {e32}"
    y16 = bf16_host(linear_ex(ctx, w, xd, m, bd, False, workspace))
    yf, rf = f32_of_bf16(y16), f32_of_bf16(y_ref)
    e16, mx = rel_l2(yf, rf), float(np.max(np.abs(yf.astype(np.float64) - rf)))
    assert e16 <= REL_L2_BF16 and mx <= MAX_ABS_BF16, f"{label}: bf16 rel-L2 {e16}, max-abs {mx}"
    # One bf16 ulp of the value, plus the spread that a change of fp32 summation order can make:
    # 8 sqrt(K) 2^-24 sqrt(sum_k (x w)^2), a loose multiple of its typical size.
    wf = oracle.dequantize(codes_kn, kind, s, oracle.SCALE_F32, oracle.LAYOUT_COLUMNS, n).reshape(k, n)
    xf = torch.from_numpy(f32_of_bf16(x_bits))
    spread = torch.sqrt((xf * xf) @ torch.from_numpy(wf * wf)).numpy().astype(np.float64)
    bound = 2.0 ** -7 * np.abs(c_ref) + 8.0 * np.sqrt(k) * 2.0 ** -24 * spread + 1e-9
    excess = np.abs(yf.astype(np.float64) - c_ref) - bound
    assert float(excess.max()) <= 0.0, f"{label}: more than one bf16 ulp from the fp32 result"
    w.close()
    return e32, e16


# ---------------------------------------------------------------------------------------------
# dequantization: bit-exact (DequantizeTests.swift:79-133 restated on the device)


def canonical(a: np.ndarray) -> np.ndarray:
    b = a.view(np.uint32).copy()
    b[np.isnan(a)] = 0x7FC00000
    return b


@pytest.mark.parametrize("kind", [abi.WEIGHT_INT8, abi.WEIGHT_E4M3])
@pytest.mark.parametrize("stype", ["f32", "bf16", "f16"])
@pytest.mark.parametrize("layout", ["columns", "tensor"])
def test_dequantize_bit_exact(ctx, kind, stype, layout):
    k, n = 300, 500                        # neither a multiple of the arena's 64 / 256
    g = refgen.SplitMix()
    q = g.codes(k * n).reshape(k, n)       # every one of the 256 codes, then draws
    sb, sv = g.scales(n if layout == "columns" else 4, stype)
    if layout == "tensor":
        sb = sb[: {"f32": 4, "bf16": 2, "f16": 2}[stype]]
    scales = torch.from_numpy(sb.copy()).view({"f32": torch.float32, "bf16": torch.bfloat16,
                                              "f16": torch.float16}[stype])
    w = QuantizedWeight(ctx, q, kind, scales)
    got = host(w.dequantize())
    st = {"f32": oracle.SCALE_F32, "bf16": oracle.SCALE_BF16, "f16": oracle.SCALE_F16}[stype]
    lay = oracle.LAYOUT_COLUMNS if layout == "columns" else oracle.LAYOUT_TENSOR
    ref = oracle.dequantize(q, oracle.INT8 if kind == abi.WEIGHT_INT8 else oracle.E4M3, sb, st, lay, n).reshape(k, n)
    assert np.array_equal(canonical(got), canonical(ref))
    w.close()


def test_dequantize_published_layout_and_shard(ctx):
    k, n = 136, 700
    g = np.random.default_rng(3)
    q_kn = g.integers(0, 256, (k, n), dtype=np.uint8)
    s = (np.abs(g.standard_normal(n)) * 1e-3 + 1e-4).astype(np.float32)
    ref = oracle.dequantize(q_kn, oracle.INT8, s, oracle.SCALE_F32, oracle.LAYOUT_COLUMNS, n).reshape(k, n)
    w = QuantizedWeight(ctx, np.ascontiguousarray(q_kn.T), abi.WEIGHT_INT8, s, published_nk=True)
    assert np.array_equal(host(w.dequantize()).view(np.uint32), ref.view(np.uint32))
    w.close()
    for (n0, n1) in ((0, 256), (256, 513), (600, 700)):
        w = QuantizedWeight(ctx, q_kn, abi.WEIGHT_INT8, s, columns=(n0, n1))
        assert w.n == n1 - n0
        assert np.array_equal(host(w.dequantize()).view(np.uint32), ref[:, n0:n1].view(np.uint32))
        w.close()
    # values already on the device
    w = QuantizedWeight(ctx, dev(q_kn), abi.WEIGHT_INT8, torch.from_numpy(s).cuda())
    assert np.array_equal(host(w.dequantize()).view(np.uint32), ref.view(np.uint32))
    w.close()


def test_subnormal_scale_is_refused(ctx):
    q = np.ones((16, 8), np.int8)
    s = np.full(8, 1e-3, np.float32)
    s[3] = np.float32(1e-39)               # |s| * 1 < 2^-126
    with pytest.raises(abi.SiliconedError) as e:
        QuantizedWeight(ctx, q, abi.WEIGHT_INT8, s)
    assert e.value.status == abi.REFUSED
    s[3] = np.float32(2.0 ** -120)         # fine for int8, subnormal for e4m3 (2^-9 * 2^-120)
    QuantizedWeight(ctx, q, abi.WEIGHT_INT8, s).close()
    with pytest.raises(abi.SiliconedError):
        QuantizedWeight(ctx, q.view(np.uint8), abi.WEIGHT_E4M3, s)


# ---------------------------------------------------------------------------------------------
# the tensor-core GEMM (m > 32) and the GEMV (m <= 32) against the oracle


@pytest.mark.parametrize("m,k,n", [(33, 64, 256), (130, 200, 300), (257, 1024, 512), (512, 3072, 768),
                                   (1000, 136, 1030)])
def test_linear_int8_matches_oracle(ctx, m, k, n):
    g = np.random.default_rng(m * 7 + k)
    x = configs.to_bf16_bits(g.standard_normal((m, k), dtype=np.float32))
    q = g.integers(-128, 128, (k, n), dtype=np.int16).astype(np.int8).view(np.uint8)
    s = (np.abs(g.standard_normal(n)) * 0.02 / 127 + 1e-6).astype(np.float32)
    b = configs.to_bf16_bits(g.standard_normal(n, dtype=np.float32) * 0.01)
    check_against_oracle(ctx, abi.WEIGHT_INT8, x, q, s, b, f"int8 {m}x{k}x{n}")


@pytest.mark.parametrize("m,k,n", [(64, 128, 256), (200, 512, 640), (513, 1024, 1024)])
def test_linear_e4m3_matches_oracle(ctx, m, k, n):
    g = np.random.default_rng(m + k + n)
    x = configs.to_bf16_bits(g.standard_normal((m, k), dtype=np.float32))
    q = configs.to_e4m3_codes(g.standard_normal((k, n), dtype=np.float32) * 4)
    q[(q & 0x7F) == 0x7F] ^= 1
    s = (np.abs(g.standard_normal(n)) * 0.02 / 448 + 1e-6).astype(np.float32)
    b = configs.to_bf16_bits(g.standard_normal(n, dtype=np.float32) * 0.01)
    check_against_oracle(ctx, abi.WEIGHT_E4M3, x, q, s, b, f"e4m3 {m}x{k}x{n}")


@pytest.mark.parametrize("m", [1, 2, 3, 5, 8, 13, 17, 32])
def test_gemv_matches_oracle(ctx, m):
    k, n = 1024, 1040
    g = np.random.default_rng(100 + m)
    x = configs.to_bf16_bits(g.standard_normal((m, k), dtype=np.float32))
    q = g.integers(-128, 128, (k, n), dtype=np.int16).astype(np.int8).view(np.uint8)
    s = (np.abs(g.standard_normal(n)) * 0.02 / 127 + 1e-6).astype(np.float32)
    b = configs.to_bf16_bits(g.standard_normal(n, dtype=np.float32) * 0.01)
    check_against_oracle(ctx, abi.WEIGHT_INT8, x, q, s, b, f"gemv m={m}")


@pytest.mark.parametrize("m", [1, 4, 32])
def test_gemv_e4m3_matches_oracle(ctx, m):
    k, n = 768, 520
    g = np.random.default_rng(7 + m)
    x = configs.to_bf16_bits(g.standard_normal((m, k), dtype=np.float32))
    q = configs.to_e4m3_codes(g.standard_normal((k, n), dtype=np.float32))
    q[(q & 0x7F) == 0x7F] ^= 1
    s = (np.abs(g.standard_normal(n)) * 0.02 / 448 + 1e-6).astype(np.float32)
    check_against_oracle(ctx, abi.WEIGHT_E4M3, x, q, s, None, f"gemv e4m3 m={m}")


@pytest.mark.parametrize("kind,m,nan", [(abi.WEIGHT_INT8, 5, False), (abi.WEIGHT_INT8, 9, False), (abi.WEIGHT_INT8, 16, False),
                                         (abi.WEIGHT_INT8, 24, False), (abi.WEIGHT_E4M3, 32, True)])
def test_skinny_tensor_core_product_agrees_with_gemv(ctx, kind, m, nan):
    """4 < m <= 32 runs on the tensor cores (K split over a cluster, partial sums added in rank order
    through distributed shared memory); sc_gemv_w8 forces the CUDA-core GEMV on the same inputs."""
    k, n = 4096, 1000
    g = np.random.default_rng(300 + m)
    x = configs.to_bf16_bits(g.standard_normal((m, k), dtype=np.float32))
    if kind == abi.WEIGHT_INT8:
        q = g.integers(-128, 128, (k, n), dtype=np.int16).astype(np.int8).view(np.uint8)
    else:
        q = configs.to_e4m3_codes(g.standard_normal((k, n), dtype=np.float32) * 4)
        q[(q & 0x7F) == 0x7F] ^= 1
        if nan:
            q[g.integers(0, k, 5), g.integers(0, n, 5)] = 0x7F
    s = (np.abs(g.standard_normal(n)) * 0.004 / 127 + 1e-7).astype(np.float32)
    b = configs.to_bf16_bits(g.standard_normal(n, dtype=np.float32) * 0.01)
    w = QuantizedWeight(ctx, q, kind, s)
    xd, bd = bf16_dev(x), bf16_dev(b)
    tc = f32_of_bf16(bf16_host(w.linear(xd, bias=bd)))
    gv = f32_of_bf16(bf16_host(w.gemv(xd, bias=bd)))
    ctx.poll_errors()
    assert np.array_equal(np.isnan(tc), np.isnan(gv))
    keep = ~np.isnan(gv)
    assert nan or keep.all()
    e = rel_l2(tc[keep], gv[keep])
    mx = float(np.max(np.abs(tc[keep].astype(np.float64) - gv[keep])))
    assert e <= REL_L2_BF16 and mx <= MAX_ABS_BF16, (e, mx)
    w.close()


@pytest.mark.parametrize("m,k,n", [(16, 4096, 12288), (12, 12288, 4096), (7, 2048, 8000), (9, 512, 38400), (13, 3000, 3200),
                                   (3, 4096, 12288), (4, 2048, 8000)])
def test_int8_skinny_product_matches_the_oracle_and_repeats(ctx, m, k, n):
    """With its workspace, an int8 product of 2 < m <= 16 rows runs on the integer tensor cores (without it,
    3 or 4 rows run the GEMV): x as three
    exact 8-bit digit planes, the codes as stored, the weight split in equal shares over one CTA per SM (with
    K = 512 a tile is two units and a share four or five: partials meet through the fix-up).  fp32 output
    within the oracle's bar (the integer sum is exact where the oracle's fp32 sum rounds), the same bits on a
    second call, within the bar of the cluster kernel that runs without the workspace, and bf16 output
    within the GEMM bar of the oracle's bf16 result."""
    g = np.random.default_rng(m * k + n)
    x = configs.to_bf16_bits(g.standard_normal((m, k), dtype=np.float32) * 2.0 ** g.integers(-3, 2, (m, 1)))
    x[0, : k // 3] = 0                                            # a stretch of zeros
    x[1, 5] = configs.to_bf16_bits(np.array([1e-30], np.float32))[0]  # far below the row's largest
    q = g.integers(-128, 128, (k, n), dtype=np.int16).astype(np.int8).view(np.uint8)
    s = (np.abs(g.standard_normal(n)) * 0.01 / 127 + 1e-6).astype(np.float32)
    b = configs.to_bf16_bits(g.standard_normal(n, dtype=np.float32) * 0.01)
    w = QuantizedWeight(ctx, q, abi.WEIGHT_INT8, s)
    assert w.workspace_bytes(m) > 0, "the integer route applies"
    xd, bd = bf16_dev(x), bf16_dev(b)
    c_ref, y_ref = oracle.linear_int8(x, q.view(np.int8), s, b)
    first = host(linear_ex(ctx, w, xd, m, bd, True))
    again = host(linear_ex(ctx, w, xd, m, bd, True))
    cluster = host(linear_ex(ctx, w, xd, m, bd, True, workspace=False))
    assert rel_l2(first, c_ref) <= REL_L2_F32, rel_l2(first, c_ref)
    assert np.array_equal(first.view(np.uint32), again.view(np.uint32)), "the same bits on a second call"
    assert rel_l2(cluster, first) <= REL_L2_F32
    y16 = f32_of_bf16(bf16_host(linear_ex(ctx, w, xd, m, bd, False)))
    rf = f32_of_bf16(y_ref)
    assert rel_l2(y16, rf) <= REL_L2_BF16 and float(np.max(np.abs(y16.astype(np.float64) - rf))) <= MAX_ABS_BF16
    w.close()


def test_int8_products_of_17_to_32_rows_take_no_workspace(ctx):
    """Above 16 rows the int8 skinny product is the cluster kernel (no workspace): the reported size is 0
    and the product still meets the oracle's bar."""
    k, n = 4096, 4096   # 512 units of 128 x 256: at least two per SM, so 16 rows take the integer route
    g = np.random.default_rng(17)
    q = g.integers(-128, 128, (k, n), dtype=np.int16).astype(np.int8).view(np.uint8)
    s = (np.abs(g.standard_normal(n)) * 0.01 / 127 + 1e-6).astype(np.float32)
    w = QuantizedWeight(ctx, q, abi.WEIGHT_INT8, s)
    assert w.workspace_bytes(16) > 0
    for m in (17, 24, 32):
        assert w.workspace_bytes(m) == 0, m
    w.close()
    x = configs.to_bf16_bits(g.standard_normal((20, k), dtype=np.float32))
    check_against_oracle(ctx, abi.WEIGHT_INT8, x, q, s, None, "int8 m=20")


@pytest.mark.parametrize("kind,m", [(abi.WEIGHT_INT8, 33), (abi.WEIGHT_INT8, 64), (abi.WEIGHT_INT8, 100),
                                    (abi.WEIGHT_INT8, 128), (abi.WEIGHT_E4M3, 80)])
def test_prefill_rows_on_the_cluster_kernel_match_the_oracle(ctx, kind, m):
    """32 < m <= 128 on a weight too narrow for 148 output tiles of 128 x 256 (the Z-Image encoder's gate / up
    shape, [9728, 2560] published): the cluster kernel with 64 or 128 token columns, K split over the cluster's
    CTAs and added in rank order."""
    k, n = 2560, 9728
    g = np.random.default_rng(900 + m)
    x = configs.to_bf16_bits(g.standard_normal((m, k), dtype=np.float32))
    if kind == abi.WEIGHT_INT8:
        q = g.integers(-128, 128, (k, n), dtype=np.int16).astype(np.int8).view(np.uint8)
        s = (np.abs(g.standard_normal(n)) * 0.02 / 127 + 1e-6).astype(np.float32)
    else:
        q = configs.to_e4m3_codes(g.standard_normal((k, n), dtype=np.float32) * 4)
        q[(q & 0x7F) == 0x7F] ^= 1
        s = (np.abs(g.standard_normal(n)) * 0.02 / 448 + 1e-6).astype(np.float32)
    b = configs.to_bf16_bits(g.standard_normal(n, dtype=np.float32) * 0.01)
    check_against_oracle(ctx, kind, x, q, s, b, f"prefill m={m}")


def test_int8_skinny_product_with_zero_and_nonfinite_rows(ctx):
    """A row of x that is all zeros gives the bias; a row holding an infinity gives NaN (its products meet
    weights of both signs); the other rows are unaffected."""
    m, k, n = 8, 2048, 8192
    g = np.random.default_rng(5)
    x = configs.to_bf16_bits(g.standard_normal((m, k), dtype=np.float32))
    x[2] = 0
    x[5, 77] = 0x7F80                                            # +inf
    q = g.integers(-128, 128, (k, n), dtype=np.int16).astype(np.int8).view(np.uint8)
    s = (np.abs(g.standard_normal(n)) * 0.01 / 127 + 1e-6).astype(np.float32)
    b = configs.to_bf16_bits(g.standard_normal(n, dtype=np.float32) * 0.01)
    w = QuantizedWeight(ctx, q, abi.WEIGHT_INT8, s)
    assert w.workspace_bytes(m) > 0
    y = host(linear_ex(ctx, w, bf16_dev(x), m, bf16_dev(b), True))
    assert np.array_equal(y[2], f32_of_bf16(b))
    assert np.isnan(y[5]).all()
    keep = [r for r in range(m) if r not in (2, 5)]
    c_ref, _ = oracle.linear_int8(x[keep], q.view(np.int8), s, b)
    assert rel_l2(y[keep], c_ref) <= REL_L2_F32
    w.close()


def test_gemv_meets_the_reference_bar(ctx):
    """Qwen3VLDecoderTests.swift:250-263 on its own inputs (x rounded to bf16): per-channel relative
    L2 against fp64, median < 1e-6 and worst < 5e-6, for every scale type."""
    import os
    from conftest import GOLDEN
    gz = np.load(os.path.join(GOLDEN, "gemv_scale_types.npz"))
    xb = configs.to_bf16_bits(gz["x"])
    xd = bf16_dev(xb)
    for st in ("bf16", "f16", "f32"):
        q, sb, sv = refgen.int8_matrix(1024, 1040, 77, st)
        scales = torch.from_numpy(sb.copy()).view({"f32": torch.float32, "bf16": torch.bfloat16,
                                                  "f16": torch.float16}[st])
        w = QuantizedWeight(ctx, q, abi.WEIGHT_INT8, scales)
        got = host(linear_ex(ctx, w, xd, 3, None, True)).astype(np.float64)
        exact = gz[f"exact_bf16x_{st}"]
        e = np.linalg.norm(got - exact, axis=0) / np.linalg.norm(exact, axis=0)
        assert np.median(e) < 1e-6 and e.max() < 5e-6, (st, float(np.median(e)), float(e.max()))
        w.close()


def test_nan_codes_propagate(ctx):
    k, n, m = 64, 256, 40
    g = np.random.default_rng(5)
    q = configs.to_e4m3_codes(g.standard_normal((k, n), dtype=np.float32))
    q[(q & 0x7F) == 0x7F] ^= 1
    q[10, 7] = 0x7F
    q[3, 100] = 0xFF
    s = np.full(n, 1e-3, np.float32)
    x = configs.to_bf16_bits(g.standard_normal((m, k), dtype=np.float32))
    w = QuantizedWeight(ctx, q, abi.WEIGHT_E4M3, s)
    for mm in (m, 2):                          # the GEMM and the GEMV
        y = f32_of_bf16(bf16_host(w.linear(bf16_dev(x[:mm]))))
        nan_cols = sorted(set(np.nonzero(np.isnan(y))[1].tolist()))
        assert nan_cols == [7, 100]
        assert np.isnan(y[:, [7, 100]]).all()
    w.close()


def test_edge_shapes_and_guards(ctx):
    """Ragged shapes, guard canaries past the output, deterministic bits, m = 0."""
    for (m, k, n) in ((33, 8, 8), (131, 72, 3), (35, 4104, 264), (1, 8, 1), (2, 4096, 257)):
        g = np.random.default_rng(m + n)
        x = configs.to_bf16_bits(g.standard_normal((m, k), dtype=np.float32))
        q = g.integers(-128, 128, (k, n), dtype=np.int16).astype(np.int8).view(np.uint8)
        s = (np.abs(g.standard_normal(n)) * 0.01 + 1e-5).astype(np.float32)
        w = QuantizedWeight(ctx, q, abi.WEIGHT_INT8, s)
        guard = torch.full((m * n + 64,), -7.0, dtype=torch.bfloat16, device="cuda")
        out = guard[: m * n].view(m, n)
        w.linear(bf16_dev(x), out=out)
        torch.cuda.synchronize()
        assert bool((guard[m * n:] == -7.0).all()), f"written past the end at {m}x{k}x{n}"
        first = bf16_host(out).copy()
        w.linear(bf16_dev(x), out=out)
        assert np.array_equal(first, bf16_host(out)), "not deterministic"
        _, y_ref = oracle.linear_int8(x, q.view(np.int8), s, None)
        e = rel_l2(f32_of_bf16(first), f32_of_bf16(y_ref))
        assert e <= REL_L2_BF16, (m, k, n, e)
        w.close()
    w = QuantizedWeight(ctx, np.ones((8, 8), np.int8), abi.WEIGHT_INT8, np.ones(8, np.float32))
    empty = torch.empty((0, 8), dtype=torch.bfloat16, device="cuda")
    assert w.linear(empty).shape == (0, 8)
    w.close()


def test_errors_are_statuses(ctx):
    w = QuantizedWeight(ctx, np.ones((64, 64), np.int8), abi.WEIGHT_INT8, np.ones(64, np.float32))
    x = torch.zeros((40, 64), dtype=torch.bfloat16, device="cuda")
    buf = torch.zeros(40 * 64 + 8, dtype=torch.bfloat16, device="cuda")
    with pytest.raises(abi.SiliconedError) as e:       # y not 16-byte aligned
        w.linear(x, out=buf[1:1 + 40 * 64].view(40, 64))
    assert e.value.status == abi.UNALIGNED
    host_x = torch.zeros((40, 64), dtype=torch.bfloat16).pin_memory()
    out = torch.empty((40, 64), dtype=torch.bfloat16, device="cuda")
    st = ctx.lib.sc_linear(ctx.ptr, w.ptr, ctypes.c_void_p(host_x.data_ptr()), 40, None,
                           ctypes.c_void_p(out.data_ptr()), None, 0, None)
    assert st == abi.INVALID_ARG                        # host memory is refused, never dereferenced
    st = ctx.lib.sc_linear_fp8(ctx.ptr, w.ptr, ctypes.c_void_p(x.data_ptr()), 40, None,
                               ctypes.c_void_p(out.data_ptr()), None, 0, None)
    assert st == abi.INVALID_ARG                        # an int8 weight on the fp8 entry
    with pytest.raises(abi.SiliconedError) as e:
        w.gemv(torch.zeros((33, 64), dtype=torch.bfloat16, device="cuda"))
    assert e.value.status == abi.UNSUPPORTED_SHAPE
    w.close()
    w = QuantizedWeight(ctx, np.ones((12, 16), np.int8), abi.WEIGHT_INT8, np.ones(16, np.float32))
    with pytest.raises(abi.SiliconedError) as e:       # K = 12: activation rows not 16-byte multiples
        w.linear(torch.zeros((40, 12), dtype=torch.bfloat16, device="cuda"))
    assert e.value.status == abi.UNSUPPORTED_SHAPE
    w.close()
    ctx.poll_errors()                                   # no device-side wait gave up


# ---------------------------------------------------------------------------------------------
# more shapes of the pair GEMM (fewer tiles than CTA pairs, ragged m and n, short K), and batch
# invariance: every output is summed in the same order whatever tile it falls in


@pytest.mark.parametrize("kind,m,k,n", [(abi.WEIGHT_INT8, 256, 3072, 3072), (abi.WEIGHT_INT8, 600, 4096, 1000),
                                        (abi.WEIGHT_INT8, 4096, 512, 3072), (abi.WEIGHT_E4M3, 384, 2048, 2560),
                                        (abi.WEIGHT_INT8, 2304, 256, 5000), (abi.WEIGHT_E4M3, 1600, 1024, 1000),
                                        # more than 16 row tiles: grouped tile order, ragged last group
                                        (abi.WEIGHT_INT8, 9000, 256, 1288), (abi.WEIGHT_E4M3, 4500, 512, 776)])
def test_linear_more_shapes_match_oracle(ctx, kind, m, k, n):
    g = np.random.default_rng(m + k + n)
    x = configs.to_bf16_bits(g.standard_normal((m, k), dtype=np.float32))
    # Scales keep |y| below 4, where the max-abs bar of 2e-2 exceeds one bf16 ulp.
    amp = 0.02 * np.sqrt(768.0 / k)
    if kind == abi.WEIGHT_INT8:
        q = g.integers(-128, 128, (k, n), dtype=np.int16).astype(np.int8).view(np.uint8)
        s = (np.abs(g.standard_normal(n)) * amp / 127 + 1e-7).astype(np.float32)
    else:
        q = configs.to_e4m3_codes(g.standard_normal((k, n), dtype=np.float32) * 4)
        q[(q & 0x7F) == 0x7F] ^= 1
        s = (np.abs(g.standard_normal(n)) * amp / 448 + 1e-7).astype(np.float32)
    b = configs.to_bf16_bits(g.standard_normal(n, dtype=np.float32) * 0.01)
    check_against_oracle(ctx, kind, x, q, s, b, f"shape {m}x{k}x{n}")


@pytest.mark.parametrize("kind,m,k,n", [(abi.WEIGHT_INT8, 600, 4096, 1000), (abi.WEIGHT_E4M3, 384, 2048, 2560),
                                        (abi.WEIGHT_INT8, 4500, 256, 1288)])
def test_fused_pair_kernel_matches_oracle(ctx, kind, m, k, n):
    """The fused pair kernel (no workspace: codes converted in shared memory) on its own."""
    g = np.random.default_rng(m * 3 + n)
    x = configs.to_bf16_bits(g.standard_normal((m, k), dtype=np.float32))
    amp = 0.02 * np.sqrt(768.0 / k)
    if kind == abi.WEIGHT_INT8:
        q = g.integers(-128, 128, (k, n), dtype=np.int16).astype(np.int8).view(np.uint8)
        s = (np.abs(g.standard_normal(n)) * amp / 127 + 1e-7).astype(np.float32)
    else:
        q = configs.to_e4m3_codes(g.standard_normal((k, n), dtype=np.float32) * 4)
        q[(q & 0x7F) == 0x7F] ^= 1
        s = (np.abs(g.standard_normal(n)) * amp / 448 + 1e-7).astype(np.float32)
    b = configs.to_bf16_bits(g.standard_normal(n, dtype=np.float32) * 0.01)
    check_against_oracle(ctx, kind, x, q, s, b, f"fused {m}x{k}x{n}", workspace=False)


@pytest.mark.parametrize("kind,m,k,n,nan", [(abi.WEIGHT_INT8, 1536, 3072, 3072, False),
                                            (abi.WEIGHT_INT8, 4096, 512, 3072, False),
                                            (abi.WEIGHT_E4M3, 2000, 2048, 2560, False),
                                            (abi.WEIGHT_E4M3, 1600, 512, 700, True),
                                            # 160 pair tiles in one group: the widening inside the GEMM
                                            (abi.WEIGHT_E4M3, 4096, 512, 2560, True),
                                            (abi.WEIGHT_E4M3, 4096, 512, 2560, False)])
def test_widened_and_fused_routes_agree(ctx, kind, m, k, n, nan):
    """The widened route (from 1536 rows, workspace given) and the fused kernel (none) give the
    same bits."""
    g = np.random.default_rng(m + 7 * k + n)
    x = configs.to_bf16_bits(g.standard_normal((m, k), dtype=np.float32))
    if kind == abi.WEIGHT_INT8:
        q = g.integers(-128, 128, (k, n), dtype=np.int16).astype(np.int8).view(np.uint8)
    else:
        q = configs.to_e4m3_codes(g.standard_normal((k, n), dtype=np.float32) * 4)
        q[(q & 0x7F) == 0x7F] ^= 1
        if nan:
            q[g.integers(0, k, 20), g.integers(0, n, 20)] = 0x7F
    s = (np.abs(g.standard_normal(n)) * 1e-3 + 1e-6).astype(np.float32)
    w = QuantizedWeight(ctx, q, kind, s)
    n_pad, k_pad = -(-n // 256) * 256, -(-k // 64) * 64
    assert w.workspace_bytes(m) == n_pad * k_pad * 2 and w.workspace_bytes(1535) == 0
    xd = bf16_dev(x)
    bd = bf16_dev(configs.to_bf16_bits(g.standard_normal(n, dtype=np.float32) * 0.01))
    for f32 in (True, False):
        got = [linear_ex(ctx, w, xd, m, bd, f32, ws) for ws in (True, False)]
        if f32:
            vals = [host(t) for t in got]
            bits = [v.view(np.uint32) for v in vals]
        else:
            bits = [bf16_host(t) for t in got]
            vals = [f32_of_bf16(b) for b in bits]
        nans = [np.isnan(v) for v in vals]
        assert np.array_equal(nans[0], nans[1]), f"NaN positions differ (f32={f32})"
        assert nan or not nans[0].any()
        assert np.array_equal(bits[0][~nans[0]], bits[1][~nans[1]]), f"routes differ (f32={f32})"
    w.close()


def test_rows_do_not_depend_on_the_batch(ctx):
    """Rows computed at different offsets in a tile and in batches of different sizes come out bit
    for bit the same."""
    g = np.random.default_rng(11)
    m, k, n = 4096, 3072, 3072
    x = configs.to_bf16_bits(g.standard_normal((m, k), dtype=np.float32))
    q = g.integers(-128, 128, (k, n), dtype=np.int16).astype(np.int8).view(np.uint8)
    s = (np.abs(g.standard_normal(n)) * 0.02 / 127 + 1e-6).astype(np.float32)
    w = QuantizedWeight(ctx, q, abi.WEIGHT_INT8, s)
    xd = bf16_dev(x)
    full = host(linear_ex(ctx, w, xd, m, None, True))
    for r0, rows in ((0, 256), (3584, 512), (1000, 600), (2048, 130)):
        part = host(linear_ex(ctx, w, xd[r0:r0 + rows].contiguous(), rows, None, True))
        assert np.array_equal(part.view(np.uint32), full[r0:r0 + rows].view(np.uint32)), (r0, rows)
    w.close()


def test_products_on_two_streams_at_once(ctx):
    """Two products of one context in flight at once on two streams, each with its own workspace, both
    of config 1's shape (whose tiles take the widening inside the GEMM, with the context's readiness
    counters): every output has the bits of the same product run alone, over alternating calls."""
    g = np.random.default_rng(17)
    m, k, n = 4096, 3072, 3072
    q = g.integers(-128, 128, (k, n), dtype=np.int16).astype(np.int8).view(np.uint8)
    s = (np.abs(g.standard_normal(n)) * 0.02 / 127 + 1e-6).astype(np.float32)
    w = QuantizedWeight(ctx, q, abi.WEIGHT_INT8, s)
    xs = [bf16_dev(configs.to_bf16_bits(g.standard_normal((m, k), dtype=np.float32))) for _ in range(2)]
    refs = [bf16_host(linear_ex(ctx, w, x, m, None, False)) for x in xs]
    streams = [torch.cuda.Stream(), torch.cuda.Stream()]
    wss = [torch.empty(w.workspace_bytes(m), dtype=torch.uint8, device="cuda") for _ in range(2)]
    torch.cuda.synchronize()
    outs = []
    for call in range(6):
        i = call % 2
        with torch.cuda.stream(streams[i]):
            torch.cuda._sleep(200000)              # keeps this stream's product in flight while the next is issued
            y = torch.empty((m, n), dtype=torch.bfloat16, device="cuda")
            w.linear(xs[i], out=y, workspace=wss[i], stream=streams[i])
            outs.append((i, y))
    torch.cuda.synchronize()
    ctx.poll_errors()
    for call, (i, y) in enumerate(outs):
        assert np.array_equal(bf16_host(y), refs[i]), call
    w.close()


# ---------------------------------------------------------------------------------------------
# the benchmark configs at full size: sampled rows against fp32 CPU products


def sampled_check(ctx, case, rows=192, seed=0):
    """The full-size product on the GPU (fp32 and bf16 outputs) against fp32 CPU products of sampled
    rows, computed from the oracle's dequantized weight."""
    w = QuantizedWeight(ctx, case.codes_nk, case.kind, case.scales, published_nk=True)
    xd = bf16_dev(case.x)
    bd = bf16_dev(case.bias) if case.bias is not None else None
    wd = host(w.dequantize())
    ref_w = oracle.dequantize(np.ascontiguousarray(case.codes_nk.T), case.kind, case.scales, oracle.SCALE_F32,
                              oracle.LAYOUT_COLUMNS, case.n).reshape(case.k, case.n)
    assert np.array_equal(canonical(wd), canonical(ref_w)), "dequantized weight differs"
    idx = np.sort(np.random.default_rng(seed).choice(case.m, size=min(rows, case.m), replace=False))
    c = (torch.from_numpy(f32_of_bf16(case.x[idx])) @ torch.from_numpy(ref_w))
    if case.bias is not None:
        c = c + torch.from_numpy(f32_of_bf16(case.bias))
    y32 = host(linear_ex(ctx, w, xd, case.m, bd, True))[idx]
    y16 = f32_of_bf16(bf16_host(linear_ex(ctx, w, xd, case.m, bd, False)))[idx]
    c16 = c.to(torch.bfloat16).to(torch.float32).numpy()
    w.close()
    return rel_l2(y32, c.numpy()), rel_l2(y16, c16), float(np.max(np.abs(y16.astype(np.float64) - c16)))


def test_config1_full_size(ctx):
    e32, e16, mx = sampled_check(ctx, configs.config1())
    assert e32 <= REL_L2_F32 and e16 <= REL_L2_BF16 and mx <= MAX_ABS_BF16, (e32, e16, mx)


def test_config2_full_size(ctx):
    e32, e16, mx = sampled_check(ctx, configs.config2())
    assert e32 <= REL_L2_F32 and e16 <= REL_L2_BF16 and mx <= MAX_ABS_BF16, (e32, e16, mx)


@pytest.mark.parametrize("m", [1, 4, 16, 32])
@pytest.mark.parametrize("nk", [(12288, 4096), (4096, 12288)])
def test_config4_full_size(ctx, m, nk):
    e32, e16, mx = sampled_check(ctx, configs.config4(m, *nk), rows=m)
    assert e32 <= REL_L2_F32 and e16 <= REL_L2_BF16 and mx <= MAX_ABS_BF16, (m, nk, e32, e16, mx)


# ---------------------------------------------------------------------------------------------
# sc_linear_epilogue: the DiT block's GELU and gated residual fused into the product's epilogue


def gelu_tanh64(v: np.ndarray) -> np.ndarray:
    v = v.astype(np.float64)
    return 0.5 * v * (1.0 + np.tanh(0.7978845608028654 * (v + 0.044715 * v ** 3)))


def linear_epilogue(ctx, w, x_dev, m, bias_dev, y, op, gate=None, ws_bytes=None):
    need = w.workspace_bytes(1536) if ws_bytes is None else ws_bytes
    ws = torch.empty(max(need, 1), dtype=torch.uint8, device="cuda")
    st = torch.cuda.current_stream().cuda_stream
    return ctx.lib.sc_linear_epilogue(ctx.ptr, w.ptr, ctypes.c_void_p(x_dev.data_ptr()), m,
                                      ctypes.c_void_p(bias_dev.data_ptr() if bias_dev is not None else 0),
                                      ctypes.c_void_p(y.data_ptr()), op,
                                      ctypes.c_void_p(gate.data_ptr() if gate is not None else 0),
                                      ctypes.c_void_p(ws.data_ptr()), need, ctypes.c_void_p(st))


@pytest.mark.parametrize("kind,m,k,n", [(abi.WEIGHT_INT8, 1600, 3072, 3072),
                                        (abi.WEIGHT_INT8, 200, 512, 700),
                                        (abi.WEIGHT_E4M3, 2048, 1024, 2304)])
def test_fused_epilogues_match_the_unfused_stages(ctx, kind, m, k, n):
    """GELU: within one bf16 rounding of gelu_tanh (fp64) of the route's fp32 output v; gated
    residual: x + gate * v in two fp32 roundings (torch's order, Ops.swift:44-54) bit for bit; both
    against the oracle's fp32 product through v."""
    g = np.random.default_rng(5 * m + n)
    x = configs.to_bf16_bits(g.standard_normal((m, k), dtype=np.float32))
    s = (np.abs(g.standard_normal(n)) * 2e-4 + 1e-6).astype(np.float32)
    bias = configs.to_bf16_bits(g.standard_normal(n, dtype=np.float32) * 0.1)
    if kind == abi.WEIGHT_INT8:
        q = g.integers(-128, 128, (k, n), dtype=np.int16).astype(np.int8).view(np.uint8)
        c_ref, _ = oracle.linear_int8(x, q.view(np.int8), s, bias)
    else:
        q = configs.to_e4m3_codes(g.standard_normal((k, n), dtype=np.float32) * 4)
        q[(q & 0x7F) == 0x7F] ^= 1
        wf = oracle.dequantize(q, oracle.E4M3, s, oracle.SCALE_F32, oracle.LAYOUT_COLUMNS, n).reshape(k, n)
        c_ref, _ = oracle.linear_widened(x, wf, bias)
    w = QuantizedWeight(ctx, q, kind, s)
    xd, bd = bf16_dev(x), bf16_dev(bias)
    # v: the same operands and summation order as the fused epilogues (the widened route's fp32 output
    # where m >= 1536; the fused pair kernel's below it, the same bits).
    v = host(linear_ex(ctx, w, xd, m, bd, True, True))
    assert rel_l2(v, c_ref) <= REL_L2_F32
    h = torch.empty((m, n), dtype=torch.bfloat16, device="cuda")
    ctx.check(linear_epilogue(ctx, w, xd, m, bd, h, abi.EPI_GELU_TANH))
    ctx.poll_errors()
    hf = f32_of_bf16(bf16_host(h)).astype(np.float64)
    ref = gelu_tanh64(v)
    # the bf16 rounding, plus 2^-10 of it for the epilogue's exp-and-divide form of tanh (~2e-6 relative)
    bound = 2.0 ** -8 * (1.0 + 2.0 ** -10) * np.abs(ref) + np.abs(v) * 2.0 ** -20 + 1e-30
    assert float((np.abs(hf - ref) - bound).max()) <= 0.0, "GELU epilogue beyond one bf16 rounding"
    hr = f32_of_bf16(configs.to_bf16_bits(gelu_tanh64(c_ref).astype(np.float32)))
    assert rel_l2(hf, hr) <= REL_L2_BF16
    # one bf16 ulp, the fp32 cancellation in 1 + tanh where v is large and negative, and the spread of
    # a change of fp32 summation order (as in check_against_oracle) times max |gelu'| < 1.2
    wf = oracle.dequantize(q, kind, s, oracle.SCALE_F32, oracle.LAYOUT_COLUMNS, n).reshape(k, n)
    xf = torch.from_numpy(f32_of_bf16(x))
    spread = torch.sqrt((xf * xf) @ torch.from_numpy(wf * wf)).numpy().astype(np.float64)
    bound = 2.0 ** -7 * np.abs(hr) + 2.0 ** -20 * np.abs(c_ref) + 1.2 * 8.0 * np.sqrt(k) * 2.0 ** -24 * spread + 1e-9
    assert float((np.abs(hf - hr) - bound).max()) <= 0.0, "more than one bf16 ulp"
    # gated residual, in place on an fp32 stream
    x0 = g.standard_normal((m, n), dtype=np.float32)
    gate = (g.standard_normal(n, dtype=np.float32) * 0.5).astype(np.float32)
    resid = dev(x0.copy())
    ctx.check(linear_epilogue(ctx, w, xd, m, bd, resid, abi.EPI_GATED_RESIDUAL, dev(gate)))
    ctx.poll_errors()
    got = host(resid)
    want = x0 + gate[None, :] * v          # numpy fp32: one rounding per operation
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), "gated residual is not x + gate * v"
    want_oracle = x0.astype(np.float64) + gate.astype(np.float64) * c_ref.astype(np.float64)
    assert rel_l2(got - x0, want_oracle - x0) <= REL_L2_F32
    w.close()


def test_fused_epilogue_guards(ctx):
    g = np.random.default_rng(3)
    k, n = 256, 512
    q = g.integers(-128, 128, (k, n), dtype=np.int16).astype(np.int8).view(np.uint8)
    w = QuantizedWeight(ctx, q, abi.WEIGHT_INT8, np.full(n, 1e-3, np.float32))
    x128 = bf16_dev(configs.to_bf16_bits(g.standard_normal((128, k), dtype=np.float32)))
    x256 = bf16_dev(configs.to_bf16_bits(g.standard_normal((256, k), dtype=np.float32)))
    h = torch.empty((256, n), dtype=torch.bfloat16, device="cuda")
    r = torch.zeros((256, n), dtype=torch.float32, device="cuda")
    gate = torch.ones(n, dtype=torch.float32, device="cuda")
    assert linear_epilogue(ctx, w, x128, 128, None, h, abi.EPI_GELU_TANH) == abi.UNSUPPORTED_SHAPE
    assert linear_epilogue(ctx, w, x256, 256, None, h, abi.EPI_GELU_TANH, ws_bytes=1024) == abi.WORKSPACE_TOO_SMALL
    assert linear_epilogue(ctx, w, x256, 256, None, r, abi.EPI_GATED_RESIDUAL) == abi.INVALID_ARG
    assert linear_epilogue(ctx, w, x256, 256, None, h, 7) == abi.INVALID_ARG
    assert linear_epilogue(ctx, w, x256, 0, None, h, abi.EPI_GELU_TANH) == abi.OK
    ctx.check(linear_epilogue(ctx, w, x256, 256, None, r, abi.EPI_GATED_RESIDUAL, gate))
    ctx.poll_errors()
    w.close()


# ---------------------------------------------------------------------------------------------
# sc_linear_host: host buffers, copies overlapped with the products in chunks of rows


@pytest.mark.parametrize("m,chunk,direct", [(4096, 0, False), (4096, 1024, False), (1000, 0, False), (700, 512, False),
                                            (600, 0, False), (3, 0, False), (40, 0, False), (2000, 256, False),
                                            (4096, 0, True), (1000, 0, True), (200, 0, True), (2000, 256, True)])
def test_linear_host_has_the_device_bits(ctx, m, chunk, direct):
    """Chunked copies and products give each row the bits of the whole batch's device product."""
    g = np.random.default_rng(m + chunk)
    k, n = 768, 1280
    x = configs.to_bf16_bits(g.standard_normal((m, k), dtype=np.float32))
    q = g.integers(-128, 128, (k, n), dtype=np.int16).astype(np.int8).view(np.uint8)
    s = (np.abs(g.standard_normal(n)) * 1e-3 + 1e-6).astype(np.float32)
    w = QuantizedWeight(ctx, q, abi.WEIGHT_INT8, s)
    bd = bf16_dev(configs.to_bf16_bits(g.standard_normal(n, dtype=np.float32) * 0.01))
    x_host = torch.from_numpy(x.view(np.int16)).view(torch.bfloat16).pin_memory()
    for f32 in (False, True):
        want = linear_ex(ctx, w, bf16_dev(x), m, bd, f32, workspace=True)
        out = torch.empty((m, n), dtype=torch.float32 if f32 else torch.bfloat16).pin_memory()
        out.fill_(float("nan"))
        w.linear_host(x_host, out, bias=bd, chunk_rows=chunk, direct=direct)
        torch.cuda.synchronize()
        ctx.poll_errors()
        a = want.cpu().view(torch.int32 if f32 else torch.int16).numpy()
        b = out.view(torch.int32 if f32 else torch.int16).numpy()
        assert np.array_equal(a, b), f"m {m}, chunk {chunk}, direct {direct}, f32 {f32}: {int(np.sum(a != b))} differ"
    w.close()
