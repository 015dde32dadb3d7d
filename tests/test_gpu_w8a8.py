"""W8A8 (the int8 weight times the activation quantized to int8 per row) on a B200, through the C ABI.

Bars: every step is one rounding the oracle makes the same (W8A8KernelTests.swift compares for equality),
so the codes, the row scales and the outputs (fp32 and bf16, with and without bias) are compared bit for
bit with the oracle's recipe (oracle.w8a8_quantize, oracle.linear_w8a8).
"""
import ctypes

import numpy as np
import pytest

import oracle
from siliconed_b200 import abi, configs

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

if not torch.cuda.is_available():  # collected on CPU boxes, skipped there
    pytest.skip("needs a CUDA device", allow_module_level=True)

from siliconed_b200.products import Context, QuantizedWeight, quantize_rows  # noqa: E402


@pytest.fixture(scope="module")
def ctx():
    c = Context(0)
    yield c
    c.close()


def recipe_inputs(m, k, seed):
    """Rows in +-3 with a row of zeros (its scale the recipe's floor) and a massive column
    (W8A8KernelTests.swift:22-24)."""
    rng = np.random.default_rng(seed)
    a = ((rng.random((m, k), dtype=np.float32) - 0.5) * 6).astype(np.float32)
    a[3 % m] = 0
    a[:, k // 3] *= 300
    return rng, a


@pytest.mark.parametrize("m,k,group", [(150, 768, 256), (70, 10240, 256), (65, 448, 64), (33, 520, 0), (9, 16, 4),
                                       (5, 32768, 256)])
@pytest.mark.parametrize("bf16_in", [False, True])
def test_quantize_rows_is_the_recipe(ctx, m, k, group, bf16_in):
    _, a = recipe_inputs(m, k, m * k + group)
    if bf16_in:
        bits = configs.to_bf16_bits(a)
        a = oracle.bf16_to_f32(bits)
        xd = torch.from_numpy(bits.view(np.int16)).cuda().view(torch.bfloat16)
    else:
        xd = torch.from_numpy(a).cuda()
    codes, sx = quantize_rows(ctx, xd, group)
    torch.cuda.synchronize()
    want_codes, want_sx = oracle.w8a8_quantize(a, group)
    assert np.array_equal(sx.cpu().numpy().view(np.uint32), want_sx.view(np.uint32))
    got = codes.cpu().numpy()
    assert np.array_equal(got, want_codes), f"{int(np.sum(got != want_codes))} codes differ"


@pytest.mark.parametrize("m,k,n,group,per_column", [(150, 768, 96, 256, True), (70, 10240, 72, 256, True),
                                                    (65, 448, 130, 64, False), (33, 520, 40, 0, True),
                                                    (600, 3072, 1000, 0, True), (1024, 3072, 3072, 256, True),
                                                    (300, 4096, 520, 16, True),
                                                    # 150 pair tiles over 74 pairs: the last round in pieces
                                                    (2560, 512, 3840, 0, True)])
def test_w8a8_products_are_the_recipe(ctx, m, k, n, group, per_column):
    rng, a = recipe_inputs(m, k, m + k + n)
    q = np.rint((rng.random((k, n), dtype=np.float32) - 0.5) * 254).astype(np.int8)
    sw = ((np.abs(rng.random(n if per_column else 1, dtype=np.float32) - 0.5) + 0.01) / 64).astype(np.float32)
    w = QuantizedWeight(ctx, q.view(np.uint8), abi.WEIGHT_INT8, sw if per_column else sw.reshape(()), rotation=group)
    codes, sx = oracle.w8a8_quantize(a, group)
    b = configs.to_bf16_bits(rng.standard_normal(n, dtype=np.float32))
    c_nb, _ = oracle.linear_w8a8(codes, sx, q, sw)
    c_b, y_b = oracle.linear_w8a8(codes, sx, q, sw, b)
    xd = torch.from_numpy(a).cuda()
    bd = torch.from_numpy(b.view(np.int16)).cuda().view(torch.bfloat16)
    y32 = torch.empty((m, n), dtype=torch.float32, device="cuda")
    w.linear_w8a8(xd, y32)
    got = y32.cpu().numpy()
    assert np.array_equal(got.view(np.uint32), c_nb.view(np.uint32)), f"{int(np.sum(got != c_nb))} of {m * n} differ"
    w.linear_w8a8(xd, y32, bias=bd)
    got = y32.cpu().numpy()
    assert np.array_equal(got.view(np.uint32), c_b.view(np.uint32)), "with bias"
    y16 = torch.empty((m, n), dtype=torch.bfloat16, device="cuda")
    w.linear_w8a8(xd, y16, bias=bd)
    assert np.array_equal(y16.view(torch.int16).cpu().numpy().view(np.uint16), y_b), "bf16 output"
    ctx.poll_errors()
    w.close()


def test_w8a8_guards(ctx):
    rng = np.random.default_rng(2)
    s = np.full(64, 1e-3, np.float32)
    e = QuantizedWeight(ctx, configs.to_e4m3_codes(rng.standard_normal((256, 64), dtype=np.float32)), abi.WEIGHT_E4M3, s)
    x = torch.zeros((8, 256), dtype=torch.float32, device="cuda")
    y = torch.empty((8, 64), dtype=torch.float32, device="cuda")
    ws = torch.empty(1 << 20, dtype=torch.uint8, device="cuda")
    st = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    P = ctypes.c_void_p
    call = lambda w, nbytes: ctx.lib.sc_linear_w8a8(ctx.ptr, w.ptr, P(x.data_ptr()), abi.IN_F32, 8, None, P(y.data_ptr()),
                                                  abi.OUT_F32, P(ws.data_ptr()), nbytes, st)
    assert call(e, ws.numel()) == abi.INVALID_ARG
    e.close()
    w = QuantizedWeight(ctx, rng.integers(-127, 128, (256, 64), dtype=np.int16).astype(np.int8).view(np.uint8),
                        abi.WEIGHT_INT8, s)
    assert call(w, 1024) == abi.WORKSPACE_TOO_SMALL
    assert call(w, ws.numel()) == abi.OK
    ctx.poll_errors()
    w.close()
    big = QuantizedWeight(ctx, np.zeros((32776, 16), np.uint8), abi.WEIGHT_INT8, np.full(16, 1e-3, np.float32))
    xb = torch.zeros((1, 32776), dtype=torch.float32, device="cuda")
    yb = torch.empty((1, 16), dtype=torch.float32, device="cuda")
    status = ctx.lib.sc_linear_w8a8(ctx.ptr, big.ptr, P(xb.data_ptr()), abi.IN_F32, 1, None, P(yb.data_ptr()),
                                    abi.OUT_F32, P(ws.data_ptr()), ws.numel(), st)
    assert status == abi.UNSUPPORTED_SHAPE
    big.close()
