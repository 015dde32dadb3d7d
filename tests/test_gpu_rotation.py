"""convrot (ComfyUI's rotated int8 maps) on a B200, through the C ABI, against the oracle.

Bars: the activation's rotation (sc_rotate_activation) and the rotated weight's export (sc_dequantize)
bit-exact against the oracle's restatements of rotate_groups (TensorGEMM.swift:183-201) and
Widen.dequantizeRotated (Widen.swift:374-428); the rotated products against the oracle's native int8
route on the oracle's rotated operand with the bars of test_gpu_linear (fp32 relative L2 <= 1e-5, bf16
relative L2 <= 1e-3 and within one bf16 ulp plus the summation-order spread), and against the fp64
product with the rotated fp32 weight within the bf16 rounding of the operand (relative L2 <= 5e-3).
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

from siliconed_b200.products import Context, QuantizedWeight, rotate_activation  # noqa: E402

REL_L2_BF16, REL_L2_F32 = 1e-3, 1e-5


@pytest.fixture(scope="module")
def ctx():
    c = Context(0)
    yield c
    c.close()


def bf16_dev(bits: np.ndarray):
    return torch.from_numpy(np.ascontiguousarray(bits.astype(np.uint16)).view(np.int16)).cuda().view(torch.bfloat16)


def bf16_host(t) -> np.ndarray:
    return t.view(torch.int16).cpu().numpy().view(np.uint16)


def rel_l2(got, ref) -> float:
    got, ref = np.asarray(got, np.float64), np.asarray(ref, np.float64)
    return float(np.linalg.norm(got - ref) / max(np.linalg.norm(ref), 1e-300))


@pytest.mark.parametrize("g,m,k", [(256, 37, 768), (64, 5, 192), (16, 3, 48), (4, 9, 8), (256, 64, 3072),
                                   (4, 2, 1000), (256, 300, 1280)])
def test_rotate_activation_is_bit_exact(ctx, g, m, k):
    rng = np.random.default_rng(g + m + k)
    x = configs.to_bf16_bits(rng.standard_normal((m, k), dtype=np.float32) * 3)
    got = bf16_host(rotate_activation(ctx, bf16_dev(x), g))
    torch.cuda.synchronize()
    want = oracle.rotate_groups_bf16(x, g)
    assert np.array_equal(got, want), f"G {g}, [{m}, {k}]: {int(np.sum(got != want))} differ"


@pytest.mark.parametrize("g,k,n", [(256, 768, 328), (64, 192, 136), (16, 32, 8200), (4, 8, 20), (256, 3072, 1000)])
def test_rotated_dequantize_is_bit_exact(ctx, g, k, n):
    rng = np.random.default_rng(g * 7 + n)
    q = rng.integers(-128, 128, (k, n), dtype=np.int16).astype(np.int8)
    h0 = np.array([1, 1, 1, -1], np.int64)
    first = h0
    while first.size < g:
        first = np.kron(first, h0)
    q[:g, 0] = np.where(first > 0, 127, -128)   # the extremes of m = H . q (H's first row)
    s32 = (np.abs(rng.standard_normal(n)) * 1e-3 + 1e-6).astype(np.float32)
    sb = configs.to_bf16_bits(s32)
    sb_t = torch.from_numpy(sb.view(np.int16).copy()).view(torch.bfloat16)
    for scales, s_f32 in ((s32, s32), (sb_t, oracle.bf16_to_f32(sb)), (s32[:1].reshape(()), np.full(n, s32[0], np.float32))):
        w = QuantizedWeight(ctx, q.view(np.uint8), abi.WEIGHT_INT8, scales, rotation=g)
        got = w.dequantize().cpu().numpy()
        want = oracle.dequantize_rotated(q, g, s_f32)
        assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), f"G {g}, [{k}, {n}]"
        w.close()


@pytest.mark.parametrize("m,k,n", [(1, 3072, 1000), (3, 768, 4096), (16, 3072, 3072), (200, 768, 1280),
                                   (1600, 3072, 3072)])
def test_rotated_products_match_oracle(ctx, m, k, n):
    g = 256
    rng = np.random.default_rng(m + k + n)
    x = configs.to_bf16_bits(rng.standard_normal((m, k), dtype=np.float32))
    q = rng.integers(-128, 128, (k, n), dtype=np.int16).astype(np.int8)
    s = (np.abs(rng.standard_normal(n)) * 0.02 * np.sqrt(768.0 / k) / 127 + 1e-7).astype(np.float32)
    b = configs.to_bf16_bits(rng.standard_normal(n, dtype=np.float32) * 0.01)
    w = QuantizedWeight(ctx, q.view(np.uint8), abi.WEIGHT_INT8, s, rotation=g)
    need = w.workspace_bytes(m)
    assert need >= m * k * 2
    xr = oracle.rotate_groups_bf16(x, g)
    c_ref, y_ref = oracle.linear_int8(xr, q, s, b)
    xd, bd = bf16_dev(x), bf16_dev(b)
    y32 = torch.empty((m, n), dtype=torch.float32, device="cuda")
    y16 = torch.empty((m, n), dtype=torch.bfloat16, device="cuda")
    w.linear_ex(xd, y32, bias=bd)
    w.linear_ex(xd, y16, bias=bd)
    ctx.poll_errors()
    got32 = y32.cpu().numpy()
    assert rel_l2(got32, c_ref) <= REL_L2_F32
    yf = oracle.bf16_to_f32(bf16_host(y16)).astype(np.float64)
    assert rel_l2(yf, oracle.bf16_to_f32(y_ref)) <= REL_L2_BF16
    xf = torch.from_numpy(oracle.bf16_to_f32(xr))
    wq = torch.from_numpy(q.astype(np.float32) * s)
    spread = torch.sqrt((xf * xf) @ (wq * wq)).numpy().astype(np.float64)
    bound = 2.0 ** -7 * np.abs(c_ref) + 8.0 * np.sqrt(k) * 2.0 ** -24 * spread + 1e-9
    assert float((np.abs(yf - c_ref) - bound).max()) <= 0.0, "more than one bf16 ulp from the fp32 result"
    # the rotated weight itself: x . W_rot in fp64, W_rot = float(H q) * s / sqrt(G)
    wr = oracle.dequantize_rotated(q, g, s).astype(np.float64)
    witness = oracle.bf16_to_f32(x).astype(np.float64) @ wr + oracle.bf16_to_f32(b)
    assert rel_l2(got32, witness) <= 5e-3
    if m > 128:
        # the fused gated residual on the same rotated operand: x + gate * v
        gate = torch.randn(n, device="cuda")
        r0 = torch.randn(m, n, device="cuda")
        r = r0.clone()
        w.linear_epilogue(xd, r, abi.EPI_GATED_RESIDUAL, bias=bd, gate=gate,
                          workspace=torch.empty(w.epilogue_workspace_bytes(m), dtype=torch.uint8, device="cuda"))
        ctx.poll_errors()
        want = (gate.double() * y32.double() + r0.double()).float()
        assert float((r - want).abs().max()) <= float(want.abs().max()) * 2.0 ** -22
    w.close()


def test_rotation_guards(ctx):
    rng = np.random.default_rng(1)
    q = rng.integers(-128, 128, (512, 256), dtype=np.int16).astype(np.int8).view(np.uint8)
    s = np.full(256, 1e-3, np.float32)
    w = QuantizedWeight(ctx, q, abi.WEIGHT_INT8, s)
    for group, status in ((128, abi.UNSUPPORTED_SHAPE), (1024, abi.UNSUPPORTED_SHAPE), (2, abi.UNSUPPORTED_SHAPE)):
        assert ctx.lib.sc_weight_set_rotation(ctx.ptr, w.ptr, group) == status
    w.close()
    w = QuantizedWeight(ctx, q[:320], abi.WEIGHT_INT8, s)           # K = 320: not a multiple of 256
    assert ctx.lib.sc_weight_set_rotation(ctx.ptr, w.ptr, 256) == abi.UNSUPPORTED_SHAPE
    assert ctx.lib.sc_weight_set_rotation(ctx.ptr, w.ptr, 64) == abi.OK
    w.close()
    e = QuantizedWeight(ctx, configs.to_e4m3_codes(rng.standard_normal((512, 256), dtype=np.float32)), abi.WEIGHT_E4M3, s)
    assert ctx.lib.sc_weight_set_rotation(ctx.ptr, e.ptr, 256) == abi.INVALID_ARG
    e.close()
    # 2^-123 is a normal int8 product, but 2^-123 / 16 is not (QuantizedMapTests.swift:464-469)
    tiny = QuantizedWeight(ctx, q, abi.WEIGHT_INT8, np.full(256, 2.0 ** -123, np.float32))
    assert ctx.lib.sc_weight_set_rotation(ctx.ptr, tiny.ptr, 256) == abi.REFUSED
    tiny.close()
    # a rotated product needs its workspace
    w = QuantizedWeight(ctx, q, abi.WEIGHT_INT8, s, rotation=256)
    x = torch.zeros((64, 512), dtype=torch.bfloat16, device="cuda")
    y = torch.empty((64, 256), dtype=torch.bfloat16, device="cuda")
    st = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    status = ctx.lib.sc_linear(ctx.ptr, w.ptr, ctypes.c_void_p(x.data_ptr()), 64, None, ctypes.c_void_p(y.data_ptr()),
                               None, 0, st)
    assert status == abi.WORKSPACE_TOO_SMALL
    ctx.poll_errors()
    w.close()
