"""sc_linear_ex_noalloc (scratch in a static device array of the library) against sc_linear_ex (the
caller's workspace), through the C ABI on a B200: the same outputs within the bars of
test_gpu_linear.py (fp32: relative L2 <= 1e-5; bf16: relative L2 <= 1e-3 and max-abs <= 2e-2), on
two calls in a row that share the array, and a clear refusal above the array's 32 MiB."""
import ctypes

import numpy as np
import pytest

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


def _ptr(t):
    return ctypes.c_void_p(t.data_ptr() if t is not None else 0)


def existing(ctx, w, x, m, b, f32):
    out = torch.empty((m, w.n), dtype=torch.float32 if f32 else torch.bfloat16, device="cuda")
    need = w.workspace_bytes(m)
    ws = torch.empty(need, dtype=torch.uint8, device="cuda") if need else None
    st = torch.cuda.current_stream().cuda_stream
    ctx.check(ctx.lib.sc_linear_ex(ctx.ptr, w.ptr, _ptr(x), m, _ptr(b), _ptr(out),
                                   abi.OUT_F32 if f32 else abi.OUT_BF16, _ptr(ws), need, ctypes.c_void_p(st)))
    return out


def noalloc(ctx, w, x, m, b, f32):
    out = torch.empty((m, w.n), dtype=torch.float32 if f32 else torch.bfloat16, device="cuda")
    st = torch.cuda.current_stream().cuda_stream
    ctx.check(ctx.lib.sc_linear_ex_noalloc(ctx.ptr, w.ptr, _ptr(x), m, _ptr(b), _ptr(out),
                                           abi.OUT_F32 if f32 else abi.OUT_BF16, ctypes.c_void_p(st)))
    return out


def as_f64(t):
    if t.dtype == torch.bfloat16:
        t = t.float()
    return t.cpu().numpy().astype(np.float64)


def rel_l2(a, b):
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-300))


@pytest.mark.parametrize("kind,m,k,n", [(abi.WEIGHT_INT8, 2048, 3072, 3072), (abi.WEIGHT_E4M3, 1600, 2048, 1000)])
def test_noalloc_matches_the_workspace_entry_point(ctx, kind, m, k, n):
    g = np.random.default_rng(m + k + n)
    x = configs.to_bf16_bits(g.standard_normal((m, k), dtype=np.float32))
    if kind == abi.WEIGHT_INT8:
        q = g.integers(-128, 128, (k, n), dtype=np.int16).astype(np.int8).view(np.uint8)
        s = (np.abs(g.standard_normal(n)) * 0.02 / 127 + 1e-7).astype(np.float32)
    else:
        q = configs.to_e4m3_codes(g.standard_normal((k, n), dtype=np.float32) * 4)
        q[(q & 0x7F) == 0x7F] ^= 1
        s = (np.abs(g.standard_normal(n)) * 0.02 / 448 + 1e-7).astype(np.float32)
    b = configs.to_bf16_bits(g.standard_normal(n, dtype=np.float32) * 0.01)
    w = QuantizedWeight(ctx, q, kind, s)
    assert 0 < w.workspace_bytes(m) <= 32 << 20      # the widened route, inside the static scratch
    xd = torch.from_numpy(x.view(np.int16)).cuda().view(torch.bfloat16)
    bd = torch.from_numpy(b.view(np.int16)).cuda().view(torch.bfloat16)
    for f32 in (True, False):
        ref = as_f64(existing(ctx, w, xd, m, bd, f32))
        for call in range(2):                         # two calls in a row share the array
            got = as_f64(noalloc(ctx, w, xd, m, bd, f32))
            ctx.poll_errors()
            e = rel_l2(got, ref)
            if f32:
                assert e <= REL_L2_F32, (call, e)
            else:
                mx = float(np.max(np.abs(got - ref)))
                assert e <= REL_L2_BF16 and mx <= MAX_ABS_BF16, (call, e, mx)
    w.close()


def test_noalloc_refuses_scratch_beyond_its_array(ctx):
    k, n = 4096, 4352                                 # widened copy: 4352 * 4096 * 2 bytes > 32 MiB
    q = np.zeros((k, n), np.uint8)
    w = QuantizedWeight(ctx, q, abi.WEIGHT_INT8, np.full(n, 1e-3, np.float32))
    m = 2048
    assert w.workspace_bytes(m) > 32 << 20
    x = torch.zeros((m, k), dtype=torch.bfloat16, device="cuda")
    y = torch.full((m, n), 7.0, dtype=torch.bfloat16, device="cuda")
    st = torch.cuda.current_stream().cuda_stream
    status = ctx.lib.sc_linear_ex_noalloc(ctx.ptr, w.ptr, _ptr(x), m, None, _ptr(y), abi.OUT_BF16,
                                          ctypes.c_void_p(st))
    assert status == abi.UNSUPPORTED_SHAPE
    assert b"static scratch" in ctx.lib.sc_last_error_string(ctx.ptr)
    assert bool((y == 7.0).all())                    # nothing ran
    w.close()
