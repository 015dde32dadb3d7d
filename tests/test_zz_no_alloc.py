"""sc_linear_ex_noalloc (scratch in a static device array of the library) against sc_linear_ex (the
caller's workspace), through the C ABI on a B200.  Both run the same kernels on the same operands, so
their outputs must agree bit for bit; the check alternates different weights (A, B, A, one of them a
convrot weight whose rotated x sits in front of the widened copy inside the array) so that a stale
widened tile or rotated row left by the previous call would show, and ends with a clear refusal above
the array's 32 MiB.  Callers of this entry point are bindings that have no scratch buffer to pass and
may not allocate per call."""
import ctypes

import numpy as np
import pytest

from siliconed_b200 import abi, configs

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

if not torch.cuda.is_available():  # collected on CPU boxes, skipped there
    pytest.skip("needs a CUDA device", allow_module_level=True)

from siliconed_b200.products import Context, QuantizedWeight  # noqa: E402

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


def bits(t):
    return t.view(torch.int32 if t.dtype == torch.float32 else torch.int16)


def make_weight(ctx, kind, k, n, seed, rotation=0):
    g = np.random.default_rng(seed)
    if kind == abi.WEIGHT_INT8:
        q = g.integers(-128, 128, (k, n), dtype=np.int16).astype(np.int8).view(np.uint8)
        s = (np.abs(g.standard_normal(n)) * 0.02 / 127 + 1e-7).astype(np.float32)
    else:
        q = configs.to_e4m3_codes(g.standard_normal((k, n), dtype=np.float32) * 4)
        q[(q & 0x7F) == 0x7F] ^= 1
        s = (np.abs(g.standard_normal(n)) * 0.02 / 448 + 1e-7).astype(np.float32)
    b = configs.to_bf16_bits(g.standard_normal(n, dtype=np.float32) * 0.01)
    w = QuantizedWeight(ctx, q, kind, s, rotation=rotation)
    bd = torch.from_numpy(b.view(np.int16)).cuda().view(torch.bfloat16)
    return w, bd


def test_noalloc_matches_the_workspace_entry_point_bit_for_bit(ctx):
    # A: config 1's shape (its tiles take the widening inside the GEMM); B: e4m3 (widen, then the GEMM);
    # R: convrot (the rotated x, then the widened copy, both in the array)
    weights = {
        "A": make_weight(ctx, abi.WEIGHT_INT8, 3072, 3072, 1) + (4096,),
        "B": make_weight(ctx, abi.WEIGHT_E4M3, 2048, 1000, 2) + (2048,),
        "R": make_weight(ctx, abi.WEIGHT_INT8, 3072, 2560, 3, rotation=64) + (2048,),
    }
    g = np.random.default_rng(4)
    xs = {}
    for name, (w, _, m) in weights.items():
        need = w.workspace_bytes(m)
        assert 0 < need <= 32 << 20, (name, need)       # the widened route, inside the static scratch
        x = configs.to_bf16_bits(g.standard_normal((m, w.k), dtype=np.float32))
        xs[name] = torch.from_numpy(x.view(np.int16)).cuda().view(torch.bfloat16)
    refs = {}
    for name, (w, bd, m) in weights.items():
        for f32 in (True, False):
            refs[name, f32] = existing(ctx, w, xs[name], m, bd, f32)
    order = ["A", "B", "A", "R", "B", "R", "A"]         # consecutive calls share the array
    for f32 in (True, False):
        for call, name in enumerate(order):
            w, bd, m = weights[name]
            got = noalloc(ctx, w, xs[name], m, bd, f32)
            ctx.poll_errors()
            assert torch.equal(bits(got), bits(refs[name, f32])), (f32, call, name)
    for w, _, _ in weights.values():
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
