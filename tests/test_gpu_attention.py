"""sd_attention (this project's tcgen05 attention) against an fp32 reference on a B200.

The reference: softmax(q k^T / sqrt(128)) v in fp32 on the bf16 q, k, v (TF32 off), a few heads at a time.
The kernel rounds P to bf16 for the P . v product (relative error up to 2^-9 a probability, as the reference's
fused kernel does, TiledAttention.swift:570-576) and o to bf16, so the bars are: relative L2 of the whole output
<= 4e-3, of every head <= 6e-3, and max-abs <= 2^-6 * max|v| (about 1.6e-3 relative L2 expected from the two
roundings).  The library attention (torch's fused SDPA on the same bf16 inputs) meets the same bars, and the
two must agree within them.  Shapes: ragged sequences (the last key tile and the last query tile partly past
the sequence), peaked scores whose row maximum keeps rising along the keys, and rising far enough that the kernel
takes the maximum again and rescales O, and configs 3 and 5 at their benchmarked sizes.
"""
import math

import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

if not torch.cuda.is_available():  # collected on CPU boxes, skipped there
    pytest.skip("needs a CUDA device", allow_module_level=True)

from siliconed_b200 import dit_abi  # noqa: E402

REL_L2, REL_L2_HEAD, MAX_ABS_OF_V = 4e-3, 6e-3, 2.0 ** -6


@pytest.fixture(autouse=True)
def _fp32_products():
    old = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    yield
    torch.backends.cuda.matmul.allow_tf32 = old


def reference(q, k, v):
    out = torch.empty(q.shape, dtype=torch.float32, device=q.device)
    scale = 1.0 / math.sqrt(q.shape[-1])
    for b in range(q.shape[0]):
        for h0 in range(0, q.shape[1], 6):
            qs, ks, vs = (t[b, h0:h0 + 6].float() for t in (q, k, v))
            out[b, h0:h0 + 6] = torch.softmax((qs @ ks.transpose(-1, -2)) * scale, dim=-1) @ vs
    return out


def ours(q, k, v):
    o = torch.empty_like(q)
    dit_abi.attention(q, k, v, o, 1.0 / math.sqrt(q.shape[-1]))
    torch.cuda.synchronize()
    assert dit_abi.attention_errors() == (0, 0)
    return o


def check(got, ref, v, label):
    g, r = got.double(), ref.double()
    total = float((g - r).norm() / r.norm())
    heads = ((g - r).flatten(2).norm(dim=-1) / r.flatten(2).norm(dim=-1).clamp_min(1e-30)).max().item()
    mx = float((g - r).abs().max())
    bound = MAX_ABS_OF_V * float(v.float().abs().max())
    print(f"{label}: rel-L2 {total:.2e}, worst head {heads:.2e}, max-abs {mx:.2e} (bound {bound:.2e})")
    assert torch.isfinite(got.float()).all(), label
    assert total <= REL_L2, (label, total)
    assert heads <= REL_L2_HEAD, (label, heads)
    assert mx <= bound, (label, mx, bound)


def operands(b, h, s, seed, q_scale=1.0):
    g = torch.Generator(device="cuda").manual_seed(seed)
    q, k, v = (torch.randn(b, h, s, 128, generator=g, device="cuda") for _ in range(3))
    return (q * q_scale).to(torch.bfloat16), k.to(torch.bfloat16), v.to(torch.bfloat16)


@pytest.mark.parametrize("b,h,s", [(1, 1, 128), (1, 2, 256), (2, 3, 200), (1, 4, 1000), (1, 1, 1), (1, 2, 129)])
def test_attention_matches_fp32(b, h, s):
    q, k, v = operands(b, h, s, seed=s + 7 * h)
    check(ours(q, k, v), reference(q, k, v), v, f"[{b}, {h}, {s}]")


def test_attention_with_rising_peaks_rescales():
    """Scores that grow along the keys (k's norm rising with the position) and a sharp softmax: each key tile
    raises the rows' maximum, and the later tiles' exponentials under the first tile's maximum run far above 1
    (kept as they are while their sum stays below the kernel's threshold)."""
    b, h, s = 1, 4, 1024
    q, k, v = operands(b, h, s, seed=3, q_scale=2.0)
    ramp = torch.linspace(0.5, 3.0, s, device="cuda").view(1, 1, s, 1)
    k = (k.float() * ramp).to(torch.bfloat16)
    check(ours(q, k, v), reference(q, k, v), v, "rising peaks")


def test_attention_with_a_maximum_that_jumps_far():
    """Scores whose row maximum rises by far more than 2^32 across the keys (q scaled by 4, k's norm rising 0.25 ->
    4): the tiles' sums cross the threshold at which the kernel takes the maximum again, redoes the tile and
    rescales O; keys past the sequence in the last tile too."""
    b, h, s = 1, 2, 1000
    q, k, v = operands(b, h, s, seed=5, q_scale=4.0)
    ramp = torch.linspace(0.25, 4.0, s, device="cuda").view(1, 1, s, 1)
    k = (k.float() * ramp).to(torch.bfloat16)
    check(ours(q, k, v), reference(q, k, v), v, "jumping maximum")


def test_attention_is_deterministic_and_agrees_with_the_library():
    q, k, v = operands(2, 8, 1536, seed=11)
    a, b = ours(q, k, v), ours(q, k, v)
    assert torch.equal(a.view(torch.int16), b.view(torch.int16)), "the same bits on a second call"
    lib = torch.nn.functional.scaled_dot_product_attention(q, k, v)
    ref = reference(q, k, v)
    check(lib, ref, v, "library")
    check(a, lib.float(), v, "ours vs library")


@pytest.mark.parametrize("b,h,s,label", [(1, 30, 4608, "config 3"), (2, 24, 4352, "config 5 (2 images)")])
def test_attention_at_the_benchmarked_shapes(b, h, s, label):
    q, k, v = operands(b, h, s, seed=h * s)
    check(ours(q, k, v), reference(q, k, v), v, label)


def test_attention_refuses_bad_arguments():
    q = torch.zeros(1, 1, 128, 64, dtype=torch.bfloat16, device="cuda")
    lib = dit_abi.load()
    p = q.data_ptr()
    assert lib.sd_attention(p, p, p, p, 1, 128, 64, 0.125, None) == 1, "head_dim 64"
    assert lib.sd_attention(p, p, p, p, 1, 0, 128, 0.125, None) == 1, "empty sequence"
    assert lib.sd_attention(p + 2, p, p, p, 1, 128, 128, 0.125, None) == 1, "unaligned q"
    assert lib.sd_attention(p, p, p, p, 1, 128, 128, 0.0, None) == 1, "zero scale"
