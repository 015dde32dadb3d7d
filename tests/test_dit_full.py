"""The DiT blocks of configs 3 and 5 at their benchmarked shapes on a B200, against fp32 references.

Config 3: one Z-Image single-stream block (Block.swift:286-376), d 3840, 30 x 128 heads, SwiGLU 10240,
4096 image + 512 text tokens.  Config 5: one double-stream MMDiT block (QwenImage21.swift:1096-1106 for
the shapes), d 3072, 24 x 128 heads, MLP 12288 GELU (tanh), 4096 image + 256 text tokens, 2 images.

The references run in fp32 on the GPU (TF32 off): every linear is x . float(q) * s (+ bias) on the
library's own exported weight, the attention is softmax(q k^T / sqrt(128)) v in fp32 on the bf16 q, k, v,
and values are rounded to bf16 exactly where the blocks round them.  Where a block fuses a stage into a
product's epilogue (from FUSE_MIN_ROWS rows), the reference applies it to the fp32 product, as the epilogue
does (QK-norm + RoPE, SwiGLU, GELU); below that row count it rounds the product to bf16 first, as the
separate pass does.

What is compared is each block's increment to the fp32 residual stream, x_out - x_in (the stream itself
is dominated by its input, which both sides share).  Bars, stated here: relative L2 of the whole
increment <= 5e-3, and in every channel (column of d) relative L2 <= 1e-2.  The products alone meet 1e-3
against their oracle; the rest is the attention's: the fused attention multiplies v by its probabilities
rounded to bf16 (relative error up to 2^-9 each, about 1.1e-3 on the output for diffuse attention), where
the reference keeps them in fp32.  Measured on B200: config 3 2.5e-3 (worst channel 2.9e-3); config 5
1.3e-3 text, 1.2e-3 image (worst channels 4.8e-3, 5.5e-3).
"""
import math

import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

if not torch.cuda.is_available():  # collected on CPU boxes, skipped there
    pytest.skip("needs a CUDA device", allow_module_level=True)

import siliconed_b200.dit as dit  # noqa: E402
from siliconed_b200.products import Context  # noqa: E402

REL_L2_INCREMENT = 5e-3
REL_L2_CHANNEL = 1e-2


@pytest.fixture(autouse=True)
def _fp32_products():
    old = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    yield
    torch.backends.cuda.matmul.allow_tf32 = old


def bf(t):
    return t.to(torch.bfloat16).float()


def rms_ref(x, w=None, eps=1e-5):
    y = x * (1.0 / torch.sqrt((x * x).mean(dim=-1, keepdim=True) + eps))
    return y * w if w is not None else y


def ln_ref(x, eps=1e-6):
    c = x - x.mean(dim=-1, keepdim=True)
    return c / torch.sqrt((c * c).mean(dim=-1, keepdim=True) + eps)


def rope_ref(x, freqs):
    re, im = x[..., 0::2], x[..., 1::2]
    c, s = freqs[..., 0], freqs[..., 1]
    out = torch.empty_like(x)
    out[..., 0::2] = re * c - im * s
    out[..., 1::2] = re * s + im * c
    return out


def gelu_ref(h):
    return 0.5 * h * (1 + torch.tanh(math.sqrt(2 / math.pi) * (h + 0.044715 * h ** 3)))


def lin_ref(layer, a):
    y = a.float() @ layer.weight.dequantize()        # the library's own export: float(q) * s, bit-exact
    if layer.bias is not None:
        y = y + layer.bias.float()
    return y


def attn_ref(q, k, v):
    """fp32 attention over [B, H, S, 128] (bf16-valued inputs), a few heads at a time."""
    out = torch.empty(q.shape, dtype=torch.float32, device=q.device)
    scale = 1.0 / math.sqrt(q.shape[-1])
    for b in range(q.shape[0]):
        for h0 in range(0, q.shape[1], 6):
            qs, ks, vs = (t[b, h0:h0 + 6].float() for t in (q, k, v))
            p = torch.softmax((qs @ ks.transpose(-1, -2)) * scale, dim=-1)
            out[b, h0:h0 + 6] = p @ vs
    return out


def fused(rows):
    return dit.FUSED_EPILOGUES and rows >= dit.FUSE_MIN_ROWS


def qk_ref(qkv32, rows, norm_q, norm_k, freqs, eps):
    """q, k, v of a q / k / v product [B, n, 3, H, 128] (fp32): QK-norm + RoPE from the fp32 product when
    the epilogue does it, else from its bf16 rounding."""
    src = qkv32 if fused(rows) else bf(qkv32)
    parts = src.permute(2, 0, 3, 1, 4)                # [3, B, H, n, 128]
    q = bf(rope_ref(rms_ref(parts[0], norm_q, eps), freqs))
    k = bf(rope_ref(rms_ref(parts[1], norm_k, eps), freqs))
    return q, k, bf(parts[2])


def compare(x, x0, x_ref):
    got, ref = (x - x0).double(), (x_ref - x0).double()
    total = float((got - ref).norm() / ref.norm())
    per_channel = ((got - ref).norm(dim=0) / ref.norm(dim=0).clamp_min(1e-30)).max().item()
    return total, per_channel


def test_zimage_block_at_config3_shape():
    """Config 3's block: S 4608 (4096 image + 512 text), d 3840, 30 heads, SwiGLU 10240."""
    ctx = Context(0)
    s_img, s_txt, d, heads, hidden = 4096, 512, 3840, 30, 10240
    s = s_img + s_txt
    blk = dit.ZImageBlock(ctx, dim=d, heads=heads, hidden=hidden, seed=11)
    g = torch.Generator(device="cuda").manual_seed(12)
    x0 = torch.randn(s, d, generator=g, device="cuda")
    freqs = dit.rope_table(dit.image_text_positions(s_txt, 64)).cuda()
    adaln = dit.timestep_embedding(0.4)
    x = x0.clone()
    blk.forward(x, freqs, adaln)
    torch.cuda.synchronize()
    ctx.poll_errors()

    mod = lin_ref(blk.modulation, adaln).reshape(4, d)
    xr = x0.clone()
    a = bf(rms_ref(xr, blk.norm1) * (1 + mod[0]))
    q, k, v = qk_ref(lin_ref(blk.qkv, a).reshape(1, s, 3, heads, 128), s, blk.norm_q, blk.norm_k, freqs, blk.eps)
    o = bf(attn_ref(q, k, v)).permute(0, 2, 1, 3).reshape(s, d)
    y = lin_ref(blk.out, o)
    xr = xr + torch.tanh(mod[1]) * rms_ref(y, blk.norm2)
    a = bf(rms_ref(xr, blk.ffn_norm1) * (1 + mod[2]))
    h = dit.deinterleave_halves(lin_ref(blk.w13, a), dit.SWIGLU_BLOCK)
    if not fused(s):
        h = bf(h)
    gg = bf(h[:, :hidden] / (1 + torch.exp(-h[:, :hidden])) * h[:, hidden:])
    y = lin_ref(blk.w2, gg)
    xr = xr + torch.tanh(mod[3]) * rms_ref(y, blk.ffn_norm2)

    total, channel = compare(x, x0, xr)
    print(f"config 3 block: increment rel-L2 {total:.3e}, worst channel {channel:.3e}")
    assert total <= REL_L2_INCREMENT, total
    assert channel <= REL_L2_CHANNEL, channel
    blk.close()
    ctx.close()


def test_mmdit_block_at_config5_shape():
    """Config 5's block: d 3072, 24 heads, MLP 12288, 256 text + 4096 image tokens per image, 2 images
    (text rows 512: the separate stages; image rows 8192: the fused epilogues)."""
    ctx = Context(0)
    batch, st, si, d, heads, mlp = 2, 256, 4096, 3072, 24, 12288
    model = dit.MMDiT(ctx, blocks=1, dim=d, heads=heads, mlp=mlp, seed=21)
    blk = model.blocks[0]
    g = torch.Generator(device="cuda").manual_seed(22)
    x_txt0 = torch.randn(batch * st, d, generator=g, device="cuda")
    x_img0 = torch.randn(batch * si, d, generator=g, device="cuda")
    freqs = dit.rope_table(dit.image_text_positions(st, 64)).cuda()
    temb = dit.timestep_embedding(0.6)
    x_txt, x_img = x_txt0.clone(), x_img0.clone()
    blk.forward(x_txt, x_img, batch, temb, freqs, model.buffers(batch, st, si))
    torch.cuda.synchronize()
    ctx.poll_errors()

    refs = [x_txt0.clone(), x_img0.clone()]
    streams = [(blk.txt, refs[0], st, 0), (blk.img, refs[1], si, st)]
    mods, qs, ks, vs = [], [], [], []
    for sw, xr, n, off in streams:
        m = lin_ref(sw.modulation, temb).reshape(6, d)
        mods.append(m)
        a = bf(ln_ref(xr) * (1 + m[1]) + m[0])
        q, k, v = qk_ref(lin_ref(sw.qkv, a).reshape(batch, n, 3, heads, 128), batch * n, sw.norm_q, sw.norm_k,
                         freqs[off:off + n], blk.eps)
        qs.append(q)
        ks.append(k)
        vs.append(v)
    o = bf(attn_ref(torch.cat(qs, 2), torch.cat(ks, 2), torch.cat(vs, 2)))   # [B, H, joint, 128]
    for (sw, xr, n, off), m in zip(streams, mods):
        rows = batch * n
        on = o[:, :, off:off + n].permute(0, 2, 1, 3).reshape(rows, d)
        xr += m[2] * lin_ref(sw.out, on)
        a = bf(ln_ref(xr) * (1 + m[4]) + m[3])
        h = lin_ref(sw.mlp1, a)
        if not fused(rows):
            h = bf(h)
        h = bf(gelu_ref(h))
        xr += m[5] * lin_ref(sw.mlp2, h)

    for name, x, x0, xr in (("text", x_txt, x_txt0, refs[0]), ("image", x_img, x_img0, refs[1])):
        total, channel = compare(x, x0, xr)
        print(f"config 5 block, {name} stream: increment rel-L2 {total:.3e}, worst channel {channel:.3e}")
        assert total <= REL_L2_INCREMENT, (name, total)
        assert channel <= REL_L2_CHANNEL, (name, channel)
    model.close()
    ctx.close()
