"""The DiT blocks' elementwise kernels (libsiliconed_dit) and the blocks of configs 3 and 5 on a B200,
against plain PyTorch fp32 references of the same formulas (Ops.swift, Block.swift, QwenImage21.swift).

Bars (stated here, used throughout): kernels with a bf16 output are within one bf16 rounding of the
fp32 reference (|got - ref| <= 2^-8 |ref| + 1e-6); fp32 outputs within 1e-5 relative; the blocks'
fp32 residual streams within 1e-2 relative L2 of the fp32 reference that rounds to bf16 at the same
points (the attention and the products' summation orders differ)."""
import math

import numpy as np
import pytest

from siliconed_b200 import dit_abi

torch = pytest.importorskip("torch")


def test_dit_library_exports_every_header_function():
    import ctypes
    names = dit_abi.header_functions()
    assert names == set(dit_abi.SIGNATURES), names ^ set(dit_abi.SIGNATURES)
    lib = ctypes.CDLL(dit_abi.LIB_PATH)
    for n in names:
        assert hasattr(lib, n), n


gpu = pytest.mark.gpu
needs_cuda = pytest.mark.skipif(not torch.cuda.is_available(), reason="needs a CUDA device")


def bf16_close(got, ref):
    got, ref = got.float(), ref.float()
    excess = (got - ref).abs() - (2.0 ** -8 * ref.abs() + 1e-6)
    return float(excess.max())


def rms_ref(x, w=None, eps=1e-5):
    inv = 1.0 / torch.sqrt((x * x).mean(dim=-1, keepdim=True) + eps)
    y = x * inv
    return y * w if w is not None else y


def ln_ref(x, eps=1e-6):
    c = x - x.mean(dim=-1, keepdim=True)
    return c / torch.sqrt((c * c).mean(dim=-1, keepdim=True) + eps)


def rope_ref(x, freqs):
    """x [..., S, D] fp32, freqs [S, D/2, 2] (cos, sin): adjacent pairs."""
    re, im = x[..., 0::2], x[..., 1::2]
    c, s = freqs[..., 0], freqs[..., 1]
    out = torch.empty_like(x)
    out[..., 0::2] = re * c - im * s
    out[..., 1::2] = re * s + im * c
    return out


@gpu
@needs_cuda
@pytest.mark.parametrize("rows,d", [(7, 3840), (33, 3072), (5, 4)])
def test_norm_kernels(rows, d):
    g = torch.Generator(device="cuda").manual_seed(rows + d)
    x = torch.randn(rows, d, generator=g, device="cuda") * 3
    w = 1 + 0.1 * torch.randn(d, generator=g, device="cuda")
    sc = 0.2 * torch.randn(d, generator=g, device="cuda")
    sh = 0.2 * torch.randn(d, generator=g, device="cuda")
    out = torch.empty(rows, d, dtype=torch.bfloat16, device="cuda")
    dit_abi.rms_norm_modulate(x, w, sc, 1e-5, out)
    assert bf16_close(out, rms_ref(x, w) * (1 + sc)) <= 0
    dit_abi.rms_norm_modulate(x, None, None, 1e-5, out)
    assert bf16_close(out, rms_ref(x)) <= 0
    dit_abi.layer_norm_modulate(x, sc, sh, 1e-6, out)
    assert bf16_close(out, ln_ref(x) * (1 + sc) + sh) <= 0
    dit_abi.layer_norm_modulate(x, None, None, 1e-6, out)
    assert bf16_close(out, ln_ref(x)) <= 0


@gpu
@needs_cuda
@pytest.mark.parametrize("norm,tanh", [(True, True), (False, False), (False, True)])
def test_gated_residual(norm, tanh):
    g = torch.Generator(device="cuda").manual_seed(3)
    rows, d = 9, 3072
    x = torch.randn(rows, d, generator=g, device="cuda")
    y = torch.randn(rows, d, generator=g, device="cuda") * 100
    gate = torch.randn(d, generator=g, device="cuda")
    w = 1 + 0.1 * torch.randn(d, generator=g, device="cuda")
    ref = x + (torch.tanh(gate) if tanh else gate) * (rms_ref(y, w) if norm else y)
    dit_abi.gated_residual(x, y, gate, tanh, w if norm else None, 1e-5)
    assert float(((x - ref).norm() / ref.norm())) <= 1e-5


@gpu
@needs_cuda
def test_qk_norm_rope_and_merge():
    g = torch.Generator(device="cuda").manual_seed(5)
    batch, tokens, heads, joint, off = 2, 24, 3, 40, 10
    hd = heads * 128
    qkv = (torch.randn(batch * tokens, 3 * hd, generator=g, device="cuda") * 2).to(torch.bfloat16)
    nq = 1 + 0.1 * torch.randn(128, generator=g, device="cuda")
    nk = 1 + 0.1 * torch.randn(128, generator=g, device="cuda")
    ang = torch.rand(joint, 64, generator=g, device="cuda") * 6.28
    freqs = torch.stack([torch.cos(ang), torch.sin(ang)], dim=-1).contiguous()
    q = torch.zeros(batch, heads, joint, 128, dtype=torch.bfloat16, device="cuda")
    k, v = torch.zeros_like(q), torch.zeros_like(q)
    dit_abi.qk_norm_rope(qkv, batch, tokens, heads, nq, nk, freqs, 1e-6, q, k, v, joint, off)
    parts = qkv.float().reshape(batch, tokens, 3, heads, 128).permute(2, 0, 3, 1, 4)  # [3, B, H, T, D]
    f = freqs[off:off + tokens]
    qr = rope_ref(rms_ref(parts[0], nq, 1e-6), f)
    kr = rope_ref(rms_ref(parts[1], nk, 1e-6), f)
    assert bf16_close(q[:, :, off:off + tokens], qr) <= 1e-6
    assert bf16_close(k[:, :, off:off + tokens], kr) <= 1e-6
    assert torch.equal(v[:, :, off:off + tokens], parts[2].to(torch.bfloat16))
    assert not q[:, :, :off].any() and not q[:, :, off + tokens:].any()
    out = torch.empty(batch * tokens, hd, dtype=torch.bfloat16, device="cuda")
    dit_abi.attention_merge(v, batch, heads, joint, off, tokens, out)
    assert torch.equal(out, qkv[:, 2 * hd:])


@gpu
@needs_cuda
def test_swiglu_and_gelu():
    g = torch.Generator(device="cuda").manual_seed(7)
    rows, hidden = 13, 1024
    h = (torch.randn(rows, 2 * hidden, generator=g, device="cuda") * 3).to(torch.bfloat16)
    out = torch.empty(rows, hidden, dtype=torch.bfloat16, device="cuda")
    dit_abi.swiglu(h, hidden, out)
    a, b = h[:, :hidden].float(), h[:, hidden:].float()
    assert bf16_close(out, a / (1 + torch.exp(-a)) * b) <= 1e-6
    for count in (4096, 4101):
        x = (torch.randn(count, generator=g, device="cuda") * 3).to(torch.bfloat16)
        ref = x.float()
        ref = 0.5 * ref * (1 + torch.tanh(math.sqrt(2 / math.pi) * (ref + 0.044715 * ref ** 3)))
        dit_abi.gelu_tanh(x)
        assert bf16_close(x, ref) <= 1e-6


# ------------------------------------------------------------------------------------------------
# the blocks against fp32 references that round to bf16 where the blocks do


def lin_ref(layer, a):
    w = layer.weight.dequantize()                      # fp32 [in, out] = q * s
    y = a.float() @ w
    if layer.bias is not None:
        y = y + layer.bias.float()
    return y


def attn_ref(q, k, v):
    s = (q.float() @ k.float().transpose(-1, -2)) / math.sqrt(q.shape[-1])
    return torch.softmax(s, dim=-1) @ v.float()


def rel(a, b):
    return float((a - b).norm() / b.norm())


@gpu
@needs_cuda
def test_zimage_block_matches_fp32_reference():
    from siliconed_b200.dit import ZImageBlock, rope_table, image_text_positions, timestep_embedding
    from siliconed_b200.products import Context
    ctx = Context(0)
    s, d, heads, hidden = 320, 512, 4, 1024
    blk = ZImageBlock(ctx, dim=d, heads=heads, hidden=hidden, seed=1)
    g = torch.Generator(device="cuda").manual_seed(2)
    x = torch.randn(s, d, generator=g, device="cuda")
    freqs = rope_table(image_text_positions(64, 16)).cuda()
    adaln = timestep_embedding(0.3)
    x_ref = x.clone()
    blk.forward(x, freqs, adaln)
    # reference
    bf = lambda t: t.to(torch.bfloat16).float()
    mod = lin_ref(blk.modulation, adaln).reshape(4, d)
    a = bf(rms_ref(x_ref, blk.norm1) * (1 + mod[0]))
    qkv = bf(lin_ref(blk.qkv, a)).reshape(s, 3, heads, 128).permute(1, 2, 0, 3)
    q = bf(rope_ref(rms_ref(qkv[0], blk.norm_q), freqs))
    k = bf(rope_ref(rms_ref(qkv[1], blk.norm_k), freqs))
    o = bf(attn_ref(q, k, qkv[2])).permute(1, 0, 2).reshape(s, d)
    y = lin_ref(blk.out, o)
    x_ref = x_ref + torch.tanh(mod[1]) * rms_ref(y, blk.norm2)
    a = bf(rms_ref(x_ref, blk.ffn_norm1) * (1 + mod[2]))
    from siliconed_b200.dit import deinterleave_halves, SWIGLU_BLOCK
    h = deinterleave_halves(bf(lin_ref(blk.w13, a)), SWIGLU_BLOCK)   # the weight is registered interleaved
    gg = bf(h[:, :hidden] / (1 + torch.exp(-h[:, :hidden])) * h[:, hidden:])
    y = lin_ref(blk.w2, gg)
    x_ref = x_ref + torch.tanh(mod[3]) * rms_ref(y, blk.ffn_norm2)
    assert rel(x, x_ref) <= 1e-2, rel(x, x_ref)
    blk.close()
    ctx.close()


@gpu
@needs_cuda
def test_mmdit_block_matches_fp32_reference():
    from siliconed_b200.dit import MMDiT, rope_table, image_text_positions, timestep_embedding
    from siliconed_b200.products import Context
    ctx = Context(0)
    batch, st, si, d, heads, mlp = 2, 32, 64, 256, 2, 512
    model = MMDiT(ctx, blocks=1, dim=d, heads=heads, mlp=mlp, seed=3)
    blk = model.blocks[0]
    g = torch.Generator(device="cuda").manual_seed(4)
    x_txt = torch.randn(batch * st, d, generator=g, device="cuda")
    x_img = torch.randn(batch * si, d, generator=g, device="cuda")
    freqs = rope_table(image_text_positions(st, 8)).cuda()
    temb = timestep_embedding(0.7)
    refs = [x_txt.clone(), x_img.clone()]
    b = model.buffers(batch, st, si)
    blk.forward(x_txt, x_img, batch, temb, freqs, b)
    # reference
    bf = lambda t: t.to(torch.bfloat16).float()
    streams = [(blk.txt, refs[0], st), (blk.img, refs[1], si)]
    mods, qs, ks, vs = [], [], [], []
    off = 0
    for sw, x, n in streams:
        m = lin_ref(sw.modulation, temb).reshape(6, d)
        mods.append(m)
        a = bf(ln_ref(x) * (1 + m[1]) + m[0])
        qkv = bf(lin_ref(sw.qkv, a)).reshape(batch, n, 3, heads, 128).permute(2, 0, 3, 1, 4)
        f = freqs[off:off + n]
        qs.append(bf(rope_ref(rms_ref(qkv[0], sw.norm_q, 1e-6), f)))
        ks.append(bf(rope_ref(rms_ref(qkv[1], sw.norm_k, 1e-6), f)))
        vs.append(qkv[2])
        off += n
    o = bf(attn_ref(torch.cat(qs, 2), torch.cat(ks, 2), torch.cat(vs, 2)))  # [B, H, J, D]
    off = 0
    for (sw, x, n), m in zip(streams, mods):
        on = o[:, :, off:off + n].permute(0, 2, 1, 3).reshape(batch * n, d)
        x += m[2] * lin_ref(sw.out, on)
        a = bf(ln_ref(x) * (1 + m[4]) + m[3])
        h = lin_ref(sw.mlp1, a)
        h = bf(bf(h))
        h = bf(0.5 * h * (1 + torch.tanh(math.sqrt(2 / math.pi) * (h + 0.044715 * h ** 3))))
        x += m[5] * lin_ref(sw.mlp2, h)
        off += n
    assert rel(x_txt, refs[0]) <= 1e-2, rel(x_txt, refs[0])
    assert rel(x_img, refs[1]) <= 1e-2, rel(x_img, refs[1])
    model.close()
    ctx.close()


@gpu
@needs_cuda
def test_fused_epilogues_agree_with_the_separate_stages():
    """From 1536 rows the MMDiT block's gated residuals and GELU run in the product's epilogue: the
    gated residual bit for bit as the product plus sd_gated_residual (both x + gate * v in two roundings); the GELU
    within one bf16 rounding of the product's bf16 output run through sd_gelu_tanh (the separate
    stages round v to bf16 first, which moves gelu by up to 1.2 |v| 2^-8)."""
    import siliconed_b200.dit as dit
    from siliconed_b200.products import Context
    ctx = Context(0)
    g = torch.Generator(device="cuda").manual_seed(9)
    lin = dit.Linear(ctx, 1280, 512, g, bias=True)
    rows = 2048
    x = torch.randn(rows, 512, generator=g, device="cuda").to(torch.bfloat16)
    gate = torch.randn(1280, generator=g, device="cuda")
    resid0 = torch.randn(rows, 1280, generator=g, device="cuda")
    ws = torch.empty(lin.workspace_bytes(rows), dtype=torch.uint8, device="cuda")
    scratch = torch.empty(rows, 1280, device="cuda")
    v = lin(x, torch.empty(rows, 1280, device="cuda"), ws)
    outs = {}
    try:
        for fused in (True, False):
            dit.FUSED_EPILOGUES = fused
            r = resid0.clone()
            lin.gated_residual(x, r, gate, scratch, ws)
            h = torch.empty(rows, 1280, dtype=torch.bfloat16, device="cuda")
            lin.gelu(x, h, ws)
            outs[fused] = (r, h)
    finally:
        dit.FUSED_EPILOGUES = True
    torch.cuda.synchronize()
    assert torch.equal(outs[True][0], outs[False][0])
    assert not torch.equal(outs[True][0], resid0)
    hf, hu = outs[True][1].float(), outs[False][1].float()
    excess = (hf - hu).abs() - (2.0 ** -7 * hu.abs() + 1.2 * 2.0 ** -8 * v.abs() + 1e-6)
    assert float(excess.max()) <= 0.0
    lin.close()
    ctx.close()


@gpu
@needs_cuda
def test_mmdit_block_with_fused_epilogues_matches_fp32_reference():
    """The block at 1536 text and 2048 image rows (the fused epilogues' range) against the same fp32
    reference, its GELU taken on the fp32 product as the fused epilogue does."""
    from siliconed_b200.dit import MMDiT, rope_table, image_text_positions, timestep_embedding
    from siliconed_b200.products import Context
    ctx = Context(0)
    batch, st, si, d, heads, mlp = 1, 1536, 2048, 256, 2, 512
    model = MMDiT(ctx, blocks=1, dim=d, heads=heads, mlp=mlp, seed=5)
    blk = model.blocks[0]
    g = torch.Generator(device="cuda").manual_seed(6)
    x_txt = torch.randn(batch * st, d, generator=g, device="cuda")
    x_img = torch.randn(batch * si, d, generator=g, device="cuda")
    freqs = rope_table(image_text_positions(st, 64)[: st + si]).cuda()
    temb = timestep_embedding(0.3)
    refs = [x_txt.clone(), x_img.clone()]
    b = model.buffers(batch, st, si)
    blk.forward(x_txt, x_img, batch, temb, freqs, b)
    bf = lambda t: t.to(torch.bfloat16).float()
    streams = [(blk.txt, refs[0], st), (blk.img, refs[1], si)]
    mods, qs, ks, vs = [], [], [], []
    off = 0
    for sw, x, n in streams:
        m = lin_ref(sw.modulation, temb).reshape(6, d)
        mods.append(m)
        a = bf(ln_ref(x) * (1 + m[1]) + m[0])
        qkv = bf(lin_ref(sw.qkv, a)).reshape(batch, n, 3, heads, 128).permute(2, 0, 3, 1, 4)
        f = freqs[off:off + n]
        qs.append(bf(rope_ref(rms_ref(qkv[0], sw.norm_q, 1e-6), f)))
        ks.append(bf(rope_ref(rms_ref(qkv[1], sw.norm_k, 1e-6), f)))
        vs.append(qkv[2])
        off += n
    o = bf(attn_ref(torch.cat(qs, 2), torch.cat(ks, 2), torch.cat(vs, 2)))
    off = 0
    for (sw, x, n), m in zip(streams, mods):
        on = o[:, :, off:off + n].permute(0, 2, 1, 3).reshape(batch * n, d)
        x += m[2] * lin_ref(sw.out, on)
        a = bf(ln_ref(x) * (1 + m[4]) + m[3])
        h = lin_ref(sw.mlp1, a)
        h = bf(0.5 * h * (1 + torch.tanh(math.sqrt(2 / math.pi) * (h + 0.044715 * h ** 3))))
        x += m[5] * lin_ref(sw.mlp2, h)
        off += n
    assert rel(x_txt, refs[0]) <= 1e-2, rel(x_txt, refs[0])
    assert rel(x_img, refs[1]) <= 1e-2, rel(x_img, refs[1])
    model.close()
    ctx.close()


@gpu
@needs_cuda
def test_qk_norm_rope_in_the_product_epilogue():
    """From 1536 rows the q / k / v product writes the attention's q, k, v itself (sc_linear_qk_norm_rope):
    v bit for bit as the product plus sd_qk_norm_rope, q and k within the bf16 rounding that the separate
    pass applies to its input first (relative L2 <= 5e-3, worst element <= 2 % of the largest)."""
    import siliconed_b200.dit as dit
    from siliconed_b200.products import Context
    ctx = Context(0)
    g = torch.Generator(device="cuda").manual_seed(13)
    heads, batch, tokens, joint, off = 2, 2, 1600, 1800, 200
    lin = dit.Linear(ctx, 3 * heads * 128, 256, g)
    x = torch.randn(batch * tokens, 256, generator=g, device="cuda").to(torch.bfloat16)
    norm_q = (1 + 0.1 * torch.randn(128, generator=g, device="cuda")).float()
    norm_k = (1 + 0.1 * torch.randn(128, generator=g, device="cuda")).float()
    freqs = dit.rope_table(torch.stack([torch.arange(joint), torch.arange(joint)], dim=1)).cuda()
    ws = torch.empty(lin.workspace_bytes(batch * tokens), dtype=torch.uint8, device="cuda")
    scratch = torch.empty(batch * tokens, 3 * heads * 128, dtype=torch.bfloat16, device="cuda")
    outs = {}
    try:
        for fused in (True, False):
            dit.FUSED_EPILOGUES = fused
            q, k, v = (torch.zeros(batch, heads, joint, 128, dtype=torch.bfloat16, device="cuda") for _ in range(3))
            lin.qkv_heads(x, q, k, v, norm_q, norm_k, freqs, 1e-6, batch, tokens, off, scratch, ws)
            outs[fused] = (q, k, v)
    finally:
        dit.FUSED_EPILOGUES = True
    torch.cuda.synchronize()
    ctx.poll_errors()
    (qf, kf, vf), (qu, ku, vu) = outs[True], outs[False]
    assert torch.equal(vf, vu)
    assert not vf[:, :, :off].any() and vf[:, :, off:].any()
    for a, b in ((qf, qu), (kf, ku)):
        a, b = a.float(), b.float()
        assert rel(a, b) <= 5e-3, rel(a, b)
        assert float((a - b).abs().max()) <= 0.02 * float(b.abs().max())
    lin.close()
    ctx.close()


@gpu
@needs_cuda
def test_swiglu_in_the_product_epilogue():
    """From 1536 rows the interleaved gate / up product applies SwiGLU in its epilogue (SC_EPI_SWIGLU):
    against the product's fp32 output v through silu(a) * b in fp64, within one bf16 rounding plus 2^-10
    of it for the epilogue's exp-and-divide form; against the separate pass (the product rounded to bf16,
    then sd_swiglu_blocks) within relative L2 5e-3."""
    import siliconed_b200.dit as dit
    from siliconed_b200.products import Context
    ctx = Context(0)
    g = torch.Generator(device="cuda").manual_seed(21)
    hidden, k, rows = 512, 384, 2048
    lin = dit.Linear(ctx, 2 * hidden, k, g, interleave=dit.SWIGLU_BLOCK)
    x = torch.randn(rows, k, generator=g, device="cuda").to(torch.bfloat16)
    ws = torch.empty(lin.workspace_bytes(rows), dtype=torch.uint8, device="cuda")
    scratch = torch.empty(rows, 2 * hidden, dtype=torch.bfloat16, device="cuda")
    v = dit.deinterleave_halves(lin(x, torch.empty(rows, 2 * hidden, device="cuda"), ws), dit.SWIGLU_BLOCK)
    outs = {}
    try:
        for fused in (True, False):
            dit.FUSED_EPILOGUES = fused
            out = torch.empty(rows, hidden, dtype=torch.bfloat16, device="cuda")
            lin.swiglu(x, out, scratch, ws)
            outs[fused] = out.float()
    finally:
        dit.FUSED_EPILOGUES = True
    torch.cuda.synchronize()
    ctx.poll_errors()
    a, b = v[:, :hidden].double(), v[:, hidden:].double()
    ref = a / (1 + torch.exp(-a)) * b
    bound = 2.0 ** -8 * (1 + 2.0 ** -10) * ref.abs() + (a.abs() * b.abs()) * 2.0 ** -20 + 1e-30
    assert float((outs[True].double() - ref).abs().sub(bound).max()) <= 0.0
    assert rel(outs[True], outs[False]) <= 5e-3
    lin.close()
    ctx.close()


def test_interleave_halves_round_trip():
    """The gate / up weight's interleaved registration and the product columns' inverse (CPU)."""
    from siliconed_b200.dit import interleave_halves, deinterleave_halves
    w = torch.randn(2 * 384, 40)
    wi = interleave_halves(w, 128)
    assert torch.equal(wi[:128], w[:128]) and torch.equal(wi[128:256], w[384:512])
    assert torch.equal(wi[256:384], w[128:256])
    x = torch.randn(7, 40, dtype=torch.float64)
    assert torch.allclose(deinterleave_halves(x @ wi.double().T, 128), x @ w.double().T)


@gpu
@needs_cuda
def test_product_reads_the_attention_output():
    """From 1536 rows the out projection reads the attention's output o [B, H, J, 128] itself through a 4-D
    tensor map (sc_linear_heads): the same operand rows as sd_attention_merge gathers, so the same bits, for
    fp32 and bf16 outputs and for the gated residual."""
    import siliconed_b200.dit as dit
    from siliconed_b200.products import Context
    ctx = Context(0)
    g = torch.Generator(device="cuda").manual_seed(31)
    batch, heads, joint, off, n = 2, 2, 900, 100, 768
    lin = dit.Linear(ctx, 640, heads * 128, g, bias=True)
    o = torch.randn(batch, heads, joint, 128, generator=g, device="cuda").to(torch.bfloat16)
    rows = batch * n
    ws = torch.empty(lin.workspace_bytes(rows), dtype=torch.uint8, device="cuda")
    merged = torch.empty(rows, heads * 128, dtype=torch.bfloat16, device="cuda")
    scratch = torch.empty(rows, 640, device="cuda")
    gate = torch.randn(640, generator=g, device="cuda")
    r0 = torch.randn(rows, 640, generator=g, device="cuda")
    outs = {}
    try:
        for fused in (True, False):
            dit.FUSED_EPILOGUES = fused
            y32 = lin.from_heads(o, off, n, torch.empty(rows, 640, device="cuda"), merged, ws).clone()
            y16 = lin.from_heads(o, off, n, torch.empty(rows, 640, dtype=torch.bfloat16, device="cuda"), merged, ws)
            r = r0.clone()
            lin.gated_residual_heads(o, off, n, r, gate, merged, scratch, ws)
            outs[fused] = (y32, y16.clone(), r)
    finally:
        dit.FUSED_EPILOGUES = True
    torch.cuda.synchronize()
    ctx.poll_errors()
    for a, b in zip(outs[True], outs[False]):
        assert torch.equal(a, b)
    lin.close()
    ctx.close()


@gpu
@needs_cuda
def test_gated_residual_then_rms_modulate_in_one_pass():
    """sd_gated_residual_rms_modulate gives the bits of sd_gated_residual followed by sd_rms_norm_modulate."""
    g = torch.Generator(device="cuda").manual_seed(41)
    rows, d = 37, 3840
    x0 = torch.randn(rows, d, generator=g, device="cuda")
    y = torch.randn(rows, d, generator=g, device="cuda")
    gate, nw = torch.randn(d, generator=g, device="cuda"), torch.rand(d, generator=g, device="cuda") + 0.5
    w2, sc = torch.rand(d, generator=g, device="cuda") + 0.5, torch.randn(d, generator=g, device="cuda") * 0.1
    xa, a1 = x0.clone(), torch.empty(rows, d, dtype=torch.bfloat16, device="cuda")
    dit_abi.gated_residual(xa, y, gate, True, nw, 1e-5)
    dit_abi.rms_norm_modulate(xa, w2, sc, 1e-6, a1)
    xb, a2 = x0.clone(), torch.empty(rows, d, dtype=torch.bfloat16, device="cuda")
    dit_abi.gated_residual_rms_modulate(xb, y, gate, True, nw, 1e-5, w2, sc, 1e-6, a2)
    torch.cuda.synchronize()
    assert torch.equal(xa, xb) and torch.equal(a1.view(torch.int16), a2.view(torch.int16))
