"""DiT blocks over the quantized linear stage: the callers on the path's far side (configs 3 and 5).

Every linear is an int8 per-channel weight in libsiliconed_cuda (``QuantizedWeight.linear_ex``);
the elementwise stages between them are libsiliconed_dit (``dit_abi``); the attention is the CUDA
library's fused scaled-dot-product attention on bf16 operands (``torch.nn.functional.
scaled_dot_product_attention``), the one stage here that is not this project's kernel.  The residual
stream stays fp32 as in the reference; the products' operands are bf16.

* ``ZImageBlock`` — config 3, the single-stream block of ``Sources/Siliconed/Block.swift:5-12`` and
  ``:286-376``: modulation ``[scale_msa, gate_msa, scale_mlp, gate_mlp] = adaLN(adaln)`` (a Linear with
  bias, no SiLU, gates through tanh, scales as 1 + scale); ``x += gate_msa * norm2(attention(norm1(x) *
  scale_msa))``; ``x += gate_mlp * ffn_norm2(w2(silu(w1 a) * w3 a))`` with ``a = ffn_norm1(x) *
  scale_mlp``; QK-norm (RMSNorm over the head, eps 1e-5) and RoPE on adjacent pairs.  q / k / v are one
  fused product (N = 3d) and w1 / w3 another (N = 2 hidden): the columns are the same products.
* ``MMDiTBlock`` / ``MMDiT`` — config 5, a double-stream (MMDiT) block as BASELINE describes it: per
  stream a modulation Linear(256 -> 6d) (shift, scale, gate twice), LayerNorm without affine (eps
  1e-6, ``Ops.layerNorm``), q / k / v, QK-norm and RoPE, one joint attention over text then image
  tokens, the out projection and an MLP with GELU (tanh) (``QwenImage21.swift:953-963``), gated
  residuals.  The reference's QwenImage21 is single-stream, so this block follows the config, not a
  reference file.
"""
from __future__ import annotations

import math

import torch

from . import abi
from . import dit_abi as dk
from .products import Context, QuantizedWeight

# From FUSE_MIN_ROWS rows the blocks run QK-norm + RoPE in the q / k / v product's epilogue
# (sc_linear_qk_norm_rope), and the MMDiT block its GELU and gated residuals in the epilogues of the
# products before them (sc_linear_epilogue).
FUSED_EPILOGUES = True
FUSE_MIN_ROWS = 1536
# The Z-Image block's gate / up product is registered with its halves in blocks of 128 columns, so that
# each 256-column tile of the product holds a gate block and its up block (SC_EPI_SWIGLU).
SWIGLU_BLOCK = 128


def interleave_halves(w: torch.Tensor, block: int) -> torch.Tensor:
    """Rows [gate (h) ; up (h)] of a [2 h, k] weight -> gate block j, up block j, ... (blocks of `block`)."""
    h = w.shape[0] // 2
    return torch.stack([w[:h].reshape(h // block, block, -1), w[h:].reshape(h // block, block, -1)], 1).reshape(w.shape)


def deinterleave_halves(v: torch.Tensor, block: int) -> torch.Tensor:
    """Columns of a product of an interleaved weight -> [gate (h) | up (h)]."""
    rows, n = v.shape
    return v.reshape(rows, n // (2 * block), 2, block).transpose(1, 2).reshape(rows, n)


def quantize_per_channel(w: torch.Tensor):
    """int8 codes and fp32 scales of a [out, in] weight: s = max|w| / 127 per output, q = round(w / s)."""
    s = w.abs().amax(dim=1).clamp_min(1e-12) / 127.0
    q = torch.round(w / s[:, None]).clamp_(-127, 127).to(torch.int8)
    return q, s.float()


class Linear:
    """One int8 per-channel linear [out, in] in the library, from N(0, std) weights (random init)."""

    def __init__(self, ctx: Context, n_out: int, k_in: int, gen: torch.Generator, std: float = 0.02,
                 bias: bool = False, interleave: int = 0):
        """interleave: a gate / up product [2 h, k] whose halves are registered in blocks of `interleave`
        columns (gate block j, then up block j), the layout of the SwiGLU epilogue; outputs keep it."""
        dev = f"cuda:{ctx.device}"
        w = torch.randn(n_out, k_in, generator=gen, device=dev) * std
        if interleave:
            w = interleave_halves(w, interleave)
        q, s = quantize_per_channel(w)
        del w
        self.weight = QuantizedWeight(ctx, q, abi.WEIGHT_INT8, s, published_nk=True)
        del q
        self.n, self.k = n_out, k_in
        self.bias = (torch.randn(n_out, generator=gen, device=dev) * 0.01).to(torch.bfloat16) if bias else None

    def __call__(self, x: torch.Tensor, out: torch.Tensor, workspace=None) -> torch.Tensor:
        return self.weight.linear_ex(x, out, bias=self.bias, workspace=workspace)

    def _fuse(self, rows: int) -> bool:
        # The fused epilogues run on the widened route, which sc_linear takes from 1536 rows anyway.
        return FUSED_EPILOGUES and rows >= FUSE_MIN_ROWS

    def gelu(self, x: torch.Tensor, out: torch.Tensor, workspace=None) -> torch.Tensor:
        """out (bf16) = gelu_tanh(x W^T + b): fused into the product's epilogue from FUSE_MIN_ROWS rows,
        else the product and sd_gelu_tanh."""
        if self._fuse(x.shape[0]):
            return self.weight.linear_epilogue(x, out, abi.EPI_GELU_TANH, bias=self.bias, workspace=workspace)
        self(x, out, workspace)
        return dk.gelu_tanh(out)

    def qkv_heads(self, x: torch.Tensor, q, k, v, norm_q, norm_k, freqs, eps: float, batch: int, tokens: int,
                  offset: int, scratch: torch.Tensor, workspace=None) -> None:
        """q / k / v [batch, heads, joint, 128] of the q / k / v product, QK-norm and RoPE applied: in the
        product's epilogue from FUSE_MIN_ROWS rows (sc_linear_qk_norm_rope), else the product into `scratch`
        (bf16 [rows, 3 d]) and sd_qk_norm_rope."""
        if self._fuse(x.shape[0]):
            self.weight.linear_qk_norm_rope(x, q, k, v, norm_q, norm_k, freqs, eps, tokens, offset, bias=self.bias,
                                            workspace=workspace)
            return
        self(x, scratch, workspace)
        dk.qk_norm_rope(scratch, batch, tokens, q.shape[1], norm_q, norm_k, freqs, eps, q, k, v, q.shape[2], offset)

    def swiglu(self, x: torch.Tensor, out: torch.Tensor, scratch: torch.Tensor, workspace=None) -> torch.Tensor:
        """out (bf16 [rows, h]) = silu(gate) * up of this interleaved gate / up product: in the product's
        epilogue from FUSE_MIN_ROWS rows, else the product into `scratch` (bf16 [rows, 2 h]) and
        sd_swiglu_blocks."""
        if self._fuse(x.shape[0]):
            return self.weight.linear_epilogue(x, out, abi.EPI_SWIGLU, bias=self.bias, workspace=workspace)
        self(x, scratch, workspace)
        return dk.swiglu_blocks(scratch, out.shape[1], SWIGLU_BLOCK, out)

    def _reads_heads(self, o: torch.Tensor, n: int) -> bool:
        return self._fuse(o.shape[0] * n) and o.is_contiguous() and n % 128 == 0

    def from_heads(self, o: torch.Tensor, off: int, n: int, out: torch.Tensor, merged: torch.Tensor,
                   workspace=None) -> torch.Tensor:
        """out = (rows of the attention's output o [B, H, J, 128] at positions off .. off + n) W^T + b: the
        product reads o itself from FUSE_MIN_ROWS rows (sc_linear_heads), else the rows are merged into
        `merged` first."""
        if self._reads_heads(o, n):
            return self.weight.linear_heads(o, n, off, out, bias=self.bias, workspace=workspace)
        rows = merged_rows(o, o.shape[0], o.shape[1], o.shape[2], off, n, merged)
        return self(rows, out, workspace)

    def gated_residual_heads(self, o: torch.Tensor, off: int, n: int, resid: torch.Tensor, gate: torch.Tensor,
                             merged: torch.Tensor, scratch: torch.Tensor, workspace=None) -> torch.Tensor:
        """resid (fp32) += gate * (rows of o) W^T: the product reading o itself with the gated residual in its
        epilogue from FUSE_MIN_ROWS rows, else merge, product and sd_gated_residual."""
        if self._reads_heads(o, n):
            return self.weight.linear_heads(o, n, off, resid, bias=self.bias, op=abi.EPI_GATED_RESIDUAL, gate=gate,
                                            workspace=workspace)
        rows = merged_rows(o, o.shape[0], o.shape[1], o.shape[2], off, n, merged)
        return self.gated_residual(rows, resid, gate, scratch, workspace)

    def gated_residual(self, x: torch.Tensor, resid: torch.Tensor, gate: torch.Tensor, scratch: torch.Tensor,
                       workspace=None) -> torch.Tensor:
        """resid (fp32) += gate * (x W^T + b): fused into the product's epilogue from FUSE_MIN_ROWS rows,
        else the product into `scratch` (fp32) and sd_gated_residual."""
        if self._fuse(x.shape[0]):
            return self.weight.linear_epilogue(x, resid, abi.EPI_GATED_RESIDUAL, bias=self.bias, gate=gate,
                                               workspace=workspace)
        self(x, scratch, workspace)
        return dk.gated_residual(resid, scratch, gate, False, None, 0.0)

    def workspace_bytes(self, m: int) -> int:
        return self.weight.workspace_bytes(m)

    def close(self) -> None:
        self.weight.close()


def timestep_embedding(t: float, dim: int = 256, device="cuda") -> torch.Tensor:
    """[1, dim] bf16: [cos | sin] of 1000 t w_j, w_j = 10000^(-j / (dim / 2)) (the 256-d embedding)."""
    half = dim // 2
    w = torch.exp(-math.log(10000.0) * torch.arange(half, dtype=torch.float64) / half)
    a = 1000.0 * t * w
    return torch.cat([torch.cos(a), torch.sin(a)]).to(torch.bfloat16).reshape(1, dim).to(device)


def rope_table(positions: torch.Tensor, head_dim: int = 128, theta: float = 10000.0) -> torch.Tensor:
    """fp32 [S, head_dim / 2, 2] of (cos, sin) for adjacent-pair RoPE; positions [S, 2] (row, column):
    the first half of the pairs turns with the row, the second with the column."""
    pairs = head_dim // 2
    half = pairs // 2
    inv = theta ** (-torch.arange(half, dtype=torch.float64) / half)
    ang = torch.cat([positions[:, :1].double() * inv, positions[:, 1:2].double() * inv], dim=1)  # [S, pairs]
    return torch.stack([torch.cos(ang), torch.sin(ang)], dim=-1).float()


def image_text_positions(txt_tokens: int, grid: int) -> torch.Tensor:
    """Positions of the joint sequence, text first: text token i at (i, i); image patch (r, c) at
    (txt_tokens + r, txt_tokens + c)."""
    t = torch.arange(txt_tokens)
    txt = torch.stack([t, t], dim=1)
    r, c = torch.meshgrid(torch.arange(grid), torch.arange(grid), indexing="ij")
    img = torch.stack([r.reshape(-1), c.reshape(-1)], dim=1) + txt_tokens
    return torch.cat([txt, img], dim=0)


# "native": sd_attention, this project's tcgen05 kernel (parity-tested at configs 3 and 5); "library": torch's
# fused scaled-dot-product attention, the default while it is the faster of the two on B200 (config 3's
# attention: 228 us against 391 us for sd_attention).
ATTENTION = "library"


def attention(q, k, v, out=None):
    """Scaled dot-product attention over [B, H, S, 128] bf16, scale 1 / sqrt(128)."""
    if ATTENTION == "library":
        return torch.nn.functional.scaled_dot_product_attention(q, k, v)
    if out is None:
        out = torch.empty_like(q)
    return dk.attention(q.contiguous(), k.contiguous(), v.contiguous(), out, 1.0 / math.sqrt(q.shape[-1]))


def merged_rows(o, batch: int, heads: int, joint: int, off: int, n: int, out: torch.Tensor) -> torch.Tensor:
    """One stream's rows [batch * n, heads * 128] of the attention's output o [batch, heads, joint, 128].
    The fused attention may hand back o as a view of [batch, joint, heads, 128] memory: then the rows
    are already laid out (a view when the stream is the whole sequence of one image, else one copy);
    a [batch, heads, joint, 128] tensor goes through sd_attention_merge."""
    if o.is_contiguous():
        return dk.attention_merge(o, batch, heads, joint, off, n, out)
    t = o.transpose(1, 2)
    if not t.is_contiguous():
        return dk.attention_merge(o.contiguous(), batch, heads, joint, off, n, out)
    if batch == 1 and off == 0 and n == joint:
        return t.reshape(n, heads * 128)
    out.view(batch, n, heads * 128).copy_(t[:, off:off + n].reshape(batch, n, heads * 128))
    return out


class ZImageBlock:
    """Config 3: one single-stream block (hidden 3840, 30 x 128 heads, SwiGLU 10240, adaLN 256 -> 4 d)."""

    def __init__(self, ctx: Context, dim: int = 3840, heads: int = 30, hidden: int = 10240, adaln: int = 256,
                 seed: int = 0, eps: float = 1e-5):
        g = torch.Generator(device=f"cuda:{ctx.device}")
        g.manual_seed(seed)
        dev = f"cuda:{ctx.device}"
        self.ctx, self.d, self.heads, self.hidden, self.eps = ctx, dim, heads, hidden, eps
        self.modulation = Linear(ctx, 4 * dim, adaln, g, bias=True)
        self.qkv = Linear(ctx, 3 * dim, dim, g)
        self.out = Linear(ctx, dim, dim, g)
        self.w13 = Linear(ctx, 2 * hidden, dim, g, interleave=SWIGLU_BLOCK)
        self.w2 = Linear(ctx, dim, hidden, g)
        ones = lambda n: (1.0 + 0.1 * torch.randn(n, generator=g, device=dev)).float()
        self.norm1, self.norm2, self.ffn_norm1, self.ffn_norm2 = ones(dim), ones(dim), ones(dim), ones(dim)
        self.norm_q, self.norm_k = ones(128), ones(128)
        self._bufs = {}

    def linears(self):
        return [self.modulation, self.qkv, self.out, self.w13, self.w2]

    def flops(self, s: int) -> float:
        d, h = self.d, self.hidden
        return 2.0 * s * (4 * d * d + 3 * d * h) + 4.0 * s * s * d

    def _buffers(self, s: int):
        if s not in self._bufs:
            dev = f"cuda:{self.ctx.device}"
            d, h, H = self.d, self.hidden, self.heads
            ws = max(l.workspace_bytes(s) for l in self.linears())
            self._bufs = {s: dict(
                mod=torch.empty(1, 4 * d, dtype=torch.float32, device=dev),
                a=torch.empty(s, d, dtype=torch.bfloat16, device=dev),
                qkv=torch.empty(s, 3 * d, dtype=torch.bfloat16, device=dev),
                q=torch.empty(1, H, s, 128, dtype=torch.bfloat16, device=dev),
                k=torch.empty(1, H, s, 128, dtype=torch.bfloat16, device=dev),
                v=torch.empty(1, H, s, 128, dtype=torch.bfloat16, device=dev),
                merged=torch.empty(s, d, dtype=torch.bfloat16, device=dev),
                y=torch.empty(s, d, dtype=torch.float32, device=dev),
                h=torch.empty(s, 2 * h, dtype=torch.bfloat16, device=dev),
                g=torch.empty(s, h, dtype=torch.bfloat16, device=dev),
                ws=torch.empty(max(ws, 1), dtype=torch.uint8, device=dev))}
        return self._bufs[s]

    def forward(self, x: torch.Tensor, freqs: torch.Tensor, adaln: torch.Tensor) -> torch.Tensor:
        """x fp32 [S, d] (modified in place), freqs fp32 [S, 64, 2], adaln bf16 [1, 256]."""
        s, d = x.shape
        b = self._buffers(s)
        ws = b["ws"]
        self.modulation(adaln, b["mod"], ws)
        mod = b["mod"].reshape(4, d)
        scale_msa, gate_msa, scale_mlp, gate_mlp = mod[0], mod[1], mod[2], mod[3]
        # attention
        dk.rms_norm_modulate(x, self.norm1, scale_msa, self.eps, b["a"])
        self.qkv.qkv_heads(b["a"], b["q"], b["k"], b["v"], self.norm_q, self.norm_k, freqs, self.eps, 1, s, 0, b["qkv"],
                           ws)
        o = attention(b["q"], b["k"], b["v"])
        self.out.from_heads(o, 0, s, b["y"], b["merged"], ws)
        # the attention's residual and the feed-forward's input norm in one pass
        dk.gated_residual_rms_modulate(x, b["y"], gate_msa, True, self.norm2, self.eps, self.ffn_norm1, scale_mlp,
                                       self.eps, b["a"])
        self.w13.swiglu(b["a"], b["g"], b["h"], ws)
        self.w2(b["g"], b["y"], ws)
        dk.gated_residual(x, b["y"], gate_mlp, True, self.ffn_norm2, self.eps)
        return x

    def close(self) -> None:
        for l in self.linears():
            l.close()


class _Stream:
    """One stream's weights of a double-stream block."""

    def __init__(self, ctx, d, mlp, adaln, g, dev):
        self.modulation = Linear(ctx, 6 * d, adaln, g, bias=True)
        self.qkv = Linear(ctx, 3 * d, d, g)
        self.out = Linear(ctx, d, d, g)
        self.mlp1 = Linear(ctx, mlp, d, g)
        self.mlp2 = Linear(ctx, d, mlp, g)
        self.norm_q = (1.0 + 0.1 * torch.randn(128, generator=g, device=dev)).float()
        self.norm_k = (1.0 + 0.1 * torch.randn(128, generator=g, device=dev)).float()

    def linears(self):
        return [self.modulation, self.qkv, self.out, self.mlp1, self.mlp2]


class MMDiTBlock:
    """Config 5: one double-stream block (d 3072, 24 x 128 heads, MLP 12288 GELU tanh)."""

    def __init__(self, ctx: Context, g: torch.Generator, dim: int = 3072, heads: int = 24, mlp: int = 12288,
                 adaln: int = 256, eps: float = 1e-6):
        dev = f"cuda:{ctx.device}"
        self.d, self.heads, self.mlp, self.eps = dim, heads, mlp, eps
        self.txt = _Stream(ctx, dim, mlp, adaln, g, dev)
        self.img = _Stream(ctx, dim, mlp, adaln, g, dev)

    def linears(self):
        return self.txt.linears() + self.img.linears()

    def forward(self, x_txt, x_img, batch: int, temb, freqs, b) -> None:
        """x_txt fp32 [batch * St, d], x_img fp32 [batch * Si, d] (both modified in place); temb bf16 [1, 256];
        freqs fp32 [St + Si, 64, 2]; b: the model's buffers."""
        d, H, ws = self.d, self.heads, b["ws"]
        st, si = x_txt.shape[0] // batch, x_img.shape[0] // batch
        joint = st + si
        streams = ((self.txt, x_txt, st, 0), (self.img, x_img, si, st))
        mods = []
        for sw, x, n, off in streams:
            mod = b["mod_txt"] if sw is self.txt else b["mod_img"]
            sw.modulation(temb, mod, ws)
            mods.append(mod.reshape(6, d))
        for (sw, x, n, off), m in zip(streams, mods):
            rows = x.shape[0]
            a, qkv = b["a"][:rows], b["qkv"][:rows]
            dk.layer_norm_modulate(x, m[1], m[0], self.eps, a)
            sw.qkv.qkv_heads(a, b["q"], b["k"], b["v"], sw.norm_q, sw.norm_k, freqs, self.eps, batch, n, off, qkv, ws)
        o = attention(b["q"], b["k"], b["v"])
        for (sw, x, n, off), m in zip(streams, mods):
            rows = x.shape[0]
            y, a, h = b["y"][:rows], b["a"][:rows], b["h"][:rows]
            sw.out.gated_residual_heads(o, off, n, x, m[2], b["merged"][:rows], y, ws)
            dk.layer_norm_modulate(x, m[4], m[3], self.eps, a)
            sw.mlp1.gelu(a, h, ws)
            sw.mlp2.gated_residual(h, x, m[5], y, ws)

    def close(self) -> None:
        for l in self.linears():
            l.close()


class MMDiT:
    """Config 5's model: img_in Linear(64 -> d), txt_in Linear(d -> d), `blocks` double-stream blocks, the
    final modulated LayerNorm (Linear(256 -> 2 d): shift, scale) and proj_out Linear(d -> 64)."""

    def __init__(self, ctx: Context, blocks: int = 60, dim: int = 3072, heads: int = 24, mlp: int = 12288,
                 patch: int = 64, seed: int = 0):
        g = torch.Generator(device=f"cuda:{ctx.device}")
        g.manual_seed(seed)
        self.ctx, self.d, self.heads, self.mlp, self.patch = ctx, dim, heads, mlp, patch
        self.img_in = Linear(ctx, dim, patch, g)
        self.txt_in = Linear(ctx, dim, dim, g)
        self.blocks = [MMDiTBlock(ctx, g, dim, heads, mlp) for _ in range(blocks)]
        self.norm_out = Linear(ctx, 2 * dim, 256, g, bias=True)
        self.proj_out = Linear(ctx, patch, dim, g)
        self._bufs = None

    def linears(self):
        out = [self.img_in, self.txt_in, self.norm_out, self.proj_out]
        for blk in self.blocks:
            out += blk.linears()
        return out

    def weight_bytes(self) -> int:
        return sum(l.weight.device_bytes for l in self.linears())

    def flops_per_step(self, batch: int, st: int, si: int) -> float:
        d, m = self.d, self.mlp
        per_token = 2.0 * (4 * d * d + 2 * d * m)
        blocks = len(self.blocks) * (batch * (st + si) * per_token + 4.0 * batch * (st + si) ** 2 * d)
        return blocks + 2.0 * batch * si * (self.patch * d * 2) + 2.0 * batch * st * d * d

    def buffers(self, batch: int, st: int, si: int):
        key = (batch, st, si)
        if self._bufs is None or self._bufs[0] != key:
            dev = f"cuda:{self.ctx.device}"
            d, H, rows, joint = self.d, self.heads, batch * si, st + si
            ws = max(l.workspace_bytes(m) for l in self.linears() for m in (batch * si, batch * st, 1))
            bf = torch.bfloat16
            self._bufs = (key, dict(
                mod_txt=torch.empty(1, 6 * d, dtype=torch.float32, device=dev),
                mod_img=torch.empty(1, 6 * d, dtype=torch.float32, device=dev),
                mod_out=torch.empty(1, 2 * d, dtype=torch.float32, device=dev),
                a=torch.empty(rows, d, dtype=bf, device=dev),
                qkv=torch.empty(rows, 3 * d, dtype=bf, device=dev),
                q=torch.empty(batch, H, joint, 128, dtype=bf, device=dev),
                k=torch.empty(batch, H, joint, 128, dtype=bf, device=dev),
                v=torch.empty(batch, H, joint, 128, dtype=bf, device=dev),
                merged=torch.empty(rows, d, dtype=bf, device=dev),
                y=torch.empty(rows, d, dtype=torch.float32, device=dev),
                h=torch.empty(rows, self.mlp, dtype=bf, device=dev),
                x_img=torch.empty(rows, d, dtype=torch.float32, device=dev),
                x_txt=torch.empty(batch * st, d, dtype=torch.float32, device=dev),
                z_bf=torch.empty(rows, self.patch, dtype=bf, device=dev),
                v_out=torch.empty(rows, self.patch, dtype=torch.float32, device=dev),
                ws=torch.empty(max(ws, 1), dtype=torch.uint8, device=dev)))
        return self._bufs[1]

    def forward(self, z: torch.Tensor, txt: torch.Tensor, batch: int, t: float, freqs: torch.Tensor) -> torch.Tensor:
        """Velocity for latents z fp32 [batch * Si, 64] at time t, text bf16 [batch * St, d]: fp32 [batch * Si, 64]."""
        st, si = txt.shape[0] // batch, z.shape[0] // batch
        b = self.buffers(batch, st, si)
        ws = b["ws"]
        temb = timestep_embedding(t, device=z.device)
        b["z_bf"].copy_(z)
        self.img_in(b["z_bf"], b["x_img"], ws)
        self.txt_in(txt, b["x_txt"], ws)
        for blk in self.blocks:
            blk.forward(b["x_txt"], b["x_img"], batch, temb, freqs, b)
        self.norm_out(temb, b["mod_out"], ws)
        m = b["mod_out"].reshape(2, self.d)
        dk.layer_norm_modulate(b["x_img"], m[1], m[0], 1e-6, b["a"])
        self.proj_out(b["a"], b["v_out"], ws)
        return b["v_out"]

    def denoise(self, z: torch.Tensor, txt: torch.Tensor, batch: int, steps: int, freqs: torch.Tensor) -> torch.Tensor:
        """`steps` Euler steps of the flow from t = 1 to t = 0 on fp32 latents z (updated in place)."""
        sig = torch.linspace(1.0, 0.0, steps + 1).tolist()
        for i in range(steps):
            v = self.forward(z, txt, batch, sig[i], freqs)
            z.add_(v, alpha=sig[i + 1] - sig[i])
        return z

    def close(self) -> None:
        for l in self.linears():
            l.close()
