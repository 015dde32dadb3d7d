"""Host-side mirror of Siliconed's quantized-linear interface, over the C ABI.

``WeightProducts.linear(name, a, c, m, k, n)`` keeps the reference's entry point
(Sources/Siliconed/WeightProducts.swift:278-279: the product ``C = A . W`` of the map's weight
``name``), and ``QuantizedWeight`` plays the map tensor + its ``Scale`` (Artifact.swift:15-57).
PyTorch is used here only to hold device buffers and to name the caller's CUDA stream; every
product runs in libsiliconed_cuda.  Errors raise ``SiliconedError`` (the reference throws).
"""
from __future__ import annotations

import ctypes

import numpy as np

from . import abi
from .abi import SiliconedError, check

try:  # torch is the device-memory plumbing of this host layer, not part of the library
    import torch
except ImportError:  # pragma: no cover
    torch = None


def _stream_ptr(stream) -> ctypes.c_void_p:
    if stream is None:
        stream = torch.cuda.current_stream()
    if hasattr(stream, "cuda_stream"):
        stream = stream.cuda_stream
    return ctypes.c_void_p(int(stream))


def _ptr(t) -> ctypes.c_void_p:
    if t is None:
        return ctypes.c_void_p(0)
    if torch is not None and isinstance(t, torch.Tensor):
        return ctypes.c_void_p(t.data_ptr())
    return t.ctypes.data_as(ctypes.c_void_p)


class Context:
    """An sc_ctx on one CUDA device."""

    def __init__(self, device: int = 0):
        self.lib = abi.load()
        self.device = int(device)
        p = ctypes.c_void_p()
        status = self.lib.sc_ctx_create(self.device, ctypes.byref(p))
        if status != abi.OK:
            raise SiliconedError(status, f"sc_ctx_create({device})")
        self.ptr = p
        self._workspace = None

    def workspace(self, nbytes: int, device) -> "torch.Tensor":
        """The context's shared product workspace, at least ``nbytes`` long (grown on demand).  Products
        that run concurrently on different streams need workspaces of their own (pass ``workspace=``);
        calls on one stream may share this one."""
        if self._workspace is None or self._workspace.numel() < nbytes:
            self._workspace = torch.empty(int(nbytes), dtype=torch.uint8, device=device)
        return self._workspace

    def close(self) -> None:
        if getattr(self, "ptr", None):
            self.lib.sc_ctx_destroy(self.ptr)
            self.ptr = None

    def __del__(self):  # pragma: no cover - best effort
        try:
            self.close()
        except Exception:
            pass

    def check(self, status: int) -> None:
        check(status, self.ptr)

    def sync(self, stream=None) -> None:
        self.check(self.lib.sc_sync(self.ptr, _stream_ptr(stream)))

    def poll_errors(self, stream=None) -> None:
        """Raises SiliconedError(SC_TIMEOUT) if a bounded device-side wait gave up since the last poll."""
        self.check(self.lib.sc_poll_errors(self.ptr, _stream_ptr(stream)))


def _scale_type_of(scales, declared: int | None = None) -> tuple[int, object]:
    """(sc_scale_type, contiguous host-or-device buffer) of a scale array as published; bf16 scales come
    as a torch bfloat16 tensor, or as 16-bit integer bits with ``declared`` = SCALE_BF16."""
    if torch is not None and isinstance(scales, torch.Tensor):
        t = scales.contiguous()
        kinds = {torch.float32: abi.SCALE_F32, torch.bfloat16: abi.SCALE_BF16, torch.float16: abi.SCALE_F16}
        if t.dtype not in kinds:
            raise SiliconedError(abi.INVALID_ARG, f"scale dtype {t.dtype}")
        return kinds[t.dtype], t
    a = np.ascontiguousarray(scales)
    if declared == abi.SCALE_BF16 and a.dtype in (np.dtype(np.uint16), np.dtype(np.int16)):
        return abi.SCALE_BF16, a
    kinds = {np.dtype(np.float32): abi.SCALE_F32, np.dtype(np.float16): abi.SCALE_F16}
    if a.dtype not in kinds:
        raise SiliconedError(abi.INVALID_ARG, f"scale dtype {a.dtype} (pass bf16 bits with scale_type=SCALE_BF16)")
    return kinds[a.dtype], a


class QuantizedWeight:
    """One 8-bit linear weight registered in the library's device arena.

    values: [K, N] codes in the map's layout (or [N, K] with ``published_nk``), int8 / uint8 bytes, as a
    numpy array or a torch tensor (CPU or CUDA).  scales: one per output (shape [N]) or one for the
    tensor (shape [] / [1]), fp32 / bf16 / fp16.  ``columns=(n0, n1)`` keeps only that column shard.
    ``arena=(k, n)``: values are the arena's own [n_pad][k_pad] bytes of a [K, N] weight (a map stored
    re-tiled), registered with one copy (SC_WEIGHT_ARENA_LAYOUT); ``nan_codes`` states that device-resident
    e4m3 codes hold NaN codes (host codes are scanned by the library).
    """

    def __init__(self, ctx: Context, values, kind: int, scales, *, scale_type: int | None = None,
                 published_nk: bool = False, columns: tuple[int, int] | None = None, rotation: int = 0, stream=None,
                 arena: tuple[int, int] | None = None, nan_codes: bool = False):
        self.ctx = ctx
        lib = ctx.lib
        on_device = torch is not None and isinstance(values, torch.Tensor) and values.is_cuda
        if torch is not None and isinstance(values, torch.Tensor):
            v = values.contiguous()
            if v.dtype not in (torch.int8, torch.uint8):
                v = v.view(torch.uint8) if v.element_size() == 1 else None
            if v is None:
                raise SiliconedError(abi.INVALID_ARG, "values must be 1-byte codes")
            shape = tuple(v.shape)
        else:
            v = np.ascontiguousarray(values)
            if v.dtype.itemsize != 1:
                raise SiliconedError(abi.INVALID_ARG, "values must be 1-byte codes")
            shape = v.shape
        if len(shape) != 2:
            raise SiliconedError(abi.INVALID_ARG, "values must be 2-D")
        if arena is not None:
            k, n = (int(arena[0]), int(arena[1]))
            if tuple(shape) != (-(-n // 256) * 256, -(-k // 64) * 64) or published_nk or columns is not None:
                raise SiliconedError(abi.INVALID_ARG, f"arena values of [{k}, {n}] are [n_pad, k_pad] bytes, whole")
        else:
            k, n = (shape[1], shape[0]) if published_nk else shape
        st, s = _scale_type_of(scales, scale_type)
        if scale_type is not None:
            st = scale_type
        s_count = int(np.prod(s.shape)) if len(s.shape) else 1
        layout = abi.SCALE_TENSOR if s_count == 1 else abi.SCALE_COLUMNS
        if layout == abi.SCALE_COLUMNS and s_count != n:
            raise SiliconedError(abi.INVALID_ARG, f"{s_count} scales for {n} outputs")
        s_on_device = torch is not None and isinstance(s, torch.Tensor) and s.is_cuda
        if on_device != s_on_device:
            s = s.to(values.device) if on_device else (s.cpu() if isinstance(s, torch.Tensor) else s)
        flags = (abi.VALUES_ON_DEVICE if on_device else 0) | (abi.PUBLISHED_NK if published_nk else 0)
        if arena is not None:
            flags |= abi.ARENA_LAYOUT | (abi.NAN_CODES if nan_codes else 0)
        n0, n1 = columns if columns is not None else (0, n)
        p = ctypes.c_void_p()
        self._keep = (v, s)
        ctx.check(lib.sc_weight_create_shard(ctx.ptr, _ptr(v), kind, k, n, _ptr(s), st, layout, flags, n0, n1,
                                             _stream_ptr(stream) if torch is not None else None, ctypes.byref(p)))
        self._keep = None
        self.ptr = p
        self.kind = kind
        self.k, self.n = int(k), int(n1 - n0)
        bk, bn, kd, by = ctypes.c_int64(), ctypes.c_int64(), ctypes.c_int(), ctypes.c_size_t()
        ctx.check(lib.sc_weight_info(self.ptr, ctypes.byref(bk), ctypes.byref(bn), ctypes.byref(kd),
                                     ctypes.byref(by)))
        self.device_bytes = int(by.value)
        self.rotation = 0
        if rotation:
            self.set_rotation(rotation)

    def set_rotation(self, group: int) -> None:
        """ComfyUI's convrot of group G on this int8 weight (sc_weight_set_rotation; 0 clears it): the
        products rotate x first, the export is float(H q) * s / sqrt(G)."""
        self.ctx.check(self.ctx.lib.sc_weight_set_rotation(self.ctx.ptr, self.ptr, int(group)))
        self.rotation = int(group)

    def close(self) -> None:
        if getattr(self, "ptr", None):
            self.ctx.lib.sc_weight_destroy(self.ctx.ptr, self.ptr)
            self.ptr = None

    def __del__(self):  # pragma: no cover
        try:
            self.close()
        except Exception:
            pass

    def workspace_bytes(self, m: int) -> int:
        b = ctypes.c_size_t()
        self.ctx.check(self.ctx.lib.sc_workspace_size(self.ctx.ptr, self.ptr, int(m), ctypes.byref(b)))
        return int(b.value)

    def dequantize(self, out=None, stream=None):
        """fp32 [K, N] on the device: float(q) * s, bit for bit (Widen.dequantize)."""
        if out is None:
            out = torch.empty((self.k, self.n), dtype=torch.float32, device=f"cuda:{self.ctx.device}")
        self.ctx.check(self.ctx.lib.sc_dequantize(self.ctx.ptr, self.ptr, _ptr(out), _stream_ptr(stream)))
        return out

    def _product(self, fn_name: str, x, bias, out, workspace, stream):
        if x.dtype != torch.bfloat16 or not x.is_cuda or x.dim() != 2 or x.shape[1] != self.k:
            raise SiliconedError(abi.INVALID_ARG, f"x must be a CUDA bf16 [M, {self.k}] tensor")
        x = x.contiguous()
        m = x.shape[0]
        if out is None:
            out = torch.empty((m, self.n), dtype=torch.bfloat16, device=x.device)
        need = self.workspace_bytes(m)
        if need and workspace is None:
            workspace = self.ctx.workspace(need, x.device)
        ws_bytes = 0 if workspace is None else workspace.numel() * workspace.element_size()
        fn = getattr(self.ctx.lib, fn_name)
        self.ctx.check(fn(self.ctx.ptr, self.ptr, _ptr(x), m, _ptr(bias), _ptr(out), _ptr(workspace), ws_bytes,
                          _stream_ptr(stream)))
        return out

    def linear_ex(self, x, out, bias=None, workspace=None, stream=None):
        """sc_linear_ex: y = (x . q) * s + bias into `out`, bf16 or fp32 [M, N] (the output's dtype chooses)."""
        if x.dtype != torch.bfloat16 or not x.is_cuda or x.dim() != 2 or x.shape[1] != self.k:
            raise SiliconedError(abi.INVALID_ARG, f"x must be a CUDA bf16 [M, {self.k}] tensor")
        m = x.shape[0]
        if out.dtype not in (torch.bfloat16, torch.float32) or tuple(out.shape) != (m, self.n) or not out.is_contiguous():
            raise SiliconedError(abi.INVALID_ARG, f"out must be a contiguous bf16 or fp32 [{m}, {self.n}] tensor")
        need = self.workspace_bytes(m)
        if need and workspace is None:
            workspace = self.ctx.workspace(need, x.device)
        ws_bytes = 0 if workspace is None else workspace.numel() * workspace.element_size()
        y_type = abi.OUT_F32 if out.dtype == torch.float32 else abi.OUT_BF16
        self.ctx.check(self.ctx.lib.sc_linear_ex(self.ctx.ptr, self.ptr, _ptr(x), m, _ptr(bias), _ptr(out), y_type,
                                                 _ptr(workspace), ws_bytes, _stream_ptr(stream)))
        return out

    def epilogue_workspace_bytes(self, m: int) -> int:
        """Workspace of sc_linear_epilogue for M rows: the widened weight (sc_workspace_size from 1536 rows),
        after the rotated x of a convrot weight."""
        return self.workspace_bytes(max(int(m), 1536))

    def linear_qk_norm_rope(self, x, q, k, v, norm_q, norm_k, freqs, eps: float, tokens: int, offset: int = 0,
                            bias=None, workspace=None, stream=None):
        """sc_linear_qk_norm_rope: the q / k / v product with QK-norm and RoPE in its epilogue, written to
        q, k, v (bf16 [images, heads, joint, 128]); x's rows are images x tokens, at joint positions
        offset + token."""
        if x.dtype != torch.bfloat16 or not x.is_cuda or x.dim() != 2 or x.shape[1] != self.k:
            raise SiliconedError(abi.INVALID_ARG, f"x must be a CUDA bf16 [M, {self.k}] tensor")
        m = x.shape[0]
        heads, joint = q.shape[1], q.shape[2]
        if workspace is None:
            workspace = self.ctx.workspace(self.epilogue_workspace_bytes(m), x.device)
        ws_bytes = workspace.numel() * workspace.element_size()
        self.ctx.check(self.ctx.lib.sc_linear_qk_norm_rope(
            self.ctx.ptr, self.ptr, _ptr(x), m, _ptr(bias), _ptr(q), _ptr(k), _ptr(v), heads, int(tokens), joint,
            int(offset), _ptr(norm_q), _ptr(norm_k), _ptr(freqs), float(eps), _ptr(workspace), ws_bytes,
            _stream_ptr(stream)))
        return q, k, v

    def linear_heads(self, o, tokens: int, offset: int, out, bias=None, op: int = 0, gate=None, workspace=None,
                     stream=None):
        """sc_linear_heads: the product of the attention's output o (bf16 [B, H, J, 128], contiguous) read as
        the rows of [B * tokens, H * 128] (positions offset ...), into out (bf16 or fp32 [B * tokens, N]; with
        op EPI_GATED_RESIDUAL the fp32 residual += gate * v)."""
        if o.dtype != torch.bfloat16 or not o.is_cuda or o.dim() != 4 or o.shape[3] != 128 or not o.is_contiguous():
            raise SiliconedError(abi.INVALID_ARG, "o must be a contiguous CUDA bf16 [B, H, J, 128] tensor")
        batch, heads, joint = o.shape[0], o.shape[1], o.shape[2]
        m = batch * tokens
        if out.dtype not in (torch.bfloat16, torch.float32) or tuple(out.shape) != (m, self.n) or not out.is_contiguous():
            raise SiliconedError(abi.INVALID_ARG, f"out must be a contiguous bf16 or fp32 [{m}, {self.n}] tensor")
        if workspace is None:
            workspace = self.ctx.workspace(self.epilogue_workspace_bytes(m), o.device)
        ws_bytes = workspace.numel() * workspace.element_size()
        y_type = abi.OUT_F32 if out.dtype == torch.float32 else abi.OUT_BF16
        self.ctx.check(self.ctx.lib.sc_linear_heads(self.ctx.ptr, self.ptr, _ptr(o), batch, heads, joint, int(offset),
                                                    int(tokens), _ptr(bias), _ptr(out), y_type, int(op), _ptr(gate),
                                                    _ptr(workspace), ws_bytes, _stream_ptr(stream)))
        return out

    def linear_epilogue(self, x, out, op: int, bias=None, gate=None, workspace=None, stream=None):
        """sc_linear_epilogue: v = (x . q) * s + bias with the DiT stage `op` fused into the product's
        epilogue.  EPI_GELU_TANH: out bf16 [M, N] = gelu_tanh(v); EPI_GATED_RESIDUAL: out fp32 [M, N]
        += gate * v in place (gate fp32 [N]); EPI_SWIGLU: out bf16 [M, N / 2] = silu(gate) * up with the
        weight's columns in blocks of 128 (gate, up).  M must exceed 128."""
        if x.dtype != torch.bfloat16 or not x.is_cuda or x.dim() != 2 or x.shape[1] != self.k:
            raise SiliconedError(abi.INVALID_ARG, f"x must be a CUDA bf16 [M, {self.k}] tensor")
        m = x.shape[0]
        want = torch.float32 if op == abi.EPI_GATED_RESIDUAL else torch.bfloat16
        n_out = self.n // 2 if op == abi.EPI_SWIGLU else self.n
        if out.dtype != want or tuple(out.shape) != (m, n_out) or not out.is_contiguous():
            raise SiliconedError(abi.INVALID_ARG, f"out must be a contiguous {want} [{m}, {n_out}] tensor")
        if gate is not None and (gate.dtype != torch.float32 or gate.numel() != self.n or not gate.is_contiguous()):
            raise SiliconedError(abi.INVALID_ARG, f"gate must be a contiguous fp32 [{self.n}] tensor")
        if workspace is None:
            workspace = self.ctx.workspace(self.epilogue_workspace_bytes(m), x.device)
        ws_bytes = workspace.numel() * workspace.element_size()
        self.ctx.check(self.ctx.lib.sc_linear_epilogue(self.ctx.ptr, self.ptr, _ptr(x), m, _ptr(bias), _ptr(out), op,
                                                       _ptr(gate), _ptr(workspace), ws_bytes, _stream_ptr(stream)))
        return out

    def linear_host(self, x_host, out_host, bias=None, x_dev=None, y_dev=None, workspace=None, chunk_rows: int = 0,
                    stream=None, direct: bool = False):
        """sc_linear_host: out_host (CPU, bf16 or fp32 [M, N]) = x_host (CPU bf16 [M, K]) . W + bias, the copies
        overlapped with the products in chunks of rows.  Pinned host tensors let the copies overlap; x_dev /
        y_dev are device staging buffers (allocated here when not given).  direct: the products write the
        pinned out_host themselves (no y_dev, no copy back)."""
        if x_host.dtype != torch.bfloat16 or x_host.is_cuda or x_host.dim() != 2 or x_host.shape[1] != self.k:
            raise SiliconedError(abi.INVALID_ARG, f"x_host must be a CPU bf16 [M, {self.k}] tensor")
        m = x_host.shape[0]
        if out_host.dtype not in (torch.bfloat16, torch.float32) or out_host.is_cuda or \
                tuple(out_host.shape) != (m, self.n) or not out_host.is_contiguous() or not x_host.is_contiguous():
            raise SiliconedError(abi.INVALID_ARG, f"out_host must be a contiguous CPU bf16 or fp32 [{m}, {self.n}] tensor")
        dev = f"cuda:{self.ctx.device}"
        if x_dev is None:
            x_dev = torch.empty((m, self.k), dtype=torch.bfloat16, device=dev)
        if direct:
            y_dev = None
        elif y_dev is None:
            y_dev = torch.empty((m, self.n), dtype=out_host.dtype, device=dev)
        need = self.epilogue_workspace_bytes(m) if direct else self.workspace_bytes(m)
        if need and workspace is None:
            workspace = self.ctx.workspace(need, dev)
        ws_bytes = 0 if workspace is None else workspace.numel() * workspace.element_size()
        y_type = abi.OUT_F32 if out_host.dtype == torch.float32 else abi.OUT_BF16
        self.ctx.check(self.ctx.lib.sc_linear_host(self.ctx.ptr, self.ptr, _ptr(x_host), m, _ptr(bias), _ptr(out_host),
                                                   y_type, _ptr(x_dev), _ptr(y_dev), _ptr(workspace), ws_bytes,
                                                   int(chunk_rows), _stream_ptr(stream)))
        return out_host

    def w8a8_workspace_bytes(self, m: int) -> int:
        b = ctypes.c_size_t()
        self.ctx.check(self.ctx.lib.sc_w8a8_workspace_size(self.ctx.ptr, self.ptr, int(m), ctypes.byref(b)))
        return int(b.value)

    def linear_w8a8(self, x, out, bias=None, workspace=None, stream=None):
        """sc_linear_w8a8: x (bf16 or fp32 [M, K]) rotated if the weight is convrot, quantized to int8 per
        row, times the int8 codes exactly, then float(acc) * (s_x * s_w) (+ bias) into `out` (bf16 or fp32)."""
        if x.dtype not in (torch.bfloat16, torch.float32) or not x.is_cuda or x.dim() != 2 or x.shape[1] != self.k:
            raise SiliconedError(abi.INVALID_ARG, f"x must be a CUDA bf16 or fp32 [M, {self.k}] tensor")
        x = x.contiguous()
        m = x.shape[0]
        if out.dtype not in (torch.bfloat16, torch.float32) or tuple(out.shape) != (m, self.n) or not out.is_contiguous():
            raise SiliconedError(abi.INVALID_ARG, f"out must be a contiguous bf16 or fp32 [{m}, {self.n}] tensor")
        if workspace is None:
            workspace = self.ctx.workspace(self.w8a8_workspace_bytes(m), x.device)
        ws_bytes = workspace.numel() * workspace.element_size()
        self.ctx.check(self.ctx.lib.sc_linear_w8a8(
            self.ctx.ptr, self.ptr, _ptr(x), abi.IN_F32 if x.dtype == torch.float32 else abi.IN_BF16, m, _ptr(bias),
            _ptr(out), abi.OUT_F32 if out.dtype == torch.float32 else abi.OUT_BF16, _ptr(workspace), ws_bytes,
            _stream_ptr(stream)))
        return out

    def linear(self, x, bias=None, out=None, workspace=None, stream=None):
        """y = bf16((x . q) * s + bias), dispatching on M (GEMV for M <= 32, tensor-core GEMM above)."""
        return self._product("sc_linear", x, bias, out, workspace, stream)

    def gemv(self, x, bias=None, out=None, workspace=None, stream=None):
        return self._product("sc_gemv_w8", x, bias, out, workspace, stream)


def rotate_activation(ctx: Context, x, group: int, out=None, stream=None):
    """sc_rotate_activation: bf16 [M, K] -> bf16(x . H / sqrt(G)) per group of G along K (rotate_groups)."""
    if x.dtype != torch.bfloat16 or not x.is_cuda or x.dim() != 2 or not x.is_contiguous():
        raise SiliconedError(abi.INVALID_ARG, "x must be a contiguous CUDA bf16 [M, K] tensor")
    if out is None:
        out = torch.empty_like(x)
    ctx.check(ctx.lib.sc_rotate_activation(ctx.ptr, _ptr(x), x.shape[0], x.shape[1], int(group), _ptr(out),
                                           _stream_ptr(stream)))
    return out


def quantize_rows(ctx: Context, x, group: int = 0, stream=None):
    """sc_quantize_rows: (codes int8 [M, K], s_x fp32 [M]) of x (bf16 or fp32 [M, K]), rotated by `group` first."""
    if x.dtype not in (torch.bfloat16, torch.float32) or not x.is_cuda or x.dim() != 2 or not x.is_contiguous():
        raise SiliconedError(abi.INVALID_ARG, "x must be a contiguous CUDA bf16 or fp32 [M, K] tensor")
    m, k = x.shape
    ld = (k + 15) // 16 * 16
    codes = torch.empty((m, ld), dtype=torch.int8, device=x.device)
    scales = torch.empty(m, dtype=torch.float32, device=x.device)
    ctx.check(ctx.lib.sc_quantize_rows(ctx.ptr, _ptr(x), abi.IN_F32 if x.dtype == torch.float32 else abi.IN_BF16, m, k,
                                       int(group), _ptr(codes), ld, _ptr(scales), _stream_ptr(stream)))
    return codes[:, :k], scales


class WeightProducts:
    """Products by weight name: the reference's ``WeightProducts.linear(_:a:c:m:k:n:)``.

    ``register`` stands for the map's tensor + scale (the reference reads them from the mmap'd
    map); ``linear`` computes ``c[m, n] = a[m, k] . W(name)`` into the caller's buffer ``c``.
    """

    def __init__(self, ctx: Context):
        self.ctx = ctx
        self.weights: dict[str, QuantizedWeight] = {}
        self.biases: dict[str, object] = {}
        self._workspace = None

    def register(self, name: str, values, kind: int, scales, bias=None, **kw) -> QuantizedWeight:
        w = QuantizedWeight(self.ctx, values, kind, scales, **kw)
        self.weights[name] = w
        if bias is not None:
            self.biases[name] = bias
        return w

    def register_map(self, artifact, names=None, device=None) -> list[str]:
        """Registers the 8-bit linears of an opened map (``artifact.Artifact``), all of them or ``names``,
        each read in place from the mapped file (WeightProducts.inPlaceInt8, WeightProducts.swift:801-862).
        A weight ``<base>.weight`` takes the map's ``<base>.bias`` when it is a bf16 vector of N values,
        as a device tensor; any other bias stays the caller's to give.  Returns the names registered."""
        names = artifact.quantized_names() if names is None else list(names)
        device = torch.device("cuda", self.ctx.device) if device is None else device
        for name in names:
            w = artifact.register(self.ctx, name)
            self.weights[name] = w
            if name.endswith(".weight"):
                b = artifact.tensors.get(name[: -len(".weight")] + ".bias")
                if b is not None and b.dtype == "bfloat16" and b.shape == (w.n,):
                    bits = np.array(artifact.array(b.name))  # a copy: the map stays read-only
                    self.biases[name] = torch.from_numpy(bits.view(np.int16)).to(device).view(torch.bfloat16)
        return names

    def linear(self, name: str, a, c, m: int, k: int, n: int, stream=None) -> None:
        w = self.weights.get(name)
        if w is None:
            raise SiliconedError(abi.INVALID_ARG, f"{name}: no such weight")
        if (w.k, w.n) != (k, n) or tuple(a.shape) != (m, k) or tuple(c.shape) != (m, n):
            raise SiliconedError(abi.UNSUPPORTED_SHAPE, f"{name}: [{m}, {k}] . [{w.k}, {w.n}] -> {tuple(c.shape)}")
        need = w.workspace_bytes(m)
        ws = None
        if need:
            if self._workspace is None or self._workspace.numel() < need:
                self._workspace = torch.empty(need, dtype=torch.uint8, device=a.device)
            ws = self._workspace
        w.linear(a, bias=self.biases.get(name), out=c, workspace=ws, stream=stream)

    def close(self) -> None:
        for w in self.weights.values():
            w.close()
        self.weights.clear()
