"""ctypes bindings of libsiliconed_dit.so (include/siliconed_dit.h), and thin tensor-level wrappers.

The library carries the elementwise stages of the DiT blocks; the linears are libsiliconed_cuda
(``abi.py``).  The wrappers take CUDA tensors (fp32 or bf16, contiguous) and the current stream.
"""
from __future__ import annotations

import ctypes
import os
import re

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libsiliconed_dit.so")
HEADER = os.path.join(os.path.dirname(HERE), "include", "siliconed_dit.h")

_P, _I, _I64, _F = ctypes.c_void_p, ctypes.c_int, ctypes.c_int64, ctypes.c_float

SIGNATURES = {
    "sd_rms_norm_modulate": (_I, [_P, _I64, _I, _P, _P, _F, _P, _P]),
    "sd_layer_norm_modulate": (_I, [_P, _I64, _I, _P, _P, _F, _P, _P]),
    "sd_gated_residual": (_I, [_P, _P, _I64, _I, _P, _I, _P, _F, _P]),
    "sd_gated_residual_rms_modulate": (_I, [_P, _P, _I64, _I, _P, _I, _P, _F, _P, _P, _F, _P, _P]),
    "sd_qk_norm_rope": (_I, [_P, _I, _I, _I, _I, _P, _P, _P, _F, _P, _P, _P, _I, _I, _P]),
    "sd_attention_merge": (_I, [_P, _I, _I, _I, _I, _I, _I, _P, _P]),
    "sd_swiglu": (_I, [_P, _I64, _I, _P, _P]),
    "sd_swiglu_blocks": (_I, [_P, _I64, _I, _I, _P, _P]),
    "sd_gelu_tanh": (_I, [_P, _I64, _P]),
    "sd_attention": (_I, [_P, _P, _P, _P, _I, _I, _I, _F, _P]),
    "sd_attention_errors": (_I, [ctypes.POINTER(ctypes.c_int)]),
}

_lib = None


def header_functions() -> set[str]:
    text = open(HEADER).read()
    return set(re.findall(r"^SD_API\s+\w+\s+(sd_\w+)\s*\(", text, flags=re.M))


def load(path: str = LIB_PATH) -> ctypes.CDLL:
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(path):
        from . import build as _build
        _build.build()
    lib = ctypes.CDLL(path)
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    _lib = lib
    return lib


class DiTKernelError(RuntimeError):
    pass


def _check(status: int, what: str) -> None:
    if status != 0:
        raise DiTKernelError(f"{what}: status {status}")


def _ptr(t):
    return ctypes.c_void_p(0 if t is None else t.data_ptr())


def _stream():
    import torch
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def rms_norm_modulate(x, weight, scale, eps, out):
    """out (bf16) = RMSNorm(x) * weight * (1 + scale), rows of x (fp32 [rows, d])."""
    rows, d = x.shape
    _check(load().sd_rms_norm_modulate(_ptr(x), rows, d, _ptr(weight), _ptr(scale), eps, _ptr(out), _stream()),
           "sd_rms_norm_modulate")
    return out


def layer_norm_modulate(x, scale, shift, eps, out):
    rows, d = x.shape
    _check(load().sd_layer_norm_modulate(_ptr(x), rows, d, _ptr(scale), _ptr(shift), eps, _ptr(out), _stream()),
           "sd_layer_norm_modulate")
    return out


def gated_residual(x, y, gate, gate_tanh: bool, norm_weight, eps):
    rows, d = x.shape
    _check(load().sd_gated_residual(_ptr(x), _ptr(y), rows, d, _ptr(gate), int(gate_tanh), _ptr(norm_weight), eps,
                                    _stream()), "sd_gated_residual")
    return x


def gated_residual_rms_modulate(x, y, gate, gate_tanh: bool, norm_weight, eps, weight, scale, eps2, out):
    rows, d = x.shape
    _check(load().sd_gated_residual_rms_modulate(_ptr(x), _ptr(y), rows, d, _ptr(gate), int(gate_tanh),
                                                 _ptr(norm_weight), eps, _ptr(weight), _ptr(scale), eps2, _ptr(out),
                                                 _stream()), "sd_gated_residual_rms_modulate")
    return out


def qk_norm_rope(qkv, batch, tokens, heads, norm_q, norm_k, freqs, eps, q, k, v, joint_len, token_offset):
    _check(load().sd_qk_norm_rope(_ptr(qkv), batch, tokens, heads, 128, _ptr(norm_q), _ptr(norm_k), _ptr(freqs), eps,
                                  _ptr(q), _ptr(k), _ptr(v), joint_len, token_offset, _stream()), "sd_qk_norm_rope")


def attention_merge(o, batch, heads, joint_len, token_offset, tokens, out):
    _check(load().sd_attention_merge(_ptr(o), batch, heads, 128, joint_len, token_offset, tokens, _ptr(out),
                                     _stream()), "sd_attention_merge")
    return out


def swiglu(h, hidden, out):
    _check(load().sd_swiglu(_ptr(h), h.shape[0], hidden, _ptr(out), _stream()), "sd_swiglu")
    return out


def swiglu_blocks(h, hidden, block, out):
    _check(load().sd_swiglu_blocks(_ptr(h), h.shape[0], hidden, block, _ptr(out), _stream()), "sd_swiglu_blocks")
    return out


def gelu_tanh(h):
    _check(load().sd_gelu_tanh(_ptr(h), h.numel(), _stream()), "sd_gelu_tanh")
    return h


def attention(q, k, v, out, scale: float):
    """out = softmax(q k^T * scale) v over [B, H, S, 128] bf16 (contiguous), on the tensor cores."""
    b, h, seq, d = q.shape
    _check(load().sd_attention(_ptr(q), _ptr(k), _ptr(v), _ptr(out), b * h, seq, d, scale, _stream()), "sd_attention")
    return out


def attention_errors() -> tuple[int, int]:
    """(status, site) of sd_attention's bounded waits since the last call: (0, 0), or SD_TIMEOUT and its site."""
    site = ctypes.c_int(0)
    return load().sd_attention_errors(ctypes.byref(site)), site.value
