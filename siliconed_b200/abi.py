"""ctypes binding of libsiliconed_cuda's C ABI (include/siliconed_cuda.h).

This is the same binding a non-C host would write (the Swift module map, a cgo or JNI stub):
plain pointers, sizes and integer status codes.  Loading never touches the GPU; every compute
entry point fails loudly (SC_NO_DEVICE) without an sm_100 device.  There is no CPU fallback.
"""
from __future__ import annotations

import ctypes
import os
import re

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libsiliconed_cuda.so")
HEADER = os.path.join(os.path.dirname(HERE), "include", "siliconed_cuda.h")

# sc_status
OK, INVALID_ARG, UNSUPPORTED_SHAPE, UNALIGNED, CUDA_ERROR, TIMEOUT, OUT_OF_MEMORY, REFUSED, \
    WORKSPACE_TOO_SMALL, NO_DEVICE = range(10)
STATUS_NAMES = {0: "SC_OK", 1: "SC_INVALID_ARG", 2: "SC_UNSUPPORTED_SHAPE", 3: "SC_UNALIGNED", 4: "SC_CUDA_ERROR",
                5: "SC_TIMEOUT", 6: "SC_OUT_OF_MEMORY", 7: "SC_REFUSED", 8: "SC_WORKSPACE_TOO_SMALL",
                9: "SC_NO_DEVICE"}
# sc_weight_kind / sc_scale_type / sc_scale_layout / flags
WEIGHT_INT8, WEIGHT_E4M3 = 1, 2
SCALE_F32, SCALE_BF16, SCALE_F16 = 1, 2, 3
SCALE_TENSOR, SCALE_COLUMNS = 0, 1
VALUES_ON_DEVICE, PUBLISHED_NK, ARENA_LAYOUT, NAN_CODES = 0x1, 0x2, 0x4, 0x8
OUT_BF16, OUT_F32 = 0, 1
EPI_GELU_TANH, EPI_GATED_RESIDUAL, EPI_SWIGLU = 1, 2, 3
IN_BF16, IN_F32 = 0, 1

_P, _I64, _I, _U32, _SZ = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int, ctypes.c_uint32, ctypes.c_size_t
_PP = ctypes.POINTER(ctypes.c_void_p)

SIGNATURES = {
    "sc_abi_version": (_I, []),
    "sc_status_string": (ctypes.c_char_p, [_I]),
    "sc_ctx_create": (_I, [_I, _PP]),
    "sc_ctx_destroy": (None, [_P]),
    "sc_last_error_string": (ctypes.c_char_p, [_P]),
    "sc_weight_create": (_I, [_P, _P, _I, _I64, _I64, _P, _I, _I, _U32, _P, _PP]),
    "sc_weight_create_shard": (_I, [_P, _P, _I, _I64, _I64, _P, _I, _I, _U32, _I64, _I64, _P, _PP]),
    "sc_weight_destroy": (_I, [_P, _P]),
    "sc_weight_info": (_I, [_P, ctypes.POINTER(_I64), ctypes.POINTER(_I64), ctypes.POINTER(_I),
                            ctypes.POINTER(_SZ)]),
    "sc_dequantize": (_I, [_P, _P, _P, _P]),
    "sc_workspace_size": (_I, [_P, _P, _I64, ctypes.POINTER(_SZ)]),
    "sc_linear": (_I, [_P, _P, _P, _I64, _P, _P, _P, _SZ, _P]),
    "sc_linear_ex": (_I, [_P, _P, _P, _I64, _P, _P, _I, _P, _SZ, _P]),
    "sc_linear_epilogue": (_I, [_P, _P, _P, _I64, _P, _P, _I, _P, _P, _SZ, _P]),
    "sc_weight_set_rotation": (_I, [_P, _P, _I]),
    "sc_linear_heads": (_I, [_P, _P, _P, _I64, _I, _I64, _I64, _I64, _P, _P, _I, _I, _P, _P, _SZ, _P]),
    "sc_linear_qk_norm_rope": (_I, [_P, _P, _P, _I64, _P, _P, _P, _P, _I, _I64, _I64, _I64, _P, _P, _P,
                                    ctypes.c_float, _P, _SZ, _P]),
    "sc_linear_host": (_I, [_P, _P, _P, _I64, _P, _P, _I, _P, _P, _P, _SZ, _I64, _P]),
    "sc_w8a8_workspace_size": (_I, [_P, _P, _I64, ctypes.POINTER(_SZ)]),
    "sc_linear_w8a8": (_I, [_P, _P, _P, _I, _I64, _P, _P, _I, _P, _SZ, _P]),
    "sc_quantize_rows": (_I, [_P, _P, _I, _I64, _I64, _I, _P, _I64, _P, _P]),
    "sc_rotate_activation": (_I, [_P, _P, _I64, _I64, _I, _P, _P]),
    "sc_linear_ex_noalloc": (_I, [_P, _P, _P, _I64, _P, _P, _I, _P]),
    "sc_linear_allgather": (_I, [_P, _P, _P, _I64, _P, _P, _P, _I, _I, _I64, _I64, ctypes.c_uint32, _P, _SZ, _P]),
    "sc_linear_allgather_mc": (_I, [_P, _P, _P, _I64, _P, _P, _P, _P, _I, _I, _I64, _I64, ctypes.c_uint32, _P, _SZ,
                                    _P]),
    "sc_allgather_wait": (_I, [_P, _P, _I, ctypes.c_uint32, _P]),
    "sc_ipc_handle": (_I, [_P, _P, _P, ctypes.POINTER(_SZ)]),
    "sc_ipc_open": (_I, [_P, _P, _SZ, ctypes.POINTER(ctypes.c_void_p)]),
    "sc_ipc_close": (_I, [_P, _P, _SZ]),
    "sc_linear_w8": (_I, [_P, _P, _P, _I64, _P, _P, _P, _SZ, _P]),
    "sc_linear_fp8": (_I, [_P, _P, _P, _I64, _P, _P, _P, _SZ, _P]),
    "sc_gemv_w8": (_I, [_P, _P, _P, _I64, _P, _P, _P, _SZ, _P]),
    "sc_sync": (_I, [_P, _P]),
    "sc_poll_errors": (_I, [_P, _P]),
}

_lib = None


class SiliconedError(RuntimeError):
    """A non-OK sc_status, with the context's message."""

    def __init__(self, status: int, message: str = ""):
        self.status = status
        super().__init__(f"{STATUS_NAMES.get(status, status)}: {message}")


def header_functions(path: str = HEADER) -> list[str]:
    """Names of every function the public header declares."""
    text = open(path).read()
    return sorted(set(re.findall(r"^SC_API\s+[\w\s\*]+?\b(sc_\w+)\s*\(", text, flags=re.M)))


def load(path: str = LIB_PATH) -> ctypes.CDLL:
    """Loads the library (building it first if the sources are newer), binding every signature."""
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


def check(status: int, ctx=None) -> None:
    if status != OK:
        msg = ""
        if ctx is not None:
            raw = load().sc_last_error_string(ctx)
            msg = raw.decode() if raw else ""
        raise SiliconedError(status, msg)
