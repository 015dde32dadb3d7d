"""The C-ABI library without a GPU: it loads, exports exactly what the header declares, and fails
loudly (never a CPU fallback) when no sm_100 device is present."""
import ctypes
import subprocess

import pytest

from siliconed_b200 import abi


def exported_symbols(path):
    out = subprocess.run(["nm", "-D", "--defined-only", path], capture_output=True, text=True, check=True).stdout
    return sorted({line.split()[-1] for line in out.splitlines() if " T " in line})


def test_library_exports_every_declared_function():
    lib = abi.load()
    declared = abi.header_functions()
    assert len(declared) >= 18
    for name in declared:
        assert hasattr(lib, name), name
    assert exported_symbols(abi.LIB_PATH) == declared, "the library exports exactly the header's functions"
    assert sorted(abi.SIGNATURES) == declared, "the ctypes binding covers every declared function"


def test_version_and_status_strings():
    lib = abi.load()
    assert lib.sc_abi_version() == 1
    for code, name in abi.STATUS_NAMES.items():
        s = lib.sc_status_string(code).decode()
        assert s and s != "unknown status", name
    assert lib.sc_status_string(99).decode() == "unknown status"


def test_null_arguments_are_refused_not_crashed():
    lib = abi.load()
    assert lib.sc_ctx_create(0, None) == abi.INVALID_ARG
    assert lib.sc_last_error_string(None).decode() == "null context"
    null = ctypes.c_void_p(0)
    for name in ("sc_linear", "sc_linear_w8", "sc_linear_fp8", "sc_gemv_w8"):
        assert getattr(lib, name)(null, null, null, 1, null, null, null, 0, null) == abi.INVALID_ARG, name
    assert lib.sc_linear_ex(null, null, null, 1, null, null, 0, null, 0, null) == abi.INVALID_ARG
    assert lib.sc_sync(null, null) == abi.INVALID_ARG
    assert lib.sc_poll_errors(null, null) == abi.INVALID_ARG
    assert lib.sc_weight_destroy(null, null) == abi.INVALID_ARG
    assert lib.sc_weight_info(null, None, None, None, None) == abi.INVALID_ARG
    b = ctypes.c_size_t()
    assert lib.sc_workspace_size(null, null, 1, ctypes.byref(b)) == abi.INVALID_ARG
    lib.sc_ctx_destroy(null)  # a no-op


def test_no_device_means_an_error_not_a_fallback():
    torch = pytest.importorskip("torch")
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    p = ctypes.c_void_p()
    assert abi.load().sc_ctx_create(0, ctypes.byref(p)) == abi.NO_DEVICE
    from siliconed_b200.products import Context
    with pytest.raises(abi.SiliconedError) as e:
        Context(0)
    assert e.value.status == abi.NO_DEVICE
