"""Failure detection on a B200 without a GPU fault: a bounded device-side wait that runs out.

The fused gather's wait (sc_allgather_wait, the kernel every rank runs before it reads the gathered y)
is given a flag array in which one rank's flag is never raised: nothing sets it, so the wait gives up
after its limit (2 s of the global timer), records the timeout and its site in the context's error word
and returns.  Bars: the launch itself succeeds; sc_poll_errors reports SC_TIMEOUT naming the gather's
site; the error word is cleared by that poll; the context stays usable (a product right after gives the
oracle's bits, and a wait whose flags are all raised returns at once).  No kernel traps, faults or spins
without a bound.
"""
import ctypes
import time

import numpy as np
import pytest

import oracle
from siliconed_b200 import abi, configs
from siliconed_b200.abi import SiliconedError

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

if not torch.cuda.is_available():  # collected on CPU boxes, skipped there
    pytest.skip("needs a CUDA device", allow_module_level=True)

from siliconed_b200.products import Context, QuantizedWeight  # noqa: E402

SITE_GATHER = 9  # kSiteGather of the library's wait sites


@pytest.fixture(scope="module")
def ctx():
    c = Context(0)
    yield c
    c.close()


def test_a_wait_that_runs_out_is_a_status_and_the_context_survives(ctx):
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    flags = torch.zeros(2, dtype=torch.int32, device="cuda")
    flags[0] = 1                                     # this rank's columns landed; rank 1's never will
    ctx.poll_errors()                                # nothing pending before
    t0 = time.monotonic()
    assert ctx.lib.sc_allgather_wait(ctx.ptr, ctypes.c_void_p(flags.data_ptr()), 2, 1, stream) == abi.OK
    with pytest.raises(SiliconedError) as e:
        ctx.poll_errors()
    waited = time.monotonic() - t0
    assert e.value.status == abi.TIMEOUT
    assert f"site {SITE_GATHER}" in str(e.value)
    assert 1.5 <= waited <= 60.0, f"the wait gave up after {waited:.2f} s"
    ctx.poll_errors()                                # the poll cleared the error word

    # the context is still usable: a product right after gives the oracle's bits
    g = np.random.default_rng(5)
    m, k, n = 200, 256, 512
    x = configs.to_bf16_bits(g.standard_normal((m, k), dtype=np.float32))
    q = g.integers(-128, 128, (k, n), dtype=np.int16).astype(np.int8)
    s = (np.abs(g.standard_normal(n)) * 0.02 / 127 + 1e-6).astype(np.float32)
    w = QuantizedWeight(ctx, q.view(np.uint8), abi.WEIGHT_INT8, s)
    xd = torch.from_numpy(x.view(np.int16)).cuda().view(torch.bfloat16)
    y = torch.empty((m, n), dtype=torch.float32, device="cuda")
    w.linear_ex(xd, y)
    ctx.poll_errors()
    c_ref, _ = oracle.linear_int8(x, q, s, None)
    got = y.cpu().numpy().astype(np.float64)
    assert np.linalg.norm(got - c_ref) / np.linalg.norm(c_ref) <= 1e-5
    w.close()

    # a wait whose flags are all raised returns at once, without an error
    flags.fill_(1)
    t0 = time.monotonic()
    assert ctx.lib.sc_allgather_wait(ctx.ptr, ctypes.c_void_p(flags.data_ptr()), 2, 1, stream) == abi.OK
    ctx.poll_errors()
    assert time.monotonic() - t0 < 1.0


def test_wait_arguments_are_checked(ctx):
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    flags = torch.ones(2, dtype=torch.int32, device="cuda")
    p = ctypes.c_void_p(flags.data_ptr())
    assert ctx.lib.sc_allgather_wait(ctx.ptr, p, 2, 0, stream) == abi.INVALID_ARG   # epoch 0 is reserved
    assert ctx.lib.sc_allgather_wait(ctx.ptr, p, 9, 1, stream) == abi.INVALID_ARG   # at most 8 ranks
    assert ctx.lib.sc_allgather_wait(ctx.ptr, None, 2, 1, stream) == abi.INVALID_ARG
    ctx.poll_errors()
