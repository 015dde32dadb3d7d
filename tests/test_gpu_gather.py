"""The gathering product (sc_linear_allgather) on one rank: world 1, this rank's y its only output.

The column-parallel gather of several GPUs stores each output tile into every rank's y from the product's
epilogue.  Its per-rank shards are narrow (config 1 over 8 GPUs: 384 columns a rank, 24 pair tiles for 74
pairs), and such products are cut into 256-row x 128-column pieces so that more SMs share the stores.  On one
GPU the same kernel runs with world 1: its y must equal, bit for bit, the plain product of the same shard
(sc_linear: the same operands in the same K order), for shards that are cut into pieces (384 columns; 200
columns of 1000 ragged rows) and one that is not (1536), and the rank's flag must be raised to the call's
epoch on two calls in a row.
"""
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


@pytest.mark.parametrize("m,k,n", [(4096, 3072, 384), (4096, 3072, 1536), (1000, 1024, 200)])
def test_the_gathering_product_on_one_rank_equals_the_product(ctx, m, k, n):
    g = np.random.default_rng(m + k + n)
    x = torch.from_numpy(configs.to_bf16_bits(g.standard_normal((m, k), dtype=np.float32)).view(np.int16)).cuda()
    q = g.integers(-128, 128, (k, n), dtype=np.int16).astype(np.int8).view(np.uint8)
    s = (np.abs(g.standard_normal(n)) * 0.02 / 127 + 1e-6).astype(np.float32)
    b = torch.from_numpy(configs.to_bf16_bits(g.standard_normal(n, dtype=np.float32) * 0.01).view(np.int16)).cuda()
    w = QuantizedWeight(ctx, q, abi.WEIGHT_INT8, s)
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    ws = torch.empty(w.workspace_bytes(max(m, 1536)), dtype=torch.uint8, device="cuda")
    ref = torch.empty((m, n), dtype=torch.int16, device="cuda")
    ctx.check(ctx.lib.sc_linear(ctx.ptr, w.ptr, ctypes.c_void_p(x.data_ptr()), m, ctypes.c_void_p(b.data_ptr()),
                                ctypes.c_void_p(ref.data_ptr()), ctypes.c_void_p(ws.data_ptr()), ws.numel(), stream))
    flags = torch.zeros(1, dtype=torch.int32, device="cuda")
    for epoch in (1, 2):
        y = torch.full((m, n), -1, dtype=torch.int16, device="cuda")
        ys = (ctypes.c_void_p * 1)(y.data_ptr())
        fs = (ctypes.c_void_p * 1)(flags.data_ptr())
        ctx.check(ctx.lib.sc_linear_allgather(ctx.ptr, w.ptr, ctypes.c_void_p(x.data_ptr()), m,
                                              ctypes.c_void_p(b.data_ptr()), ys, fs, 1, 0, 0, n, epoch,
                                              ctypes.c_void_p(ws.data_ptr()), ws.numel(), stream))
        ctx.check(ctx.lib.sc_allgather_wait(ctx.ptr, ctypes.c_void_p(flags.data_ptr()), 1, epoch, stream))
        torch.cuda.synchronize()
        ctx.poll_errors()
        assert int(flags[0].item()) == epoch
        assert torch.equal(y, ref), f"epoch {epoch}: {(y != ref).sum().item()} outputs differ"
    w.close()
