"""The fused column-parallel gather (sc_linear_allgather) on 2+ GPUs of one box: every rank's y equals
the single-GPU product bit for bit (the same sums in the same order), over consecutive calls that
alternate the double buffer.  Runs its ranks as child processes (NCCL for set-up only); skipped with
fewer than two GPUs."""
import os
import socket

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

if not torch.cuda.is_available() or torch.cuda.device_count() < 2:
    pytest.skip("needs two CUDA devices", allow_module_level=True)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, results, multicast=False):
    import torch.distributed as dist
    from datetime import timedelta
    from siliconed_b200 import configs, parallel
    from siliconed_b200.products import Context, QuantizedWeight
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    ctx = fused = full = None
    try:
        ctx = Context(rank)
        case = configs.config1(m=1600, k=512, n=1000)
        bias = torch.from_numpy(case.bias.view(np.int16)).cuda().view(torch.bfloat16)
        fused = parallel.FusedColumnParallelLinear(ctx, case.codes_nk, case.kind, case.scales, case.n, 2048,
                                                   published_nk=True, bias=bias, multicast=multicast)
        results[f"mc{rank}"] = fused.uses_multicast
        full = QuantizedWeight(ctx, case.codes_nk, case.kind, case.scales, published_nk=True)
        ok = True
        for call in range(3):
            x = torch.from_numpy(case.x.view(np.int16)).cuda().view(torch.bfloat16)
            if call == 1:
                x = x[: 1536].contiguous()
            y = fused(x)
            ref = full.linear(x, bias=bias)
            torch.cuda.synchronize()
            ctx.poll_errors()
            ok &= bool(torch.equal(y.view(torch.int16), ref.view(torch.int16)))
        results[rank] = ok
        dist.barrier()
    finally:
        # Every wait a rank can meet is bounded (the device-side waits at 2 s, the process group at 60 s), so
        # a rank that fails gets here by itself and releases its outputs (and their multicast binding) before
        # it exits; nothing ends it from outside.
        torch.cuda.synchronize()
        if fused is not None:
            fused.close()
        if full is not None:
            full.close()
        if ctx is not None:
            ctx.close()
        dist.destroy_process_group()


@pytest.mark.parametrize("multicast", [False, True])
def test_fused_gather_matches_single_gpu_product(multicast):
    """Peer stores to every rank (multicast False), or one multimem store per piece to the outputs'
    NVLink multicast address when the system offers one (multicast True; else it takes the peer path)."""
    import torch.multiprocessing as mp
    world = 2
    ctx = mp.get_context("spawn")
    manager = ctx.Manager()
    results = manager.dict()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, results, multicast)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=600)
    # A rank still alive here has outlived every bound it waits under; the test fails without ending it
    # from outside (its outputs may be bound to an NVLink multicast object).
    assert not any(p.is_alive() for p in procs), "a rank did not exit within its bounded waits"
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    got = dict(results)
    assert got[0] is True and got[1] is True, got
    assert got["mc0"] == got["mc1"] and (multicast or not got["mc0"]), got
    print("multicast outputs:", got["mc0"])
