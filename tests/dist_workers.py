"""Worker bodies of the multi-process CPU tests (spawned ranks on the gloo backend)."""
import os
import traceback
from datetime import timedelta

import numpy as np


def _init(rank, world, port, timeout_s=30):
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=timeout_s))
    return dist


def column_parallel_worker(rank, world, port, m, k, n, seed, result_dir):
    """Each rank computes its column block with a CPU stand-in for the local product (the oracle,
    on the shard's columns); the gathered y must equal the single-process product."""
    try:
        import torch
        import oracle
        from siliconed_b200.parallel import ColumnParallelLinear
        dist = _init(rank, world, port)
        g = np.random.default_rng(seed)
        x = (g.standard_normal((m, k), dtype=np.float32).view(np.uint32) >> 16).astype(np.uint16)
        q = g.integers(-128, 128, (k, n), dtype=np.int16).astype(np.int8)
        s = (np.abs(g.standard_normal(n)) * 1e-3 + 1e-5).astype(np.float32)
        b = (g.standard_normal(n, dtype=np.float32).view(np.uint32) >> 16).astype(np.uint16)

        def make_local(n0, n1):
            def local(xt, bias_shard):
                _, y = oracle.linear_int8(xt.numpy(), np.ascontiguousarray(q[:, n0:n1]), s[n0:n1],
                                          None if bias_shard is None else bias_shard.numpy())
                return torch.from_numpy((y.astype(np.uint32) << 16).view(np.float32))  # gloo: no 16-bit types
            return local

        layer = ColumnParallelLinear(n, make_local)
        y = layer(torch.from_numpy(x), torch.from_numpy(b)).numpy()
        _, ref = oracle.linear_int8(x, q, s, b)
        ok = bool(np.array_equal(y.view(np.uint32), ref.astype(np.uint32) << 16))
        dist.barrier()
        dist.destroy_process_group()
        with open(os.path.join(result_dir, f"rank{rank}"), "w") as f:
            f.write("ok" if ok else "mismatch")
    except Exception:  # reported to the parent through the result file
        with open(os.path.join(result_dir, f"rank{rank}"), "w") as f:
            f.write("error\n" + traceback.format_exc())


def failed_rank_worker(rank, world, port, result_dir):
    """Rank 1 leaves before the gather (between steps, nothing in flight); rank 0's gather must end
    with an error within the process group's short timeout, not wait forever."""
    import torch
    try:
        dist = _init(rank, world, port, timeout_s=5)
        from siliconed_b200.parallel import gather_columns
        if rank == 1:
            with open(os.path.join(result_dir, f"rank{rank}"), "w") as f:
                f.write("left")
            os._exit(0)
        try:
            gather_columns(torch.zeros((4, 8), dtype=torch.float32), [(0, 8), (8, 16)])
            outcome = "no error"
        except Exception as e:  # the expected path
            outcome = "error: " + type(e).__name__
        with open(os.path.join(result_dir, f"rank{rank}"), "w") as f:
            f.write(outcome)
        os._exit(0)
    except Exception:
        with open(os.path.join(result_dir, f"rank{rank}"), "w") as f:
            f.write("setup error\n" + traceback.format_exc())
        os._exit(0)
