"""Multi-GPU host logic on the CPU: shard ranges, the column-parallel gather, a failed rank (gloo)."""
import os
import socket

import pytest
import torch.multiprocessing as mp

import dist_workers
from siliconed_b200.parallel import batch_range, column_ranges


def free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("n,world", [(3072, 2), (3072, 8), (1030, 3), (10240, 8), (12, 8), (1, 2)])
def test_column_ranges_cover_exactly(n, world):
    r = column_ranges(n, world)
    assert len(r) == world and r[0][0] == 0 and r[-1][1] == n
    for (a, b), (c, d) in zip(r, r[1:]):
        assert b == c and a <= b
    for a, b in r[:-1]:
        assert a % 8 == 0 and b % 8 == 0
    widths = [b - a for a, b in r]
    assert max(widths) - min(widths) <= 8 or n < 8 * world


@pytest.mark.parametrize("m,world", [(4096, 8), (8, 8), (9, 2), (1, 4)])
def test_batch_ranges_partition(m, world):
    rows = [batch_range(m, world, r) for r in range(world)]
    assert rows[0][0] == 0 and rows[-1][1] == m
    assert all(a <= b for a, b in rows) and all(rows[i][1] == rows[i + 1][0] for i in range(world - 1))


def _spawn(fn, world, args, tmp_path):
    ctx = mp.get_context("spawn")
    procs = [ctx.Process(target=fn, args=(r, world, *args)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    for p in procs:
        if p.is_alive():
            p.kill()
            p.join()
    return {r: open(os.path.join(tmp_path, f"rank{r}")).read() if os.path.exists(os.path.join(tmp_path, f"rank{r}"))
            else "missing" for r in range(world)}


@pytest.mark.parametrize("world,n", [(2, 96), (3, 100)])
def test_column_parallel_gather_equals_single_process(tmp_path, world, n):
    res = _spawn(dist_workers.column_parallel_worker, world, (free_port(), 5, 64, n, 11, str(tmp_path)), tmp_path)
    assert all(v == "ok" for v in res.values()), res


def test_a_rank_that_leaves_ends_the_gather_with_an_error(tmp_path):
    res = _spawn(dist_workers.failed_rank_worker, 2, (free_port(), str(tmp_path)), tmp_path)
    assert res[1] == "left", res
    assert res[0].startswith("error"), res
