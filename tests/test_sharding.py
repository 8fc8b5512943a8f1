"""Host logic of the multi-GPU row sharding, on CPU with gloo ranks
(world size 2 and 3): every row is owned exactly once, the validation
all-gather reassembles C exactly, and a rank that fails makes the others
fail within a short process-group timeout instead of hanging."""
import datetime
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from gb300_microbench_b200.sharding import row_shard, sharded_gemm


@pytest.mark.parametrize("m,world,granule", [(4096, 8, 128), (512, 8, 128), (1000, 3, 64), (16384, 4, 256),
                                             (7, 4, 1), (0, 2, 1)])
def test_row_shard_partitions_rows(m, world, granule):
    shards = [row_shard(m, world, r, granule) for r in range(world)]
    covered = []
    for s in shards:
        covered += list(range(s.row0, s.row0 + s.rows))
    assert covered == list(range(m))
    sizes = [s.rows for s in shards]
    assert max(sizes) - min(sizes) <= granule
    if m > 0:
        assert shards[0].rows > 0  # rank 0 (which writes the results) always holds rows


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, fail_rank, results, m_rows=300):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=10))
    try:
        g = torch.Generator().manual_seed(0)
        a = torch.randn(m_rows, 64, generator=g)
        b = torch.randn(40, 64, generator=g)
        if rank == fail_rank:
            raise RuntimeError("injected rank failure before the validation all-gather")
        c_local, full, me = sharded_gemm(a, b, world, rank, lambda x, y: x @ y.t(), granule=32)
        ok = torch.equal(full, a @ b.t()) and c_local.shape[0] == me.rows
        results[rank] = "ok" if ok else "mismatch"
    except RuntimeError as exc:
        results[rank] = f"error: {exc}"[:200]
    finally:
        try:
            dist.destroy_process_group()
        except Exception:
            pass


def _run(world, fail_rank=-1, m_rows=300):
    port = _free_port()
    with mp.Manager() as mgr:
        results = mgr.dict()
        mp.spawn(_worker, args=(world, port, fail_rank, results, m_rows), nprocs=world, join=True)
        return dict(results)


@pytest.mark.parametrize("world", [2, 3])
def test_gloo_sharded_gemm_reassembles_exactly(world):
    res = _run(world)
    assert res == {r: "ok" for r in range(world)}


def test_failed_rank_surfaces_on_every_rank():
    res = _run(2, fail_rank=1)
    assert res[1].startswith("error: injected")
    assert res[0].startswith("error")  # the survivor's all-gather ends with an error, not a hang


def test_gloo_sharded_gemm_with_empty_ranks():
    """40 rows in 32-row granules over 3 ranks: two granules, so rank 2's
    block is empty; it still joins the all-gather and C reassembles."""
    res = _run(3, m_rows=40)
    assert res == {r: "ok" for r in range(3)}
