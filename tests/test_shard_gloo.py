"""Multi-process sharding on CPU (gloo, world size 2): shard maps cover every
unit exactly once, each rank's slice computed with the oracle and all-gathered
reassembles the full result, and a rank that leaves early makes the other
rank's collective fail within the process-group timeout instead of hanging."""
import math
import os
import socket
import sys
from datetime import timedelta
from pathlib import Path

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

ROOT = Path(__file__).resolve().parent.parent
sys.path.insert(0, str(ROOT))

from neso_b200 import shard  # noqa: E402


@pytest.mark.parametrize("n,world,align", [(0, 2, 1), (1, 2, 1), (256, 8, 1), (11008, 8, 16), (11008, 3, 16),
                                           (1 << 28, 8, 1024), (1000, 4, 128), (5, 8, 1)])
def test_shard_range_partitions(n, world, align):
    shards = [shard.shard_range(n, world, r, align) for r in range(world)]
    assert shards[0].start == 0 and shards[-1].stop == n
    for a, b in zip(shards, shards[1:]):
        assert a.stop == b.start
    for s in shards[:-1]:
        assert s.stop % align == 0 or s.stop == n
    sizes = [s.size for s in shards]
    assert sum(sizes) == n
    assert max(sizes) - min(sizes) <= align


def test_quant_columns_8_gpus():
    # BASELINE: N = 11008 over 8 GPUs -> 1376 columns each (a multiple of 16, not of 128)
    sizes = [shard.shard_columns(11008, 8, r).size for r in range(8)]
    assert sizes == [1376] * 8


def _free_port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, mode, results):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.set_num_threads(1)
    sys.path.insert(0, str(ROOT))
    import oracle
    from neso_b200 import shard as sh

    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=10))
    try:
        if mode == "attention":
            g = torch.Generator().manual_seed(0)
            B, H, S, D = 2, 3, 64, 64
            q, k, v = (torch.randn(B, H, S, D, generator=g).half() for _ in range(3))
            table = torch.randn(H, 2 * S - 1, generator=g) * 0.02
            piece, s = sh.attention_sharded(q, k, v, lambda a, b, c, **kw: oracle.attention(a, b, c, 0.125, **kw),
                                            world, rank, table=table)
            sizes = [sh.shard_heads(B, H, world, r).size for r in range(world)]
            full = sh.gather(piece, sizes, dim=0).reshape(B, H, S, D)
            ref = oracle.attention(q, k, v, 0.125, table=table)
            results[rank] = bool(torch.allclose(full, ref, atol=1e-5))
        elif mode == "matmul":
            g = torch.Generator().manual_seed(1)
            a = torch.randn(40, 64, generator=g).half()
            b = torch.randn(64, 200, generator=g).half()
            piece, s = sh.matmul_sharded(a, b, oracle.gemm, world, rank)
            sizes = [sh.shard_columns(200, world, r).size for r in range(world)]
            full = sh.gather(piece, sizes, dim=1)
            results[rank] = bool(torch.allclose(full, oracle.gemm(a, b), atol=1e-4))
        elif mode == "drop":
            if rank == 1:
                results[rank] = "left"
                return  # leaves between steps, before the collective, without destroying the group
            t = torch.ones(4)
            try:
                dist.all_reduce(t)
                results[rank] = "no-error"
            except Exception as e:  # gloo reports the missing peer within the timeout
                results[rank] = "error:" + type(e).__name__
    finally:
        if mode != "drop":
            dist.destroy_process_group()


def _spawn(mode, world=2):
    port = _free_port()
    mgr = mp.get_context("spawn").Manager()
    results = mgr.dict()
    ctx = mp.spawn(_worker, args=(world, port, mode, results), nprocs=world, join=False)
    ok = ctx.join(timeout=120)
    while not ok:
        ok = ctx.join(timeout=120)
    return dict(results)


def test_attention_sharded_over_batch_heads_gloo():
    res = _spawn("attention")
    assert res == {0: True, 1: True}


def test_matmul_sharded_over_columns_gloo():
    res = _spawn("matmul")
    assert res == {0: True, 1: True}


def test_rank_leaving_early_fails_collective_not_hangs():
    res = _spawn("drop")
    assert res[1] == "left"
    assert str(res[0]).startswith("error:")
