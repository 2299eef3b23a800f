"""Token-row sharding and output gather on CPU ranks (gloo, world size 2 and 3).

The FFN kernels need a B200, so a row-wise stand-in layer takes their place:
what is tested is the partition, the per-rank compute on its own rows, the
all-gather of uneven blocks, and that a rank that dies makes the others fail
within the process-group timeout instead of hanging.
"""
import os
import socket
from datetime import timedelta

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from flashvsr_optimizations_b200.sharding import ShardedFFN, gather_rows, row_range


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


class _RowLayer(torch.nn.Module):
    """Row-wise stand-in for the FFN: y = tanh(x W) + row_sum(x), no cross-row mixing."""

    def __init__(self, d):
        super().__init__()
        g = torch.Generator().manual_seed(0)
        self.w = torch.randn(d, d, generator=g)

    def forward(self, x):
        return torch.tanh(x @ self.w) + x.sum(dim=1, keepdim=True)


def _worker(rank, world, port, total, d, q):
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=30))
        x = torch.randn(total, d, generator=torch.Generator().manual_seed(1))
        layer = _RowLayer(d)
        y = ShardedFFN(layer)(x)
        ok = torch.allclose(y, layer(x), atol=1e-6, rtol=1e-6)
        # gathering into a caller's buffer gives the same rows in place
        lo, hi = row_range(total, world, rank)
        out = torch.full((total, d), float("nan"))
        got = gather_rows(x[lo:hi] * 2.0, total, out=out)
        ok = ok and got.data_ptr() == out.data_ptr() and torch.equal(out, x * 2.0)
        q.put((rank, bool(ok), tuple(y.shape)))
        dist.barrier()
        dist.destroy_process_group()
    except Exception as e:  # pragma: no cover - reported to the parent
        q.put((rank, False, repr(e)))


@pytest.mark.parametrize("world,total", [(2, 7680), (2, 131), (3, 10), (3, 2), (4, 15360), (4, 15363)])
def test_sharded_ffn_matches_single_rank(world, total):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, total, 16, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = [q.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
    for rank, ok, info in results:
        assert ok, (rank, info)
        assert info == (total, 16)


def test_row_range_partitions_exactly():
    for total in (0, 1, 7, 7680, 64800):
        for world in (1, 2, 3, 4, 8):
            spans = [row_range(total, world, r) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == total
            assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
            sizes = [e - s for s, e in spans]
            assert max(sizes) - min(sizes) <= 1
    with pytest.raises(ValueError):
        row_range(10, 2, 2)


def _dying_worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=5))
    if rank == 1:
        os._exit(3)          # the rank dies between steps, before the gather
    try:
        gather_rows(torch.ones(4, 8), 8)
        q.put((rank, "no error"))
    except Exception as e:
        q.put((rank, type(e).__name__))


def test_dead_rank_makes_gather_fail_instead_of_hanging():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_dying_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    rank, outcome = q.get(timeout=120)
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    assert rank == 0 and outcome != "no error"


def _amax_worker(rank, world, port, q):
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=30))
        from flashvsr_optimizations_b200.sharding import global_amax
        a = torch.tensor([float(rank + 1) * 1.5])
        global_amax(a)
        q.put((rank, float(a.item())))
        dist.barrier()
        dist.destroy_process_group()
    except Exception as e:  # pragma: no cover
        q.put((rank, repr(e)))


def test_global_amax_is_the_max_over_ranks():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_amax_worker, args=(r, 3, port, q)) for r in range(3)]
    for p in procs:
        p.start()
    results = [q.get(timeout=120) for _ in range(3)]
    for p in procs:
        p.join(timeout=60)
    assert sorted(v for _, v in results) == [4.5, 4.5, 4.5]
