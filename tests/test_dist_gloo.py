"""Halo exchange of the row-partitioned path on CPU ranks (gloo)."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from diagpu_b200.dist import Halo, row_block


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, n, lo, hi, K, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        h = Halo(n, world, rank, lo, hi)
        ext = torch.full((K, h.width + 5), -1.0)     # padded pitch, non-contiguous slices
        cols = torch.arange(h.xlo, h.xhi, dtype=torch.float32)
        own = (cols >= h.r0) & (cols < h.r1)
        for k in range(K):
            ext[k, :h.width][own] = cols[own] + 1000.0 * k
        h.start(ext).wait()
        expect = torch.stack([cols + 1000.0 * k for k in range(K)])
        ok = bool(torch.equal(ext[:, :h.width], expect))
        a, b = h.interior()
        ok &= h.r0 <= a <= b <= h.r1
        q.put((rank, ok, (h.r0, h.r1, h.xlo, h.xhi)))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,n,lo,hi,K", [(2, 1000, -70, 70, 1), (3, 1000, -40, 7, 3),
                                              (2, 4096, -1, 300, 2), (4, 50000, -6000, 6000, 1)])
def test_halo_exchange(world, n, lo, hi, K):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_worker, args=(r, world, port, n, lo, hi, K, q)) for r in range(world)]
    for p in ps:
        p.start()
    res = [q.get(timeout=120) for _ in ps]
    for p in ps:
        p.join(timeout=60)
    assert all(ok for _, ok, _ in res), res


def test_halo_too_wide_rejected():
    with pytest.raises(ValueError):
        Halo(1000, 8, 0, -200, 200)


def test_row_blocks_cover():
    for n, w in ((67108864, 8), (1000, 3), (33, 2)):
        blocks = [row_block(n, w, r) for r in range(w)]
        assert blocks[0][0] == 0 and blocks[-1][1] == n


def _leaver(rank, world, port, q):
    """Rank 1 leaves between steps, before the halo exchange; rank 0 must
    get an error from its exchange within the process-group timeout, not
    hang."""
    import datetime
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=4))
    h = Halo(1000, world, rank, -30, 30)
    ext = torch.zeros(h.width)
    if rank == 1:
        os._exit(7)   # leaves between steps; reported through the exit code
    try:
        h.start(ext).wait(timeout=datetime.timedelta(seconds=4))
        q.put((rank, "no error"))
    except Exception as e:  # noqa: BLE001 - any distributed error is the expected outcome
        q.put((rank, "error: " + type(e).__name__))


def test_missing_peer_is_reported_not_hung():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_leaver, args=(r, 2, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    rank, res = q.get(timeout=120)
    for p in ps:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    assert rank == 0 and res.startswith("error"), res
    assert ps[1].exitcode == 7
