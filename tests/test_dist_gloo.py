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


def _hb_worker(rank, world, port, mode, q):
    """Three ranks step with heartbeats; rank 1 leaves after two steps
    (announced, or silently).  Ranks 0 and 2 must raise PeerLost before
    their third step's launch instead of waiting on rank 1."""
    import datetime
    from diagpu_b200.dist import Heartbeat, PeerLost
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=20))
    h = Halo(3000, world, rank, -30, 30)
    hb = Heartbeat(h, timeout=2.0)
    ext = torch.zeros(h.width)
    done = 0
    try:
        for step in range(4):
            if rank == 1 and step == 2:
                # between steps: its last exchange has been delivered
                # (neighbours finished step 1) before it goes
                import time
                time.sleep(1.0)
                if mode == "announced":
                    hb.leave()
                q.put((rank, "left", done))
                q.close()
                q.join_thread()
                os._exit(0)
            hb.beat()
            h.start(ext).wait(timeout=datetime.timedelta(seconds=20))
            done += 1
        q.put((rank, "no error", done))
    except PeerLost as e:
        q.put((rank, "PeerLost: " + str(e), done))
    except Exception as e:  # noqa: BLE001 - reported to the test as a failure
        q.put((rank, "other error: " + repr(e)[:200], done))
    q.close()
    q.join_thread()   # flush before the hard exit below
    if rank == 0:
        import time
        time.sleep(3.0)   # rank 0 hosts the store the others are still reading
    os._exit(0)


@pytest.mark.parametrize("mode", ["announced", "silent"])
def test_heartbeat_reports_a_rank_that_left_between_steps(mode):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_hb_worker, args=(r, 3, port, mode, q)) for r in range(3)]
    for p in ps:
        p.start()
    res = {}
    for _ in range(3):
        r, msg, done = q.get(timeout=120)
        res[r] = (msg, done)
    for p in ps:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    assert res[1][0] == "left"
    for r in (0, 2):
        assert res[r][0].startswith("PeerLost"), res
        assert res[r][1] == 2, res     # both full steps ran; the third never launched
