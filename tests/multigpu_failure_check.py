"""Failure detection of the native communicator on 2 GPUs (run under torchrun).

    NCCL_NVLS_ENABLE=0 python -m torch.distributed.run --nnodes=1 --nproc-per-node 2 \\
        --master-addr 127.0.0.1 --master-port 29535 tests/multigpu_failure_check.py

1. Both ranks create a non-blocking communicator (dia_dist_create_timeout)
   and run four NCCL-exchanged partitioned SpMV steps; every step must equal
   the whole-matrix product bit for bit.
2. Rank 1 never joins a second communicator: rank 0's
   dia_dist_create_timeout(5 s) must return DIA_ERR_TIMEOUT (communicator
   aborted) in well under a minute instead of blocking.  Nothing is launched
   on either GPU for it; the failure is made on the host.
Unique ids travel over a gloo group.  Prints PASS/FAIL per rank; exit code
0 only if both pass.
"""
import ctypes as C
import os
import sys
import time

import numpy as np
import torch
import torch.distributed as dist

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)
import diagpu_b200 as dg  # noqa: E402
from diagpu_b200.dist import DistSpmv, Halo  # noqa: E402


def new_id(rank):
    buf = (C.c_char * 128)()
    if rank == 0:
        dg.check(dg.lib().dia_nccl_unique_id(buf, 128))
    obj = [bytes(buf.raw)]
    dist.broadcast_object_list(obj, src=0)
    return (C.c_char * 128).from_buffer_copy(obj[0])


class Comm:
    def __init__(self, h):
        self._h = h

    @property
    def handle(self):
        return self._h


def main():
    world, rank = int(os.environ["WORLD_SIZE"]), int(os.environ["RANK"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dist.init_process_group("gloo")
    L = dg.lib()
    ok = True
    # 1. a working non-blocking communicator, NCCL-mode steps
    h = C.c_void_p()
    dg.check(L.dia_dist_create_timeout(rank, world, new_id(rank), 30000, C.byref(h)))
    n = 256 * 256 * 16
    offs = np.array([i + 256 * j + 65536 * k for k in (-1, 0, 1) for j in (-1, 0, 1)
                     for i in (-1, 0, 1)], np.int32)
    hl = Halo(n, world, rank, int(offs.min()), int(offs.max()))
    A = dg.DiaRows.synth(n, n, offs, 61, vrow0=hl.r0, nrows=hl.r1 - hl.r0)
    Af = dg.DiaRows.synth(n, n, offs, 61)
    ds = DistSpmv(A, hl, native=Comm(h), overlap=2)
    for step in range(4):
        dg.synth_vector(hl.r1 - hl.r0, 70 + step, i0=hl.r0, out=ds.x_own)
        y = ds.step()[:hl.r1 - hl.r0]
        ok &= bool(torch.equal(y, dg.spmv(Af, dg.synth_vector(n, 70 + step))[hl.r0:hl.r1]))
    torch.cuda.synchronize()
    dist.barrier()
    dg.check(L.dia_dist_destroy(h))
    msg = f"steps {'ok' if ok else 'MISMATCH'}"
    # 2. rank 1 never joins
    uid = new_id(rank)
    if rank == 0:
        h2 = C.c_void_p()
        t0 = time.monotonic()
        rc = L.dia_dist_create_timeout(rank, world, uid, 5000, C.byref(h2))
        dt = time.monotonic() - t0
        good = rc == dg.DIA_ERR_TIMEOUT and dt < 60
        msg += f"; missing rank: rc={rc} after {dt:.1f} s ({L.dia_last_error().decode()[:80]})"
        ok &= good
    dist.barrier()
    print(f"rank {rank}/{world} {msg} -> {'PASS' if ok else 'FAIL'}", flush=True)
    t = torch.tensor([0 if ok else 1])
    dist.all_reduce(t)
    dist.destroy_process_group()
    sys.exit(int(t.item() != 0))


if __name__ == "__main__":
    main()
