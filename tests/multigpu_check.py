"""Multi-GPU check of the row-partitioned products (run under torchrun).

    python -m torch.distributed.run --nnodes=1 --nproc-per-node N \\
        --master-addr 127.0.0.1 --master-port 29533 tests/multigpu_check.py

Every rank builds its row block of a 27-point-stencil matrix (3D grid
256 x 256 x 64, offsets up to +-65,793, so every block needs halo rows
from both neighbours), runs the partitioned SpMV and C = A*A through
diagpu_b200.dist, and compares its rows bit for bit with the same
products computed for the whole matrix on its own GPU.  SpMV runs four
steps with a new x each step in every exchange mode: the fused peer-halo
kernel (halo pushed over NVLink inside the step kernel, receive buffers
alternating by step parity) and the three NCCL forms.  Prints one PASS/FAIL line
per rank; exit code 0 only if all ranks pass.
"""
import os
import sys

import numpy as np
import torch
import torch.distributed as dist

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)
import diagpu_b200 as dg  # noqa: E402
from diagpu_b200.dist import DistSpmspm, DistSpmv, Halo  # noqa: E402


def main():
    world = int(os.environ["WORLD_SIZE"])
    rank = int(os.environ["RANK"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", device_id=torch.device("cuda", local))
    n = 256 * 256 * 64
    offs = np.array([i + 256 * j + 65536 * k for k in (-1, 0, 1) for j in (-1, 0, 1)
                     for i in (-1, 0, 1)], np.int32)
    h = Halo(n, world, rank, int(offs.min()), int(offs.max()))
    A = dg.DiaRows.synth(n, n, offs, 11, vrow0=h.r0, nrows=h.r1 - h.r0)
    Af = dg.DiaRows.synth(n, n, offs, 11)
    ok_y = True
    modes = {3: "peer", 2: "nccl-overlap2", 1: "nccl-overlap1", 0: "nccl-serial"}
    for mode, name in modes.items():
        ds = DistSpmv(A, h, overlap=mode)
        for step in range(4):
            seed = 12 + 7 * step + 100 * mode
            dg.synth_vector(h.r1 - h.r0, seed, i0=h.r0, out=ds.x_own)
            y = ds.step()[:h.r1 - h.r0].clone()
            yf = dg.spmv(Af, dg.synth_vector(n, seed))[h.r0:h.r1]
            good = bool(torch.equal(y, yf))
            if not good:
                print(f"rank {rank} {name} step {step}: MISMATCH", flush=True)
            ok_y &= good
        if mode == 3:
            st = ds.native.status() if ds.native is not None else 0
            if st:
                print(f"rank {rank} peer status {st}", flush=True)
                ok_y = False
        del ds
    B_ext = dg.DiaRows.empty(n, n, offs, vrow0=h.xlo, nrows=h.width, zero=True)
    B_ext.vals[:, h.r0 - h.xlo:h.r1 - h.xlo] = A.vals[:, :h.r1 - h.r0]
    dm = DistSpmspm(A, B_ext, h)
    Cd = dm.step().vals[:, :h.r1 - h.r0].clone()
    torch.cuda.synchronize()
    dist.barrier()

    Cf = dg.spmspm(Af, Af)
    ok_c = np.array_equal(Cf.offsets, dm.C.offsets) and bool(
        torch.equal(Cd, Cf.vals[:, h.r0:h.r1]))
    ok = ok_y and ok_c
    print(f"rank {rank}/{world} rows [{h.r0},{h.r1}) spmv {'ok' if ok_y else 'MISMATCH'} "
          f"spmspm {'ok' if ok_c else 'MISMATCH'} -> {'PASS' if ok else 'FAIL'}", flush=True)
    t = torch.tensor([0 if ok else 1], device="cuda")
    dist.all_reduce(t)
    dist.destroy_process_group()
    sys.exit(int(t.item() != 0))


if __name__ == "__main__":
    main()
