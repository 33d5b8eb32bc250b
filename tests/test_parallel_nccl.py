"""mlx_nufft_b200.parallel on two GPUs over NCCL (skipped with fewer than two
GPUs): two spawned ranks, one per GPU, run

  * type 1 split by point (per-rank spread + all-reduce of the fine grid),
  * type 2 split by target (root's grid broadcast + per-rank interp,
    gathered in caller order),

on real plans and compare with one plan over all points on GPU 0.  The
process group uses a short timeout; NVLS is off (NCCL_NVLS_ENABLE=0), and
no kernel of this library waits on another rank.
"""

import os
import socket

import numpy as np
import pytest

from oracle import port

pytestmark = pytest.mark.gpu


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _inputs():
    rng = np.random.default_rng(11)
    M, N = 200_000, (96, 80)
    x = [rng.uniform(-np.pi, np.pi, M) for _ in range(2)]
    c = rng.standard_normal(M) + 1j * rng.standard_normal(M)
    f = rng.standard_normal(N) + 1j * rng.standard_normal(N)
    return x, c, f, M, N


def _worker(rank, world, port_, queue):
    import datetime
    import torch
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port_),
                      NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    try:
        from mlx_nufft_b200 import Type1PlanND, Type2PlanND, parallel as par
        x, c, f, M, N = _inputs()
        lo, hi = par.split_range(M, rank, world)
        xl = tuple(v[lo:hi] for v in x)
        p1 = Type1PlanND(xl, N, eps=1e-6)
        r1 = par.Type1PointSplit(par.PlanStages(p1)).execute(c[lo:hi])
        p2 = Type2PlanND(xl, N, eps=1e-6)
        r2 = par.Type2TargetSplit(par.PlanStages(p2), M).execute(
            f if rank == 0 else np.zeros(N), gather=True)
        torch.cuda.synchronize()
        queue.put((rank, np.asarray(r1), np.asarray(r2)))
        dist.barrier()
    finally:
        dist.destroy_process_group()


def test_split_type1_type2_over_nccl():
    import torch
    import torch.multiprocessing as mp
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port_ = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port_, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = {}
    for _ in procs:
        r, a, b = q.get(timeout=300)
        res[r] = (a, b)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    from mlx_nufft_b200 import Type1PlanND, Type2PlanND
    x, c, f, M, N = _inputs()
    ref1 = Type1PlanND(tuple(x), N, eps=1e-6).execute(c)
    ref2 = Type2PlanND(tuple(x), N, eps=1e-6).execute(f)
    for r in (0, 1):
        # float atomics / summation order only
        assert port.rel_l2(res[r][0].reshape(N), ref1) <= 1e-6
        np.testing.assert_array_equal(res[r][1], ref2)
