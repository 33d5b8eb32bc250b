"""nufft_interp_noalloc: the type-2 interpolation stage for callers that must
not allocate device memory (a host framework that owns the GPU's memory
budget through its own allocator, a latency-critical loop that cannot pay
for cudaMalloc / cudaFree).  It keeps its per-point scratch in one static
device array instead of plan memory.

Checked through the C ABI against the existing entry point: a type-2 plan
(global method, caller order) executes, leaving its transformed fine grid in
plan memory (nufft_get_grid); interpolating that grid with the no-alloc
entry point must reproduce the plan's output within the suite's tolerance,
on two calls in a row (the second call reuses the shared scratch left by the
first).  This file is named to be collected last.
"""

import ctypes

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

TOL = 1e-5      # max(10 * eps, 1e-5) at eps = 1e-6, as in the other GPU tests


@pytest.mark.parametrize("dim,N,M", [(1, (4096,), 200_000),
                                     (2, (96, 80), 100_000),
                                     (3, (24, 20, 16), 60_000)])
def test_interp_noalloc_matches_plan(dim, N, M):
    import torch
    from mlx_nufft_b200 import Type2PlanND
    from mlx_nufft_b200._lib import check, lib
    from oracle import port

    rng = np.random.default_rng(2024 + dim)
    x = [rng.uniform(-np.pi, np.pi, M) for _ in range(dim)]
    fk = rng.standard_normal(N) + 1j * rng.standard_normal(N)
    eps = 1e-6
    plan = Type2PlanND(tuple(x), N, eps=eps, isign=-1, spread_method="gm",
                       sort_points=False)
    ref = plan.execute(fk)                  # existing entry: nufft_execute
    grid_ptr, ncomplex = plan._plan.grid()  # its post-FFT fine grid
    assert ncomplex >= int(np.prod(plan.n_up))
    xs = [torch.from_numpy(v).cuda() for v in x] + [None] * (3 - dim)
    n = (ctypes.c_int64 * 3)(*(list(plan.n_up) + [1] * (3 - dim)))
    stream = torch.cuda.current_stream().cuda_stream
    outs = []
    for _ in range(2):
        out = torch.full((M,), float("nan"), dtype=torch.complex64, device="cuda")
        check(lib.nufft_interp_noalloc(
            dim, n, eps, 2.0, grid_ptr, M,
            *[None if t is None else t.data_ptr() for t in xs],
            out.data_ptr(), stream))
        torch.cuda.synchronize()
        got = out.cpu().numpy()
        assert np.all(np.isfinite(got))
        assert port.rel_l2(got, ref) <= TOL
        outs.append(got)
    assert np.array_equal(outs[0], outs[1])


def test_interp_noalloc_allocates_nothing_and_edge_points():
    """The second call must leave the device's free memory unchanged (the
    first call may look up the scratch address and load its kernels), and
    points outside [-pi, pi) fold periodically while a non-finite
    coordinate gives a NaN output; finite outputs match the fp64 CPU
    oracle (oracle.port cells_fold + interp) on the same grid."""
    import torch
    from mlx_nufft_b200 import Type2PlanND
    from mlx_nufft_b200._lib import check, lib
    from oracle import port

    rng = np.random.default_rng(77)
    N, M, eps = (40, 36), 5000, 1e-6
    x = [rng.uniform(-3 * np.pi, 3 * np.pi, M) for _ in range(2)]
    x[0][:4] = [3 * np.pi - 1e-9, -3 * np.pi, 2.5 * np.pi, -7.0]
    x[1][5] = np.nan
    x[0][6] = np.inf
    fk = rng.standard_normal(N) + 1j * rng.standard_normal(N)
    ok = np.ones(M, dtype=bool)
    ok[[5, 6]] = False
    plan = Type2PlanND(tuple(v[ok] for v in x), N, eps=eps, isign=-1)
    plan.execute(fk)
    assert plan._plan.info().fft64 == 0      # complex64 grid
    grid_ptr, _ = plan._plan.grid()
    n_up = list(plan.n_up)
    xs = [torch.from_numpy(v).cuda() for v in x]
    n = (ctypes.c_int64 * 3)(*(n_up + [1]))
    stream = torch.cuda.current_stream().cuda_stream
    outs = [torch.zeros(M, dtype=torch.complex64, device="cuda") for _ in range(2)]
    torch.cuda.synchronize()

    def call(out):
        check(lib.nufft_interp_noalloc(2, n, eps, 2.0, grid_ptr, M, xs[0].data_ptr(),
                                       xs[1].data_ptr(), None, out.data_ptr(), stream))
        torch.cuda.synchronize()

    call(outs[0])
    free0, _ = torch.cuda.mem_get_info()
    call(outs[1])
    free1, _ = torch.cuda.mem_get_info()
    assert free1 == free0, (free0, free1)
    got = outs[1].cpu().numpy()
    assert np.array_equal(got[ok], outs[0].cpu().numpy()[ok])
    assert np.all(np.isnan(got[~ok].real)) and np.all(np.isnan(got[~ok].imag))
    assert np.all(np.isfinite(got[ok]))
    # fp64 CPU oracle on the same (downloaded) grid
    from mlx_nufft_b200.parallel import plan_grid_view
    G = plan_grid_view(plan._plan, n_up).reshape(n_up).cpu().numpy().astype(np.complex128)
    w, beta = port.kernel_params(eps, 2.0)
    i1s, frs = [], []
    for d in range(2):
        i1, fr64, _ = port.cells_fold(x[d][ok], n_up[d], w)
        i1s.append(i1)
        frs.append(fr64)
    ref = port.interp(G, i1s, frs, w, beta)
    assert port.rel_l2(got[ok], ref) <= TOL


def test_interp_noalloc_rejects_oversize():
    import torch
    from mlx_nufft_b200._lib import NUFFT_ERR_ARG, last_error, lib

    limit = (16 << 20) // 8
    x = torch.zeros(8, dtype=torch.float64, device="cuda")
    grid = torch.zeros(64, dtype=torch.complex64, device="cuda")
    out = torch.zeros(8, dtype=torch.complex64, device="cuda")
    n = (ctypes.c_int64 * 3)(64, 1, 1)
    # M beyond the scratch: rejected before any launch
    rc = lib.nufft_interp_noalloc(1, n, 1e-6, 2.0, grid.data_ptr(), limit + 1,
                                  x.data_ptr(), None, None, out.data_ptr(), None)
    assert rc == NUFFT_ERR_ARG and "scratch limit" in last_error()
    rc = lib.nufft_interp_noalloc(3, n, 1e-6, 2.0, grid.data_ptr(), limit // 3 + 1,
                                  x.data_ptr(), x.data_ptr(), x.data_ptr(),
                                  out.data_ptr(), None)
    assert rc == NUFFT_ERR_ARG
    # M == 0 is a no-op
    assert lib.nufft_interp_noalloc(1, n, 1e-6, 2.0, grid.data_ptr(), 0,
                                    x.data_ptr(), None, None, out.data_ptr(),
                                    None) == 0
