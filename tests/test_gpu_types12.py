"""GPU parity: type-1 / type-2 transforms (dims 1-3) against the fp64 oracle.

Gates (written as constants below):
  * vs the exact direct sum: rel-L2 <= max(10*eps, 1e-5)  (north-star gate;
    the reference's own API gate against finufft is 4*eps + 2e-4,
    harness/test_api_parity.py:7-10);
  * vs the oracle restatement of the same algorithm in fp64
    (oracle/port.py): rel-L2 <= 2e-5 (the fp32 pipeline's rounding floor;
    the reference measures 1.4e-5 for its fp32 pipeline, mlx-nufft.pdf p.4);
  * setpts cells: i1 bit-exact and fr identical in fp32 to the host fp64
    rule (harness/test_type1_setsources_gpu.py:48-69 gates i1 exact,
    fr <= 1e-6).
"""

import numpy as np
import pytest

from oracle import port, fast

pytestmark = pytest.mark.gpu

FP32_FLOOR = 2e-5


def gate(eps):
    return max(10 * eps, 1e-5)


def pts(rng, dim, M, lo=-np.pi, hi=np.pi):
    return [rng.uniform(lo, hi, M) for _ in range(dim)]


CASES = [(1, (90,)), (1, (87,)), (2, (48, 36)), (2, (45, 34)),
         (3, (24, 20, 16)), (3, (21, 18, 14))]


@pytest.mark.parametrize("dim,N", CASES)
@pytest.mark.parametrize("isign", [+1, -1])
@pytest.mark.parametrize("eps", [1e-3, 1e-5, 1e-6])
@pytest.mark.parametrize("method", ["gm", "od"])
def test_type1_small(dim, N, isign, eps, method, rng):
    from mlx_nufft_b200 import Type1PlanND
    M = 4000
    x = pts(rng, dim, M)
    c = rng.standard_normal(M) + 1j * rng.standard_normal(M)
    plan = Type1PlanND(tuple(x), N, eps=eps, isign=isign, spread_method=method)
    assert plan._od == (method == "od")
    f = plan.execute(c)
    assert f.shape == N and f.dtype == np.complex64
    exact = fast.direct_t1(x, c, N, isign).reshape(N)
    assert port.rel_l2(f, exact) <= gate(eps)
    ref = port.nufft_t1(x, c, N, eps, isign)
    assert port.rel_l2(f, ref) <= FP32_FLOOR


@pytest.mark.parametrize("dim,N", CASES)
@pytest.mark.parametrize("isign", [+1, -1])
@pytest.mark.parametrize("eps", [1e-3, 1e-5, 1e-6])
@pytest.mark.parametrize("method", ["gm", "od"])
def test_type2_small(dim, N, isign, eps, method, rng):
    from mlx_nufft_b200 import Type2PlanND
    M = 4000
    x = pts(rng, dim, M)
    fk = rng.standard_normal(N) + 1j * rng.standard_normal(N)
    plan = Type2PlanND(tuple(x), N, eps=eps, isign=isign, spread_method=method)
    c = plan.execute(fk)
    assert c.shape == (M,) and c.dtype == np.complex64
    exact = fast.direct_t2(x, fk, isign)
    assert port.rel_l2(c, exact) <= gate(eps)
    ref = port.nufft_t2(x, fk, eps, isign)
    assert port.rel_l2(c, ref) <= FP32_FLOOR


@pytest.mark.parametrize("dim,N,M", [(1, (4096,), 300_000),
                                     (2, (128, 100), 300_000),
                                     (3, (64, 48, 40), 300_000)])
def test_tiled_auto_large(dim, N, M, rng):
    """P >= 2e4 takes the tiled (bin-sorted) path automatically; check a
    random subset of outputs against the exact sum."""
    from mlx_nufft_b200 import Type1PlanND, Type2PlanND
    x = pts(rng, dim, M)
    c = rng.standard_normal(M) + 1j * rng.standard_normal(M)
    p1 = Type1PlanND(tuple(x), N, eps=1e-6, isign=+1)
    assert p1._od
    f = p1.execute(c).ravel()
    idx = rng.choice(f.size, 200, replace=False)
    assert port.rel_l2(f[idx], fast.direct_t1(x, c, N, +1, idx)) <= gate(1e-6)
    fk = rng.standard_normal(N) + 1j * rng.standard_normal(N)
    p2 = Type2PlanND(tuple(x), N, eps=1e-6, isign=-1)
    assert p2._od
    cj = p2.execute(fk)
    idx = rng.choice(M, 200, replace=False)
    assert port.rel_l2(cj[idx], fast.direct_t2(x, fk, -1, idx)) <= gate(1e-6)


def test_2d_low_density_spread_global(rng):
    """A 2-D type-1 plan below 2 points per fine cell (the quickstart's
    1e5 points on 512^2 cells) spreads with the global kernel; its type-2
    sibling keeps the tiled interpolation."""
    from mlx_nufft_b200 import Type1PlanND, Type2PlanND
    M, N = 100_000, (256, 256)
    x = pts(rng, 2, M)
    c = rng.standard_normal(M) + 1j * rng.standard_normal(M)
    p1 = Type1PlanND(tuple(x), N, eps=1e-6, isign=+1)
    assert not p1._od
    f = p1.execute(c).ravel()
    idx = rng.choice(f.size, 200, replace=False)
    assert port.rel_l2(f[idx], fast.direct_t1(x, c, N, +1, idx)) <= gate(1e-6)
    assert Type2PlanND(tuple(x), N, eps=1e-6)._od


@pytest.mark.parametrize("dim,N", [(1, (4096,)), (2, (512, 384)),
                                   (3, (64, 64, 48))])
@pytest.mark.parametrize("prec", ["crit64", "fp32"])
def test_setpts_cells_exact(dim, N, prec, rng):
    """Device fold/rescale == host rule, bit for bit, including |x| up to
    1000*2pi; perm is a bijection and points are grouped by bin."""
    from mlx_nufft_b200 import Type1PlanND
    P = 60_000
    x = [np.concatenate([rng.uniform(-np.pi, np.pi, P // 2),
                         rng.uniform(-2000 * np.pi, 2000 * np.pi, P - P // 2)])
         for _ in range(dim)]
    plan = Type1PlanND(tuple(x), N, eps=1e-5, prec=prec)
    i1, fr, perm = plan.cells()
    assert np.array_equal(np.sort(perm), np.arange(P))
    key = np.zeros(P, dtype=np.int64)
    info = plan._plan.info()
    for d in range(dim):
        ri1, _, rfr = port.cells_fold(x[d][perm], plan.n_up[d], plan.w, prec)
        np.testing.assert_array_equal(
            i1[d], port.normalize_cells(ri1, plan.n_up[d], plan.w))
        np.testing.assert_array_equal(fr[d], rfr)
        b = (i1[d].astype(np.int64) + plan.w // 2) // info.bin[d]
        nb = -(-plan.n_up[d] // info.bin[d])
        key = key * nb + b
    assert np.all(np.diff(key) >= 0)


def test_quickstart_known_answer(golden):
    """examples/quickstart.py:52-73: 1D type 1, rel-L2 < 10*eps vs exact DFT."""
    import mlx_nufft_b200 as finufft
    g = golden("quickstart")
    fk = finufft.nufft1d1(g["x"], g["c"], int(g["N"]), eps=float(g["eps"]),
                          isign=+1)
    assert port.rel_l2(fk, g["f_exact"]) < 10 * float(g["eps"])


@pytest.mark.parametrize("dim", [1, 2, 3])
def test_direct_golden(golden, dim):
    """Golden exact sums from the reference's direct_sum."""
    from mlx_nufft_b200 import Type1PlanND, Type2PlanND
    g = golden("direct")
    t = f"t1_{dim}d_"
    N = tuple(int(n) for n in g[t + "N"])
    f = Type1PlanND(tuple(g[t + "x"]), N, eps=1e-6,
                    isign=int(g[t + "isign"])).execute(g[t + "c"])
    assert port.rel_l2(f, g[t + "f"]) <= gate(1e-6)
    t = f"t2_{dim}d_"
    c = Type2PlanND(tuple(g[t + "x"]), N, eps=1e-6,
                    isign=int(g[t + "isign"])).execute(g[t + "f"])
    assert port.rel_l2(c, g[t + "c"]) <= gate(1e-6)


def test_clustered_points_wrap(rng):
    """Points clustered at the periodic corner (the cfg-4 hot spot) and the
    cuFINUFFT 'cluster' distribution: many subproblems per bin."""
    from mlx_nufft_b200 import Type1PlanND, Type2PlanND
    from mlx_nufft_b200.gen import uniform_points
    x, N, M = uniform_points(3, 24, rho=8.0, dist="cluster", seed=9)
    x = [np.mod(v + np.pi, 2 * np.pi) - np.pi for v in x]
    c = rng.standard_normal(M) + 1j * rng.standard_normal(M)
    p1 = Type1PlanND(tuple(x), N, eps=1e-6)
    f = p1.execute(c).ravel()
    idx = rng.choice(f.size, 300, replace=False)
    assert port.rel_l2(f[idx], fast.direct_t1(x, c, N, +1, idx)) <= gate(1e-6)
    xg = [np.mod(rng.normal(0, 0.3, 200_000) + np.pi, 2 * np.pi) - np.pi
          for _ in range(3)]
    fk = rng.standard_normal((32, 32, 32)) + 1j * rng.standard_normal((32, 32, 32))
    cj = Type2PlanND(tuple(xg), (32, 32, 32), eps=1e-6).execute(fk)
    idx = rng.choice(200_000, 200, replace=False)
    assert port.rel_l2(cj[idx], fast.direct_t2(xg, fk, -1, idx)) <= gate(1e-6)


def test_upsampfac_125_and_odd_sizes(rng):
    from mlx_nufft_b200 import Type1PlanND, Type2PlanND
    x = pts(rng, 2, 30_000)
    c = rng.standard_normal(30_000) + 1j * rng.standard_normal(30_000)
    N = (33, 17)
    for sig in (1.25, 1.5, 3.0):
        f = Type1PlanND(tuple(x), N, eps=1e-5, upsampfac=sig).execute(c)
        assert port.rel_l2(f, fast.direct_t1(x, c, N, +1).reshape(N)) <= gate(1e-5)
    fk = rng.standard_normal(N) + 1j * rng.standard_normal(N)
    cj = Type2PlanND(tuple(x), N, eps=1e-5, upsampfac=1.25).execute(fk)
    idx = np.arange(0, 30_000, 97)
    assert port.rel_l2(cj[idx], fast.direct_t2(x, fk, -1, idx)) <= gate(1e-5)


@pytest.mark.parametrize("N", [(64, 48, 40), (48, 64, 36)])
def test_type2_3d_batch_tma_staged_tiles(N, rng):
    """3-D type 2 over several vectors on cuFFT-sized grids (no periodic
    halo: TMA-staged tiles, one tensor-map coordinate per vector, and the
    bins at the periodic edge loaded by hand): the batch equals per-vector
    executes bit for bit (interpolation is deterministic) and the direct
    sum within the gate; points cluster at the grid corner so both tile
    paths carry dense bins."""
    from mlx_nufft_b200 import Type2PlanND
    P = 120_000
    x = [np.concatenate([rng.uniform(-np.pi, np.pi, P // 2),
                         np.mod(rng.normal(0, 0.3, P // 2) + np.pi, 2 * np.pi) - np.pi])
         for _ in range(3)]
    B = 3
    fks = (rng.standard_normal((B,) + N) + 1j * rng.standard_normal((B,) + N)
           ).astype(np.complex64)
    plan = Type2PlanND(tuple(x), N, eps=1e-6)
    assert plan._plan.info().tiled
    got = plan.execute_batch(fks)
    idx = rng.choice(P, 300, replace=False)
    for b in range(B):
        one = plan.execute(fks[b])
        np.testing.assert_array_equal(got[b], one)
        exact = fast.direct_t2([v[idx] for v in x], fks[b], -1)
        assert port.rel_l2(got[b][idx], exact) <= 1e-5


@pytest.mark.parametrize("isign", [-1, +1])
def test_type2_3d_dense_point_pairs(isign, rng):
    """Dense 3-D interpolation subproblems (thousands of points per 10^3
    bin, many points per cell, split into several subproblems of one bin),
    with a sparse fringe.  Every output against the fp64 restatement of the
    pipeline, and a sample against the exact sum."""
    from mlx_nufft_b200 import Type2PlanND
    N, M = (24, 20, 28), 300_001
    x = [np.mod(rng.normal(0, 0.25, M) + np.pi, 2 * np.pi) - np.pi for _ in range(3)]
    x[0][:1000] = rng.uniform(-np.pi, np.pi, 1000)       # a sparse fringe too
    fk = rng.standard_normal(N) + 1j * rng.standard_normal(N)
    plan = Type2PlanND(tuple(x), N, eps=1e-6, isign=isign)
    assert plan._plan.info().tiled
    c = plan.execute(fk)
    assert port.rel_l2(c, port.nufft_t2(x, fk, 1e-6, isign)) <= 2e-5
    idx = rng.choice(M, 200, replace=False)
    assert port.rel_l2(c[idx], fast.direct_t2(x, fk, isign, idx)) <= gate(1e-6)
    # deterministic: a second execute is bit-identical
    np.testing.assert_array_equal(plan.execute(fk), c)


@pytest.mark.parametrize("N,eps,isign", [((32, 32, 32), 1e-6, -1),
                                         ((32, 64, 32), 1e-6, +1),
                                         ((32, 32, 64), 1e-9, -1)])
def test_type2_3d_halo_grid(N, eps, isign, rng):
    """3-D type 2 on power-of-two fine grids: the pruned FFT writes the grid
    with a periodic halo (the stage API reports more cells than the grid
    has) and every tile is copied by TMA, none wraps.  Points half uniform,
    half clustered at the periodic corner (where the halo copies are read),
    two vectors: all outputs against the fp64 restatement of the pipeline,
    a sample against the exact sum, batch equal to single executes."""
    from mlx_nufft_b200 import Type2PlanND
    P = 150_000
    x = [np.concatenate([rng.uniform(-np.pi, np.pi, P // 2),
                         np.mod(rng.normal(0, 0.3, P // 2) + np.pi, 2 * np.pi) - np.pi])
         for _ in range(3)]
    fks = (rng.standard_normal((2,) + N) + 1j * rng.standard_normal((2,) + N)
           ).astype(np.complex64)
    plan = Type2PlanND(tuple(x), N, eps=eps, isign=isign)
    info = plan._plan.info()
    assert info.tiled
    nup = int(np.prod([int(info.n_up[d]) for d in range(3)]))
    assert info.grid_cells > nup                       # halo in effect
    _, ncomplex = plan._plan.grid()
    assert ncomplex % info.grid_cells == 0
    got = plan.execute_batch(fks)
    idx = rng.choice(P, 200, replace=False)
    for b in range(2):
        np.testing.assert_array_equal(got[b], plan.execute(fks[b]))
        assert port.rel_l2(got[b], port.nufft_t2(x, fks[b], eps, isign)) <= max(20 * eps, 2e-5)
        exact = fast.direct_t2([v[idx] for v in x], fks[b], isign)
        assert port.rel_l2(got[b][idx], exact) <= gate(eps)


@pytest.mark.parametrize("lo,hi", [(-0.4, 0.5), (1.0, 1.6)])
def test_type2_3d_slab_points_pruned_planes(lo, hi, rng):
    """A 3-D type-2 plan whose points fill one slab of the first coordinate
    (as each rank's share in the x-slab split of bench.py): setpts marks the
    grid planes its tiles read, and the execute computes only those (the
    slab order of the pruned FFT: X pass first, then Y and Z over the marked
    planes, plus their halo copies).  The first slab straddles the periodic
    seam at 0 (tiles at both ends of the grid).  The execute matches the
    staged execute (whose grid is the whole plain-order FFT) to FFT
    rounding, and the fp64 restatement of the pipeline within the gate."""
    import torch
    from mlx_nufft_b200 import Type2PlanND, _lib
    N, P = (32, 32, 32), 100_000
    x = [rng.uniform(lo, hi, P), rng.uniform(-np.pi, np.pi, P),
         rng.uniform(-np.pi, np.pi, P)]
    fk = (rng.standard_normal(N) + 1j * rng.standard_normal(N)).astype(np.complex64)
    plan = Type2PlanND(tuple(x), N, eps=1e-6)
    info = plan._plan.info()
    assert info.tiled and info.grid_cells > np.prod([int(info.n_up[d]) for d in range(3)])
    got = plan.execute(fk)
    ft = torch.from_numpy(fk).cuda()
    out = torch.empty(P, dtype=torch.complex64, device="cuda")
    plan._plan.execute_stage(_lib.STAGE_SPREAD, ft, None, 1)
    plan._plan.execute_stage(_lib.STAGE_FINISH, None, out, 1)
    torch.cuda.synchronize()
    assert port.rel_l2(got, out.cpu().numpy()) <= 2e-6
    assert port.rel_l2(got, port.nufft_t2(x, fk, 1e-6, -1)) <= 2e-5
    # and again with two vectors (one launch over both)
    fks = np.stack([fk, (fk * (0.5 - 1j)).astype(np.complex64)])
    gb = plan.execute_batch(fks)
    assert port.rel_l2(gb[0], got) <= 1e-6
    assert port.rel_l2(gb[1], port.nufft_t2(x, fks[1], 1e-6, -1)) <= 2e-5
