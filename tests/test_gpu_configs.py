"""The five benchmark workloads on the GPU: every config at its full size,
checked against the exact fp64 direct sum on a random output subset (the
reference's subset-oracle protocol, harness/run_acceptance.py:86-97), plus
size-independent properties at full size (linearity, repeatability)."""

import numpy as np
import pytest

from oracle import fast, port
from mlx_nufft_b200 import gen

pytestmark = pytest.mark.gpu

NSUB = 64


def gate(eps):
    return max(10 * eps, 1e-5)


def test_cfg1_2d_type1_full():
    import mlx_nufft_b200 as finufft
    cfg = gen.config(1)
    f = finufft.nufft2d1(*cfg["x"], cfg["data"], cfg["n_modes"], eps=1e-6)
    rng = np.random.default_rng(1)
    idx = rng.choice(f.size, 400, replace=False)
    ref = fast.direct_t1(cfg["x"], cfg["data"], cfg["n_modes"], +1, idx)
    assert port.rel_l2(f.ravel()[idx], ref) <= gate(1e-6)


def test_cfg2_1d_type2_full():
    from mlx_nufft_b200 import Type2PlanND
    cfg = gen.config(2)
    plan = Type2PlanND(tuple(cfg["x"]), cfg["n_modes"], eps=1e-6, isign=-1)
    c = plan.execute(cfg["data"])
    rng = np.random.default_rng(2)
    idx = rng.choice(c.size, NSUB, replace=False)
    ref = fast.direct_t2(cfg["x"], cfg["data"], -1, idx)
    assert port.rel_l2(c[idx], ref) <= gate(1e-6)
    # repeat execute on the same plan: identical (no atomics on this path)
    assert np.array_equal(plan.execute(cfg["data"]), c)
    # linearity at full size
    f2 = cfg["data"] * (0.5 - 1.5j)
    c2 = plan.execute(f2)
    assert port.rel_l2(c2, c * (0.5 - 1.5j)) < 1e-6


def test_cfg2_every_output_vs_fp64_restatement():
    """All 1e7 outputs of the 1-D type-2 workload against the fp64 CPU
    restatement of the reference pipeline (oracle/port.py: deconvolve, pad,
    FFT, fold, interp in fp64) -- rel-L2 2e-5, the fp32 pipeline floor --
    and the largest pointwise error against the output scale."""
    from mlx_nufft_b200 import Type2PlanND
    cfg = gen.config(2)
    plan = Type2PlanND(tuple(cfg["x"]), cfg["n_modes"], eps=1e-6, isign=-1)
    c = plan.execute(cfg["data"])
    ref = port.nufft_t2(cfg["x"], cfg["data"], 1e-6, -1)
    assert c.shape == ref.shape == (10_000_000,)
    assert port.rel_l2(c, ref) <= 2e-5
    assert np.max(np.abs(c - ref)) <= 2e-4 * np.sqrt(np.mean(np.abs(ref) ** 2))


def _port_grid_t2(f, N, eps, isign):
    """The fp64 fine grid of the CPU restatement (deconvolve + pad + FFT),
    FFT on all host threads."""
    import os
    import scipy.fft as sf
    w, beta, nup = port.fine_grid_sizes(N, eps)
    g = np.asarray(f, dtype=np.complex128)
    for d in range(len(N)):
        k = np.arange(-(N[d] // 2), N[d] - N[d] // 2, dtype=np.float64)
        dec = 1.0 / port.kernel_ft(2.0 * np.pi * k / nup[d], beta, w)
        g = g * dec.reshape((1,) * d + (-1,) + (1,) * (len(N) - d - 1))
    H = np.zeros(nup, dtype=np.complex128)
    H[np.ix_(*[port._band(N[d], nup[d]) for d in range(len(N))])] = g
    workers = os.cpu_count() or 1
    V = (sf.ifftn(H, workers=workers) * H.size if isign > 0
         else sf.fftn(H, workers=workers))
    return V, w, beta, nup


def test_cfg4_subset_vs_fp64_restatement():
    """2e5 outputs of the clustered 3-D type-2 workload (half from the
    uniform half, half from the cluster) against the fp64 CPU restatement
    interpolating the same points from its own fp64 grid."""
    from mlx_nufft_b200 import Type2PlanND
    cfg = gen.config(4)
    plan = Type2PlanND(tuple(cfg["x"]), cfg["n_modes"], eps=1e-6, isign=-1)
    c = plan.execute(cfg["data"])
    del plan
    V, w, beta, nup = _port_grid_t2(cfg["data"], cfg["n_modes"], 1e-6, -1)
    rng = np.random.default_rng(44)
    M = c.size
    idx = np.concatenate([rng.choice(M // 2, 100_000, replace=False),
                          M // 2 + rng.choice(M - M // 2, 100_000, replace=False)])
    i1s, frs = [], []
    for d in range(3):
        i1, fr64, _ = port.cells_fold(cfg["x"][d][idx], nup[d], w)
        i1s.append(i1)
        frs.append(fr64)
    ref = port.interp(V, i1s, frs, w, beta, chunk=8192)
    assert port.rel_l2(c[idx], ref) <= 2e-5
    assert port.rel_l2(c[idx[:100_000]], ref[:100_000]) <= 2e-5   # uniform half
    assert port.rel_l2(c[idx[100_000:]], ref[100_000:]) <= 2e-5   # cluster


def test_cfg3_3d_type1_batch_full():
    from mlx_nufft_b200 import Type1PlanND
    cfg = gen.config(3)
    plan = Type1PlanND(tuple(cfg["x"]), cfg["n_modes"], eps=1e-5, isign=+1)
    fb = plan.execute_batch(cfg["data"])
    assert fb.shape == (8, 128, 128, 128)
    rng = np.random.default_rng(3)
    idx = rng.choice(128 ** 3, 24, replace=False)
    for b in (0, 7):
        ref = fast.direct_t1(cfg["x"], cfg["data"][b], cfg["n_modes"], +1, idx)
        assert port.rel_l2(fb[b].ravel()[idx], ref) <= gate(1e-5)
    # linearity across the batch: f(c0 + c1) = f(c0) + f(c1)
    s = plan.execute(cfg["data"][0] + cfg["data"][1])
    assert port.rel_l2(s, fb[0] + fb[1]) < 2e-5


def test_cfg4_3d_type2_clustered_full():
    from mlx_nufft_b200 import Type2PlanND
    cfg = gen.config(4)
    plan = Type2PlanND(tuple(cfg["x"]), cfg["n_modes"], eps=1e-6, isign=-1)
    c = plan.execute(cfg["data"])
    rng = np.random.default_rng(4)
    # half the subset from the uniform half, half from the cluster
    M = c.size
    idx = np.concatenate([rng.choice(M // 2, NSUB // 2, replace=False),
                          M // 2 + rng.choice(M - M // 2, NSUB // 2,
                                              replace=False)])
    ref = fast.direct_t2(cfg["x"], cfg["data"], -1, idx)
    assert port.rel_l2(c[idx], ref) <= gate(1e-6)


def test_cfg5_3d_type3_and_expi_full():
    from mlx_nufft_b200 import Type3Plan, expi
    cfg = gen.config(5)
    plan = Type3Plan(tuple(cfg["x"]), tuple(cfg["s"]), eps=1e-5, isign=+1)
    assert plan.nf == [180] * 3 and plan.n_up == [240] * 3 and plan.w == 9
    f = plan.execute(cfg["data"])
    rng = np.random.default_rng(5)
    idx = rng.choice(f.size, NSUB, replace=False)
    ref = fast.direct_sum(cfg["x"], cfg["data"], cfg["s"], +1, idx)
    assert port.rel_l2(f[idx], ref) <= gate(1e-5)
    e = gen.config(6)
    out = expi(e["phi"], return_np=True)
    assert np.max(np.abs(out - port.expi_ref(e["phi"]))) <= 5e-7
