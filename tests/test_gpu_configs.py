"""The five BASELINE workloads on the GPU: every config at its full size,
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
