"""GPU parity: the two-pass 1-D FFT with the pad / crop fused into its passes
(csrc/fft1.cu), used for complex64 1-D fine grids of 2^12..2^22 cells.

Every supported pass-length pair (N1, N2) = (64, 64) .. (1024, 2048) runs
through type 2 (pad fused into pass 1) and type 1 (crop fused into pass 2),
both signs, against the fp64 oracle restatement of the same algorithm
(oracle/port.py; rel-L2 <= 2e-5, the fp32 pipeline floor) and, on sampled
outputs, against the exact direct sum (rel-L2 <= max(10 eps, 1e-5)).
Batches and execute_disjoint go through the same passes.
"""

import numpy as np
import pytest

from oracle import port

pytestmark = pytest.mark.gpu

FP32_FLOOR = 2e-5


def gate(eps):
    return max(10 * eps, 1e-5)


# n_up = 2 N: 2^12 .. 2^22 cells
SIZES = [2 ** k for k in range(11, 22)]


@pytest.mark.parametrize("N", SIZES)
@pytest.mark.parametrize("isign", [-1, +1])
def test_type2_fft1_sizes(N, isign, rng):
    from mlx_nufft_b200 import Type2PlanND
    eps = 1e-6
    M = 20_000
    x = [rng.uniform(-np.pi, np.pi, M)]
    f = rng.standard_normal(N) + 1j * rng.standard_normal(N)
    plan = Type2PlanND(tuple(x), (N,), eps=eps, isign=isign)
    assert plan._plan.info().fft_own == 1
    c = plan.execute(f)
    ref = port.nufft_t2(x, f, eps, isign)
    assert port.rel_l2(c, ref) <= FP32_FLOOR
    idx = rng.choice(M, 48, replace=False)
    assert port.rel_l2(c[idx], port.direct_t2(x, f, isign, idx)) <= gate(eps)


@pytest.mark.parametrize("N", SIZES)
@pytest.mark.parametrize("isign", [+1, -1])
def test_type1_fft1_sizes(N, isign, rng):
    from mlx_nufft_b200 import Type1PlanND
    eps = 1e-6
    M = 20_000
    x = [rng.uniform(-np.pi, np.pi, M)]
    c = rng.standard_normal(M) + 1j * rng.standard_normal(M)
    plan = Type1PlanND(tuple(x), (N,), eps=eps, isign=isign)
    assert plan._plan.info().fft_own == 1
    f = plan.execute(c)
    ref = port.nufft_t1(x, c, (N,), eps, isign)
    assert port.rel_l2(f, ref) <= FP32_FLOOR
    kidx = rng.choice(N, 48, replace=False)
    assert port.rel_l2(f[kidx], port.direct_t1(x, c, (N,), isign, kidx)) <= gate(eps)


def test_fft1_odd_modes_and_cufft_sizes(rng):
    """An odd mode count in a power-of-two grid uses the fused passes; a
    2,3,5-smooth grid that is not a power of two keeps cuFFT."""
    from mlx_nufft_b200 import Type2PlanND
    M = 30_000
    x = [rng.uniform(-np.pi, np.pi, M)]
    for N, own in ((4095, 1), (3000, 0)):
        f = rng.standard_normal(N) + 1j * rng.standard_normal(N)
        plan = Type2PlanND(tuple(x), (N,), eps=1e-6)
        assert plan._plan.info().fft_own == own
        assert port.rel_l2(plan.execute(f), port.nufft_t2(x, f, 1e-6, -1)) <= FP32_FLOOR


def test_fft1_batch_and_disjoint(rng):
    from mlx_nufft_b200 import Plan, Type1PlanND
    N, M, nv = 1 << 14, 50_000, 3
    x = rng.uniform(-np.pi, np.pi, M)
    # batched type 2 (vectors through both passes at once)
    fs = rng.standard_normal((nv, N)) + 1j * rng.standard_normal((nv, N))
    p2 = Plan(2, (N,), n_trans=nv, eps=1e-6, isign=-1)
    p2.setpts(x)
    cs = p2.execute(fs)
    for v in range(nv):
        assert port.rel_l2(cs[v], port.nufft_t2([x], fs[v], 1e-6, -1)) <= FP32_FLOOR
    # batched type 1
    cj = rng.standard_normal((nv, M)) + 1j * rng.standard_normal((nv, M))
    p1 = Plan(1, (N,), n_trans=nv, eps=1e-6, isign=+1)
    p1.setpts(x)
    fk = p1.execute(cj)
    for v in range(nv):
        assert port.rel_l2(fk[v], port.nufft_t1([x], cj[v], (N,), 1e-6, +1)) <= FP32_FLOOR
    # execute_disjoint: groups of points, one type-1 transform each
    groups = rng.integers(0, 4, M).astype(np.int32)
    c = rng.standard_normal(M) + 1j * rng.standard_normal(M)
    plan = Type1PlanND((x,), (N,), eps=1e-6)
    out = plan.execute_disjoint(c, groups)
    for g in range(4):
        sel = groups == g
        ref = port.nufft_t1([x[sel]], c[sel], (N,), 1e-6, +1)
        assert port.rel_l2(out[g], ref) <= FP32_FLOOR


def test_type3_1d_fused_pad(rng):
    """1-D type 3 with sigma_inner = 2: sources spread onto nf = 2048 cells,
    padded to a 4096-cell grid by the first FFT pass (the pad reads the
    spread grid with the type-3 (-1)^q corrections).  At the default
    sigma_inner = 1.25 no type-3 grid is a power of two."""
    from oracle import fast
    from mlx_nufft_b200 import Type3Plan
    P, M, X, S = 30_000, 40_000, 8.0, 317.3
    x = rng.uniform(-X, X, P)
    s = rng.uniform(-S, S, M)
    x[:2] = (-X, X)                       # pin the extents
    s[:2] = (-S, S)
    c = rng.standard_normal(P) + 1j * rng.standard_normal(P)
    plan = Type3Plan((x,), (s,), eps=1e-5, sigma_inner=2.0)
    info = plan._plan.info()
    assert info.fft_own == 1 and info.nf[0] == 2048 and info.n_up[0] == 4096
    f = plan.execute(c)
    idx = rng.choice(M, 400, replace=False)
    exact = fast.direct_sum([x], c, [s], +1, idx)
    assert port.rel_l2(f[idx], exact) <= gate(1e-5)
