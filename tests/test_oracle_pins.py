"""Pin the CPU oracle (oracle/) against golden vectors produced by the
reference's own CPU code (tests/golden/make_golden.py): sizing
(mlx_nufft/sizing.py), the type-3 CPU plan (mlx_nufft/ref_t3.py, FULL64),
the exact direct sum and the generators (harness/gen.py), and the
known-answer check of examples/quickstart.py:52-73."""

import numpy as np
import pytest

from oracle import port, fast
from mlx_nufft_b200 import gen


def test_sizing_kernel_params(golden):
    g = golden("sizing")
    for i, e in enumerate(g["eps"]):
        for j, s in enumerate(g["sigma"]):
            w, b = port.kernel_params(float(e), float(s))
            assert w == g["w"][i, j]
            assert b == g["beta"][i, j]


def test_sizing_next235even(golden):
    g = golden("sizing")
    got = np.array([port.next235even(int(n)) for n in g["n235_in"]])
    np.testing.assert_array_equal(got, g["n235"])


def test_sizing_kernel_ft(golden):
    g = golden("sizing")
    for (w, b), ref in zip(g["kft_wb"], g["kft_val"]):
        got = port.kernel_ft(g["kft_xi"], b, int(w))
        np.testing.assert_allclose(got, ref, rtol=1e-13, atol=0)


def test_sizing_set_nhg_type3(golden):
    g = golden("sizing")
    for (S, X, s, w), ref in zip(g["nhg_in"], g["nhg_out"]):
        nf, h, gam = port.set_nhg_type3(S, X, s, int(w))
        assert nf == ref[0] and h == ref[1] and gam == ref[2]


def test_generators_match_reference(golden):
    g = golden("gen")
    x, _, M = gen.uniform_points(2, 16, rho=1.0, dist="rand", seed=3)
    np.testing.assert_array_equal(np.stack(x), g["rand_x"])
    assert M == g["rand_M"]
    xc, _, Mc = gen.uniform_points(3, 8, rho=0.5, dist="cluster", seed=4)
    np.testing.assert_array_equal(np.stack(xc), g["cl_x"])
    p = gen.gen_generic(N=6, P=50, seed=1, X=3.0, S=2.0)
    np.testing.assert_array_equal(np.stack(p["x"]), g["gen_x"])
    np.testing.assert_array_equal(np.stack(p["s"]), g["gen_s"])
    np.testing.assert_array_equal(p["c"], g["gen_c"])
    a = gen.gen_anisotropic(N=6, P=40, lat=1.5, seed=0)
    np.testing.assert_array_equal(np.stack(a["x"]), g["an_x"])
    np.testing.assert_array_equal(np.stack(a["s"]), g["an_s"])
    np.testing.assert_array_equal(a["c"], g["an_c"])


@pytest.mark.parametrize("dim", [1, 2, 3])
def test_direct_sum_matches_reference(golden, dim):
    g = golden("direct")
    t = f"t1_{dim}d_"
    x = list(g[t + "x"])
    N = tuple(g[t + "N"])
    f = port.direct_t1(x, g[t + "c"], N, int(g[t + "isign"]))
    np.testing.assert_allclose(f, g[t + "f"].ravel(), rtol=0, atol=1e-10)
    f2 = fast.direct_t1(x, g[t + "c"], N, int(g[t + "isign"]))
    np.testing.assert_allclose(f2, g[t + "f"].ravel(), rtol=0, atol=1e-10)
    t = f"t2_{dim}d_"
    c = port.direct_t2(list(g[t + "x"]), g[t + "f"], int(g[t + "isign"]))
    np.testing.assert_allclose(c, g[t + "c"], rtol=0, atol=1e-10)
    c2 = fast.direct_t2(list(g[t + "x"]), g[t + "f"], int(g[t + "isign"]))
    np.testing.assert_allclose(c2, g[t + "c"], rtol=0, atol=1e-10)


@pytest.mark.parametrize("case", [0, 1, 2])
def test_type3_geometry_matches_ref_t3(golden, case):
    g = golden("t3_ref")
    p = f"c{case}_"
    geo = port.T3Geometry(list(g[p + "x"]), list(g[p + "s"]),
                          eps=float(g[p + "eps"]), isign=int(g[p + "isign"]))
    assert geo.nf == list(g[p + "nf"]) and geo.n_up == list(g[p + "n_up"])
    assert geo.w == g[p + "w"] and geo.beta == g[p + "beta"]
    np.testing.assert_array_equal(geo.C, g[p + "C"])
    np.testing.assert_array_equal(geo.D, g[p + "D"])
    np.testing.assert_array_equal(geo.gam, g[p + "gam"])
    np.testing.assert_array_equal(np.stack(geo.i1), g[p + "i1"])
    np.testing.assert_array_equal(np.stack(geo.fr), g[p + "fr"])
    np.testing.assert_array_equal(np.stack(geo.t_i1), g[p + "t_i1"])
    np.testing.assert_array_equal(np.stack(geo.t_fr), g[p + "t_fr"])
    np.testing.assert_allclose(geo.prephase, g[p + "prephase"], rtol=0, atol=1e-15)
    np.testing.assert_allclose(geo.post, g[p + "post"], rtol=1e-13)
    for d in range(3):
        np.testing.assert_allclose(geo.mode_dec[d], g[p + f"mode_dec{d}"],
                                   rtol=1e-13)


@pytest.mark.parametrize("case", [0, 1, 2])
def test_type3_output_matches_ref_t3(golden, case):
    g = golden("t3_ref")
    p = f"c{case}_"
    f = port.nufft_t3(list(g[p + "x"]), g[p + "c"], list(g[p + "s"]),
                      eps=float(g[p + "eps"]), isign=int(g[p + "isign"]))
    # same fp64 algorithm: agreement to summation-order rounding
    assert port.rel_l2(f, g[p + "out"]) < 1e-12
    # and both are within the method's truncation error of the exact sum
    assert port.rel_l2(f, g[p + "direct"]) < 10 * float(g[p + "eps"])


def test_quickstart_known_answer(golden):
    g = golden("quickstart")
    f = port.nufft_t1([g["x"]], g["c"], (int(g["N"]),), float(g["eps"]), +1)
    assert port.rel_l2(f, g["f_exact"]) < 10 * float(g["eps"])


@pytest.mark.parametrize("dim,N", [(1, (37,)), (2, (16, 11)), (3, (8, 7, 6))])
@pytest.mark.parametrize("isign", [+1, -1])
def test_oracle_types12_vs_direct(dim, N, isign, rng):
    M = 700
    x = [rng.uniform(-np.pi, np.pi, M) for _ in range(dim)]
    c = rng.standard_normal(M) + 1j * rng.standard_normal(M)
    f = port.nufft_t1(x, c, N, 1e-6, isign)
    assert port.rel_l2(f, port.direct_t1(x, c, N, isign)) < 1e-5
    fk = rng.standard_normal(N) + 1j * rng.standard_normal(N)
    cj = port.nufft_t2(x, fk, 1e-6, isign)
    assert port.rel_l2(cj, port.direct_t2(x, fk, isign)) < 1e-5


def test_oracle_cells_fold_matches_formula():
    x = np.array([-np.pi, -1.0, 0.0, 1e-300, 3.0, np.pi, 100.0, -1e4])
    i1, fr64, fr32 = port.cells_fold(x, 64, 7)
    xi = np.mod(x, 2 * np.pi) / (2 * np.pi / 64)
    np.testing.assert_array_equal(i1, np.ceil(xi - 3.5).astype(np.int32))
    assert np.all(fr64 > 2.5 - 1e-12) and np.all(fr64 <= 3.5)


@pytest.mark.parametrize("case", [0, 1, 2])
def test_type3_fp32_pipeline_matches_ref_t3(golden, case):
    """oracle.port.nufft_t3_fp32 reproduces the reference's fp32 type-3
    pipeline (RefT3Plan with crit64 geometry, fp32 stages) bit for bit."""
    g = golden("t3_ref")
    p = f"c{case}_"
    f = port.nufft_t3_fp32(list(g[p + "x"]), g[p + "c"], list(g[p + "s"]),
                           eps=float(g[p + "eps"]), isign=int(g[p + "isign"]))
    np.testing.assert_array_equal(f, g[p + "out32"])
