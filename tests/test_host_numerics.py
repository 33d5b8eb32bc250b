"""Host-side numerics of libnufft_b200 (csrc/sizing.cpp, through the C ABI)
against the reference's golden values.  No GPU needed."""

import numpy as np

from mlx_nufft_b200 import sizing


def test_kernel_params_exact(golden):
    g = golden("sizing")
    for i, e in enumerate(g["eps"]):
        for j, s in enumerate(g["sigma"]):
            w, b = sizing.kernel_params(float(e), float(s))
            assert w == g["w"][i, j]
            assert b == g["beta"][i, j]


def test_next235even_exact(golden):
    g = golden("sizing")
    got = np.array([sizing.next235even(int(n)) for n in g["n235_in"]])
    np.testing.assert_array_equal(got, g["n235"])


def test_kernel_ft(golden):
    g = golden("sizing")
    for (w, b), ref in zip(g["kft_wb"], g["kft_val"]):
        got = sizing.kernel_ft(g["kft_xi"], b, int(w))
        # own Gauss-Legendre nodes (Newton) vs numpy's: fp64 rounding only
        # (absolute, relative to phihat(0) ~ 2)
        np.testing.assert_allclose(got, ref, rtol=1e-12, atol=1e-13)


def test_set_nhg_type3_exact(golden):
    g = golden("sizing")
    for (S, X, s, w), ref in zip(g["nhg_in"], g["nhg_out"]):
        nf, h, gam = sizing.set_nhg_type3(S, X, s, int(w))
        assert nf == ref[0] and h == ref[1] and gam == ref[2]


def test_es_kernel_support():
    v = sizing.es_kernel(np.array([-4.0, -3.5, 0.0, 3.5, 4.0]), 16.1, 7)
    assert v[0] == 0 and v[-1] == 0 and v[2] == 1.0
