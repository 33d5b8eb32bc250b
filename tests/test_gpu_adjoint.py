"""nufft_execute_adjoint through the C ABI (ctypes, raw device pointers).

For every plan type the adjoint is the sibling transform with the opposite
sign (mlx_nufft/api.py:347-388).  Checked two ways:
  * the pairing identity <A c, f> = <c, A* f> (A the plan's transform, A*
    its adjoint, <a, b> = sum conj(a) b), to max(10 eps, 1e-5) relative;
  * A* f against the exact fp64 direct sum of the sibling transform (the
    CPU oracle) on a subset of its outputs.
At upsampfac 1.25 (type 3, and the type-1 fp64-FFT case) the gate is the
1e-4 floor of the fp32 spread / interp at that upsampling.
Types 1/2 run the adjoint on the plan's own sorted points (the tiled,
streamed and TMA-staged interp kernels on a spread-sorted point set, and
the spread kernels on an interp-sorted one); type 3 builds its sibling plan
inside the library on the first call."""

import ctypes

import numpy as np
import pytest

from oracle import port

pytestmark = pytest.mark.gpu

CASES = [  # (type, N or None, M, eps)
    (1, (4096,), 300_000, 1e-6),      # 1-D: streamed interp on a spread sort
    (2, (4096,), 300_000, 1e-6),      # 1-D: tiled spread on an interp sort
    (1, (64, 48), 120_000, 1e-6),
    (2, (64, 48), 120_000, 1e-5),
    (1, (32, 28, 24), 200_000, 1e-6),  # 3-D: TMA interp on 8^3 bins
    (2, (32, 28, 24), 200_000, 1e-6),  # 3-D: plane spread on 10^3 bins
    (1, (40, 36), 30_000, 1e-7),       # fp64-FFT plan (upsampfac 1.25)
    (3, None, 40_000, 1e-5),
]


def _ip(a, b):
    return np.vdot(np.asarray(a).ravel(), np.asarray(b).ravel())


@pytest.mark.parametrize("typ,N,M,eps", CASES)
def test_execute_adjoint_cabi(typ, N, M, eps):
    import torch
    from mlx_nufft_b200._lib import check, lib, default_opts

    rng = np.random.default_rng(100 + typ + M % 97)
    dim = len(N) if N else 3
    x = [rng.uniform(-np.pi, np.pi, M) for _ in range(dim)]
    opts = default_opts()
    upsamp = 1.25 if eps == 1e-7 else 0.0
    opts.upsampfac = upsamp
    isign = +1 if typ != 2 else -1
    nm = (ctypes.c_int64 * 3)(*((list(N) if N else []) + [1] * (3 - (len(N) if N else 0))))
    h = ctypes.c_void_p()
    check(lib.nufft_plan_create(typ, dim, nm, 1, eps, isign, ctypes.byref(opts), 0,
                                ctypes.byref(h)))
    try:
        dev = torch.device("cuda", 0)
        xs = [torch.from_numpy(v).to(dev) for v in x]
        st = torch.cuda.current_stream().cuda_stream
        if typ == 3:
            Nt = 30_000
            s = [rng.uniform(-25, 25, Nt) for _ in range(3)]
            ss = [torch.from_numpy(v).to(dev) for v in s]
            check(lib.nufft_setpts(h, M, *[t.data_ptr() for t in xs], Nt,
                                   *[t.data_ptr() for t in ss], st))
            nin, nout = M, Nt
        else:
            ptrs = [t.data_ptr() for t in xs] + [None] * (3 - dim)
            check(lib.nufft_setpts(h, M, *ptrs, 0, None, None, None, st))
            K = int(np.prod(N))
            nin, nout = (M, K) if typ == 1 else (K, M)
        a = rng.standard_normal(nin) + 1j * rng.standard_normal(nin)
        b = rng.standard_normal(nout) + 1j * rng.standard_normal(nout)
        ta = torch.from_numpy(a.astype(np.complex64)).to(dev)
        tb = torch.from_numpy(b.astype(np.complex64)).to(dev)
        Aa = torch.empty(nout, dtype=torch.complex64, device=dev)
        Ab = torch.empty(nin, dtype=torch.complex64, device=dev)
        check(lib.nufft_execute(h, ta.data_ptr(), Aa.data_ptr(), 1, st))
        check(lib.nufft_execute_adjoint(h, tb.data_ptr(), Ab.data_ptr(), 1, st))
        check(lib.nufft_plan_check(h, st))
        Aa, Ab = Aa.cpu().numpy(), Ab.cpu().numpy()
        assert np.all(np.isfinite(Ab))
        # upsampfac 1.25: the fp32 spread / interp error is amplified by the
        # 1/phihat corrections near the band edge (1e3..1e5), a floor of
        # ~1e-5..1e-4 for any fp32 pipeline of this algorithm
        tol = max(10 * eps, 1e-5) if (upsamp == 0.0 and typ != 3) else 1e-4
        lhs, rhs = _ip(Aa, b), _ip(a, Ab)
        scale = np.linalg.norm(Aa) * np.linalg.norm(b)
        assert abs(lhs - rhs) <= tol * scale, (lhs, rhs)
        # the adjoint against the exact sum of the sibling transform
        idx = rng.choice(nin, 48, replace=False)
        if typ == 1:     # modes -> points, sign -isign
            ref = port.direct_t2(x, b.reshape(N), -isign, idx)
        elif typ == 2:   # points -> modes, sign -isign
            ref = port.direct_t1(x, b, N, -isign, idx)
        else:            # targets -> sources, sign -isign
            xs_sub = [v[idx] for v in x]
            ref = port.direct_sum(s, b, xs_sub, -isign)
        assert port.rel_l2(Ab[idx], ref) <= tol
        # a second call reuses the sibling (type 3) / the plan's buffers
        Ab2 = torch.empty(nin, dtype=torch.complex64, device=dev)
        check(lib.nufft_execute_adjoint(h, tb.data_ptr(), Ab2.data_ptr(), 1, st))
        torch.cuda.synchronize()
        # spreads sum with atomics (order varies between calls), and type 3's
        # corrections amplify that rounding
        assert port.rel_l2(Ab2.cpu().numpy(), Ab) <= (1e-6 if typ == 1 else tol)
    finally:
        lib.nufft_plan_destroy(h)


def test_execute_adjoint_errors():
    import torch
    from mlx_nufft_b200._lib import NUFFT_ERR_STATE, lib, default_opts
    opts = default_opts()
    nm = (ctypes.c_int64 * 3)(16, 1, 1)
    h = ctypes.c_void_p()
    assert lib.nufft_plan_create(1, 1, nm, 1, 1e-6, 1, ctypes.byref(opts), 0,
                                 ctypes.byref(h)) == 0
    buf = torch.zeros(16, dtype=torch.complex64, device="cuda")
    try:
        rc = lib.nufft_execute_adjoint(h, buf.data_ptr(), buf.data_ptr(), 1, None)
        assert rc == NUFFT_ERR_STATE
    finally:
        lib.nufft_plan_destroy(h)
