"""GPU parity of the finufft-compatible API (mirrors the reference's
harness/test_api_parity.py matrix, with the exact direct sum as the oracle
instead of CPU finufft), the Plan interface, execute_adjoint, batched /
re-pointed / disjoint type-1 execution (harness/test_type1_batch.py,
harness/test_type1_setsources_gpu.py) and the error conventions."""

import warnings

import numpy as np
import pytest

from oracle import port, fast

pytestmark = pytest.mark.gpu


def gate(eps):
    return max(10 * eps, 1e-5)


M = 4000


def pts(rng, dim, n=M):
    return [rng.uniform(-np.pi, np.pi, n) for _ in range(dim)]


@pytest.mark.parametrize("eps", [1e-3, 1e-5])
@pytest.mark.parametrize("dim,N", [(1, (90,)), (1, (87,)), (2, (48, 36)),
                                   (2, (45, 34)), (3, (24, 20, 16)),
                                   (3, (21, 18, 14))])
@pytest.mark.parametrize("isign", [+1, -1])
def test_api_matrix(eps, dim, N, isign, rng):
    import mlx_nufft_b200 as gpu
    x = pts(rng, dim)
    c = rng.standard_normal(M) + 1j * rng.standard_normal(M)
    f1 = getattr(gpu, f"nufft{dim}d1")(*x, c, N, eps=eps, isign=isign)
    assert f1.dtype == np.complex128 and f1.shape == N
    assert port.rel_l2(f1, fast.direct_t1(x, c, N, isign).reshape(N)) <= gate(eps)
    fk = rng.standard_normal(N) + 1j * rng.standard_normal(N)
    c2 = getattr(gpu, f"nufft{dim}d2")(*x, fk, eps=eps, isign=isign)
    assert c2.shape == (M,)
    assert port.rel_l2(c2, fast.direct_t2(x, fk, isign)) <= gate(eps)
    s = [rng.uniform(-30, 30, 1500) for _ in range(dim)]
    f3 = getattr(gpu, f"nufft{dim}d3")(*x, c, *s, eps=eps, isign=isign)
    assert f3.shape == (1500,)
    exact = fast.direct_sum(x, c, s, isign)
    # type 3 runs at sigma = 1.25: the reference's fp32 pipeline on the
    # same inputs sets the floor (oracle.port.nufft_t3_fp32, pinned to it)
    floor = port.rel_l2(port.nufft_t3_fp32(x, c, s, eps=eps, isign=isign), exact)
    assert port.rel_l2(f3, exact) <= max(gate(eps), 1.5 * floor)


def test_plan_interface_ntrans_c64_out(rng):
    import mlx_nufft_b200 as gpu
    eps = 1e-5
    N = (40, 36)
    x = pts(rng, 2)
    cs = (rng.standard_normal((3, M)) + 1j * rng.standard_normal((3, M))
          ).astype(np.complex64)
    p = gpu.Plan(1, N, n_trans=3, eps=eps, isign=+1, dtype="complex64")
    p.setpts(*x)
    out = np.empty((3,) + N, dtype=np.complex64)
    got = p.execute(cs, out=out)
    assert got is out and out.dtype == np.complex64
    for b in range(3):
        ref = fast.direct_t1(x, cs[b], N, +1).reshape(N)
        assert port.rel_l2(out[b], ref) <= gate(eps)
    p2 = gpu.Plan(2, N, n_trans=3, eps=eps, isign=-1, dtype="complex64")
    p2.setpts(*x)
    fks = (rng.standard_normal((3,) + N) + 1j * rng.standard_normal((3,) + N)
           ).astype(np.complex64)
    got2 = p2.execute(fks)
    for b in range(3):
        assert port.rel_l2(got2[b], fast.direct_t2(x, fks[b], -1)) <= gate(eps)
    p3 = gpu.Plan(3, 2, n_trans=1, eps=eps, isign=+1)
    s = [rng.uniform(-30, 30, 1500) for _ in range(2)]
    p3.setpts(x[0], x[1], s=s[0], t=s[1])
    c = rng.standard_normal(M) + 1j * rng.standard_normal(M)
    assert port.rel_l2(p3.execute(c), fast.direct_sum(x, c, s, +1)) <= gate(eps)
    with pytest.raises(ValueError):
        p.execute(cs[:2])


def test_execute_adjoint(rng):
    import mlx_nufft_b200 as gpu
    N = (30, 22)
    x = pts(rng, 2)
    p = gpu.Plan(1, N, eps=1e-6, isign=+1)
    p.setpts(*x)
    fk = rng.standard_normal(N) + 1j * rng.standard_normal(N)
    adj = p.execute_adjoint(fk)          # type 2 with isign -1
    assert port.rel_l2(adj, fast.direct_t2(x, fk, -1)) <= gate(1e-6)
    q = gpu.Plan(2, N, eps=1e-6)
    q.setpts(*x)
    c = rng.standard_normal(M) + 1j * rng.standard_normal(M)
    adj2 = q.execute_adjoint(c)          # type 1 with isign +1
    assert port.rel_l2(adj2, fast.direct_t1(x, c, N, +1).reshape(N)) <= gate(1e-6)
    r = gpu.Plan(3, 1, eps=1e-6)
    s = rng.uniform(-20, 20, 900)
    r.setpts(x[0], s=s)
    g = rng.standard_normal(900) + 1j * rng.standard_normal(900)
    adj3 = r.execute_adjoint(g)          # targets -> sources, isign -1
    assert port.rel_l2(adj3, fast.direct_sum([s], g, [x[0]], -1)) <= gate(1e-6)


def test_adjoint_pairing_3d(rng):
    """<T1 c, f> == <c, T2 f> (harness/test_types12.py:40-48)."""
    from mlx_nufft_b200 import Type1Plan, Type2Plan
    N = (32, 24, 16)
    x = pts(rng, 3, 50_000)
    c = rng.standard_normal(50_000) + 1j * rng.standard_normal(50_000)
    fk = rng.standard_normal(N) + 1j * rng.standard_normal(N)
    f1 = Type1Plan(x, N, eps=1e-5, isign=+1).execute(c.astype(np.complex64))
    c2 = Type2Plan(x, N, eps=1e-5, isign=-1).execute(fk.astype(np.complex64))
    lhs = np.vdot(fk, f1)
    rhs = np.vdot(c2, c)
    # Cauchy-Schwarz scale (the pairing itself cancels; the reference only
    # prints this number)
    scale = np.linalg.norm(fk) * np.linalg.norm(f1)
    assert abs(lhs - rhs) / scale < 1e-5
    with pytest.raises(AssertionError):
        Type1Plan(x, (31, 24, 16))


def test_dtype_roundtrip_and_options(rng):
    import mlx_nufft_b200 as gpu
    x = pts(rng, 1)
    c = (rng.standard_normal(M) + 1j * rng.standard_normal(M)).astype(np.complex64)
    assert gpu.nufft1d1(x[0], c, 16).dtype == np.complex64
    assert gpu.nufft1d1(x[0], c.astype(np.complex128), 16).dtype == np.complex128
    with pytest.raises(NotImplementedError):
        gpu.nufft1d1(x[0], c, 16, modeord=1)
    with warnings.catch_warnings(record=True) as w:
        warnings.simplefilter("always")
        gpu.nufft1d1(x[0], c, 16, eps=1e-9)
        gpu.nufft1d1(x[0], c, 16, foo=3, nthreads=4)
    msgs = " ".join(str(v.message) for v in w)
    assert "clamping" in msgs and "foo" in msgs and "nthreads" not in msgs
    out = np.empty(16, dtype=np.complex128)
    assert gpu.nufft1d1(x[0], c, out=out) is out
    cs = np.stack([c, c])
    f2 = gpu.nufft1d1(x[0], cs, 16)
    assert f2.shape == (2, 16)
    with pytest.raises(ValueError):
        gpu.nufft1d1(x[0], c[:10], 16)
    with pytest.raises(ValueError):
        gpu.Plan(4, (8,))
    with pytest.raises(ValueError):
        gpu.Plan(1, (8,), dtype="float32")
    with pytest.raises(RuntimeError):
        gpu.Plan(1, (8,)).execute(c)


def test_torch_inputs_and_device_outputs(rng):
    import torch
    from mlx_nufft_b200 import Type1PlanND, Type2PlanND
    x = torch.from_numpy(rng.uniform(-np.pi, np.pi, M)).cuda()
    c = torch.randn(M, dtype=torch.complex64, device="cuda")
    p = Type1PlanND(x, (64,), eps=1e-6)
    f = p.execute(c, return_np=False)
    assert isinstance(f, torch.Tensor) and f.is_cuda and f.shape == (64,)
    ref = fast.direct_t1([x.cpu().numpy()], c.cpu().numpy(), (64,), +1)
    assert port.rel_l2(f.cpu().numpy(), ref) <= gate(1e-6)
    q = Type2PlanND(x.cpu(), (64,), eps=1e-6)
    cj = q.execute(f, return_np=False)
    assert cj.is_cuda and cj.shape == (M,)


# ---------------------------------------------------- batch / re-point
@pytest.mark.parametrize("dim,N,P,B", [(1, (4096,), 200_000, 5),
                                       (2, (256, 256), 200_000, 5),
                                       (2, (192, 160), 5_000, 4),
                                       (3, (64, 64, 48), 5_000, 6),
                                       (3, (64, 64, 48), 200_000, 8)])
@pytest.mark.parametrize("isign", [+1, -1])
def test_execute_batch(dim, N, P, B, isign, rng):
    from mlx_nufft_b200 import Type1PlanND
    x = pts(rng, dim, P)
    cs = (rng.standard_normal((B, P)) + 1j * rng.standard_normal((B, P))
          ).astype(np.complex64)
    plan = Type1PlanND(tuple(x), N, eps=1e-5, isign=isign)
    fb = plan.execute_batch(cs)
    assert fb.shape == (B,) + N
    idx = rng.choice(int(np.prod(N)), 100, replace=False)
    for b in range(B):
        fl = plan.execute(cs[b])
        assert port.rel_l2(fb[b], fl) < 1e-5                    # batch == loop
        ref = fast.direct_t1(x, cs[b], N, isign, idx)
        assert port.rel_l2(fb[b].ravel()[idx], ref) <= gate(1e-5)


@pytest.mark.parametrize("dim,N,P", [(2, (256, 256), 50_000),
                                     (3, (64, 64, 48), 50_000)])
def test_set_sources_repoint(dim, N, P, rng):
    from mlx_nufft_b200 import Type1PlanND
    x1, x2 = pts(rng, dim, P), pts(rng, dim, P)
    c = (rng.standard_normal(P) + 1j * rng.standard_normal(P)).astype(np.complex64)
    plan = Type1PlanND(tuple(x1), N, eps=1e-5, isign=+1)
    for backend in ("host", "gpu"):
        plan.set_sources(x2, backend=backend)
        fresh = Type1PlanND(tuple(x2), N, eps=1e-5, isign=+1).execute(c)
        assert port.rel_l2(plan.execute(c), fresh) < 1e-5
    P2 = P // 3
    x3 = pts(rng, dim, P2)
    c3 = c[:P2]
    plan.set_sources(x3)
    assert plan.P == P2
    fresh = Type1PlanND(tuple(x3), N, eps=1e-5, isign=+1).execute(c3)
    assert port.rel_l2(plan.execute(c3), fresh) < 1e-5
    with pytest.raises(ValueError):
        plan.set_sources(x3, backend="cuda")


@pytest.mark.parametrize("dim,N,P,G", [(2, (128, 96), 100_000, 4),
                                       (1, (2048,), 60_000, 3),
                                       (3, (32, 32, 16), 80_000, 5)])
def test_execute_disjoint(dim, N, P, G, rng):
    """Each group's transform against the exact direct sum of that group's
    points alone (the CPU oracle), on a subset of the modes, and against
    the fp64 restatement of the type-1 pipeline on the group's points."""
    from mlx_nufft_b200 import Type1PlanND
    x = pts(rng, dim, P)
    c = (rng.standard_normal(P) + 1j * rng.standard_normal(P)).astype(np.complex64)
    groups = rng.integers(0, G, P)
    eps = 1e-5
    plan = Type1PlanND(tuple(x), N, eps=eps)
    fd = plan.execute_disjoint(c, groups)
    assert fd.shape == (G,) + N
    K = int(np.prod(N))
    kidx = rng.choice(K, 64, replace=False)
    for g in range(G):
        sel = groups == g
        xg = [v[sel] for v in x]
        ref = fast.direct_t1(xg, c[sel], N, +1, kidx)
        assert port.rel_l2(fd[g].ravel()[kidx], ref) <= gate(eps)
        full = port.nufft_t1(xg, c[sel], N, eps, +1)
        assert port.rel_l2(fd[g], full) <= 2e-5
    with pytest.raises(ValueError):
        plan.execute_disjoint(c, groups[:10])


def test_error_conventions(rng):
    from mlx_nufft_b200 import Type1PlanND, Type2PlanND, Type3Plan
    x = pts(rng, 2, 1000)
    with pytest.raises(ValueError):
        Type1PlanND(tuple(x), (16, 16, 16))
    with pytest.raises(ValueError):
        Type1PlanND(tuple(x), (16, 0))
    with pytest.raises(ValueError):
        Type1PlanND(tuple(x), (16, 16), upsampfac=5.0)
    with pytest.raises(ValueError):
        Type1PlanND(tuple(x), (16, 16), prec="fp16")
    with pytest.raises(ValueError):
        Type1PlanND((x[0], x[1][:10]), (16, 16))
    p = Type1PlanND(tuple(x), (16, 16))
    with pytest.raises(ValueError):
        p.execute(np.zeros(999, np.complex64))
    q = Type2PlanND(tuple(x), (16, 16))
    with pytest.raises(ValueError):
        q.execute(np.zeros((16, 15), np.complex64))
    with pytest.raises(ValueError):
        Type1PlanND((np.array([0.0, np.nan]),), (8,))
    with pytest.raises(AssertionError):
        Type3Plan(tuple(x), tuple(x), prec="bad")
    with pytest.raises(RuntimeError):
        Type3Plan(tuple(x), tuple(x), fft_backend="vkfft")
    t3 = Type3Plan(tuple(x), tuple(x))
    with pytest.raises(AssertionError):
        t3.execute(np.zeros(5, np.complex64))


def test_execute_into_host_out_and_launch_count(rng):
    """execute(..., out=) writes the result into a caller-provided host
    buffer (pinned torch tensor or numpy array) and returns it; the plan's
    launch counter advances by this library's own kernels per execute."""
    import torch
    from mlx_nufft_b200 import Type1PlanND, Type2PlanND
    x = pts(rng, 1, 50_000)
    fk = (rng.standard_normal(4096) + 1j * rng.standard_normal(4096)).astype(np.complex64)
    q = Type2PlanND(tuple(x), (4096,))
    ref = q.execute(fk)
    host = torch.empty(50_000, dtype=torch.complex64).pin_memory()
    assert q.execute(torch.from_numpy(fk).pin_memory(), out=host) is host
    assert np.array_equal(host.numpy(), ref)
    arr = np.empty(50_000, np.complex64)
    assert q.execute(fk, out=arr) is arr
    assert np.array_equal(arr, ref)
    with pytest.raises(ValueError):
        q.execute(fk, out=np.empty(10, np.complex64))
    n0 = q._plan.info().kernel_launches
    f0 = q._plan.info().fft_execs
    q.execute(fk)
    info = q._plan.info()
    # 8192-cell grid: the two-pass FFT with the pad fused + interp, no cuFFT
    assert info.fft_own == 1
    assert info.kernel_launches - n0 == 3
    assert info.fft_execs == f0
    c = (rng.standard_normal(50_000) + 1j * rng.standard_normal(50_000)).astype(np.complex64)
    p = Type1PlanND(tuple(x), (4096,))
    n0 = p._plan.info().kernel_launches
    out = np.empty((4096,), np.complex64)
    p.execute(c, out=out)
    assert p._plan.info().kernel_launches - n0 == 3  # spread, FFT pass 1, pass 2 + crop
    # spreading accumulates with float atomics: order-dependent rounding
    assert port.rel_l2(out, p.execute(c)) <= 1e-6


@pytest.mark.parametrize("upsampfac", [2.0, 1.25])
def test_staged_execute_and_parallel_stages(upsampfac, rng):
    """Staged execute (type 1: spread | FFT+crop; type 2: pad+FFT | interp)
    through mlx_nufft_b200.parallel's single-rank path equals execute();
    at upsampfac 1.25 the type-2 grid is the fp64-FFT complex128 grid."""
    import torch
    from mlx_nufft_b200 import Type1PlanND, Type2PlanND, parallel as par
    x = pts(rng, 2, 30_000)
    N = (40, 36)
    c = rng.standard_normal(30_000) + 1j * rng.standard_normal(30_000)
    eps = 1e-5    # at upsampfac 1.25 the fp32 floor is above 1e-5
    p1 = Type1PlanND(tuple(x), N, eps=eps, upsampfac=upsampfac)
    got1 = par.Type1PointSplit(par.PlanStages(p1)).execute(c).reshape(N)
    # spreading sums with float atomics, and 1/phihat at upsampfac 1.25
    # amplifies their order noise: both paths are held to the exact sum
    exact = fast.direct_t1(x, c, N, +1).reshape(N)
    assert port.rel_l2(got1, exact) <= gate(eps)
    assert port.rel_l2(p1.execute(c), exact) <= gate(eps)
    f = rng.standard_normal(N) + 1j * rng.standard_normal(N)
    p2 = Type2PlanND(tuple(x), N, eps=eps, upsampfac=upsampfac)
    st = par.PlanStages(p2)
    assert st.fp64 == (upsampfac < 1.5)
    g = st.first(f)
    assert g.shape == (1,) + tuple(p2.n_up)
    assert g.dtype == (torch.complex128 if st.fp64 else torch.complex64)
    got2 = par.Type2TargetSplit(st, 30_000).execute(f)
    np.testing.assert_array_equal(got2, p2.execute(f))
