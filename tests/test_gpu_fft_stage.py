"""The fine-grid FFT stage pinned against numpy.fft (fp64).

The reference's FFT boundary is mlx_nufft/gpu_t3.py:94-148 (axis-by-axis
c2c transforms, inverse for isign > 0, scale folded into the corrections);
no reference test pins it on its own.  Here the stage is isolated through
the staged C ABI:

  * type 2: nufft_execute_stage(SPREAD) leaves the transformed padded grid
    in plan memory (nufft_get_grid); it must equal numpy's FFT of the
    padded, deconvolved modes (the corrections come from the CPU oracle);
  * type 1: the spread grid after SPREAD is copied out, FINISH runs the FFT
    with the crop; the result must equal numpy's FFT of that grid, cropped
    to the mode box and deconvolved.

Paths: this library's two-pass 1-D FFT (fft1.cu, 2^12..2^22 cells), its
pruned three-pass 3-D FFT (power-of-two sides), cuFFT C2C (other sizes)
and cuFFT Z2Z (the fp64-FFT mode at upsampfac 1.25).  Gate: relative L2
error of an fp32 FFT with accurately rounded twiddles, 2e-6 (5e-7 rms is
typical; numpy's own complex64 FFT is ~4e-8 rms); fp64 mode 2e-7 (its
input is rounded to fp32).
"""

import numpy as np
import pytest

from oracle import port

pytestmark = pytest.mark.gpu

FP32_FFT = 2e-6


def _decs(N, n_up, eps, upsampfac):
    w, beta = port.kernel_params(eps, upsampfac)
    out = []
    for d in range(len(N)):
        k = np.arange(-(N[d] // 2), N[d] - N[d] // 2, dtype=np.float64)
        out.append(1.0 / port.kernel_ft(2.0 * np.pi * k / n_up[d], beta, w))
    return out


def _np_fft(H, isign):
    if isign > 0:
        return np.fft.ifftn(H) * H.size
    return np.fft.fftn(H)


def _scale(dec, N):
    s = np.ones(N)
    for d, v in enumerate(dec):
        s = s * v.reshape((1,) * d + (-1,) + (1,) * (len(N) - d - 1))
    return s


PAD_CASES = [  # (N, upsampfac, eps, expected own-FFT flag)
    ((2048,), 2.0, 1e-6, 1),           # fft1: 4096 cells = 64 x 64
    ((1 << 16,), 2.0, 1e-6, 1),
    ((1 << 21,), 2.0, 1e-6, 1),         # fft1: 2^22 cells = 2048 x 2048
    ((3000,), 2.0, 1e-6, 0),            # cuFFT (n_up 6000)
    ((64, 32, 32), 2.0, 1e-6, 1),       # pruned 3-D: 128 x 64 x 64
    ((256, 64, 128), 2.0, 1e-5, 1),     # pruned 3-D, unequal sides
    ((24, 20, 16), 2.0, 1e-6, 0),       # cuFFT 3-D (48 x 40 x 32)
    ((50, 40), 2.0, 1e-6, 0),           # cuFFT 2-D
    ((40, 36, 30), 1.25, 1e-7, 0),      # cuFFT Z2Z (fp64 mode)
]


@pytest.mark.parametrize("N,upsampfac,eps,own", PAD_CASES)
@pytest.mark.parametrize("isign", [-1, +1])
def test_type2_fft_stage(N, upsampfac, eps, own, isign, rng):
    import torch
    from mlx_nufft_b200 import Type2PlanND, _lib
    from mlx_nufft_b200.parallel import plan_grid_view
    dim = len(N)
    x = [rng.uniform(-np.pi, np.pi, 1000) for _ in range(dim)]
    plan = Type2PlanND(tuple(x), N, eps=eps, isign=isign, upsampfac=upsampfac)
    info = plan._plan.info()
    assert info.fft_own == own
    f = rng.standard_normal(N) + 1j * rng.standard_normal(N)
    ft = torch.from_numpy(f.astype(np.complex64)).cuda()
    plan._plan.execute_stage(_lib.STAGE_SPREAD, ft, None, 1)
    torch.cuda.synchronize()
    G = plan_grid_view(plan._plan, plan.n_up, fp64=bool(info.fft64)).cpu().numpy()[0]
    # numpy: the same complex64 modes, padded with the fp64 corrections
    H = np.zeros(plan.n_up, dtype=np.complex128)
    H[np.ix_(*[port._band(N[d], plan.n_up[d]) for d in range(dim)])] = \
        f.astype(np.complex64).astype(np.complex128) * _scale(
            _decs(N, plan.n_up, eps, upsampfac), N)
    ref = _np_fft(H, isign)
    err = port.rel_l2(G, ref)
    # fp64 mode: the FFT is fp64 but its input (complex64 modes times the
    # fp32-stored corrections) carries fp32 rounding, ~6e-8 relative
    assert err <= (2e-7 if info.fft64 else FP32_FFT), err


CROP_CASES = [
    ((2048,), 1e-6, 1),
    ((1 << 20,), 1e-6, 1),
    ((3000,), 1e-6, 0),
    ((64, 32, 32), 1e-6, 1),
    ((128, 64, 32), 1e-5, 1),
    ((24, 20, 16), 1e-6, 0),
]


@pytest.mark.parametrize("N,eps,own", CROP_CASES)
@pytest.mark.parametrize("isign", [+1, -1])
def test_type1_fft_crop_stage(N, eps, own, isign, rng):
    import torch
    from mlx_nufft_b200 import Type1PlanND, _lib
    from mlx_nufft_b200.parallel import plan_grid_view
    dim = len(N)
    M = 30_000
    x = [rng.uniform(-np.pi, np.pi, M) for _ in range(dim)]
    plan = Type1PlanND(tuple(x), N, eps=eps, isign=isign)
    assert plan._plan.info().fft_own == own
    c = rng.standard_normal(M) + 1j * rng.standard_normal(M)
    ct = torch.from_numpy(c.astype(np.complex64)).cuda()
    plan._plan.execute_stage(_lib.STAGE_SPREAD, ct, None, 1)
    torch.cuda.synchronize()
    G = plan_grid_view(plan._plan, plan.n_up).cpu().numpy()[0].astype(np.complex128)
    out = torch.empty(N, dtype=torch.complex64, device="cuda")
    plan._plan.execute_stage(_lib.STAGE_FINISH, None, out, 1)
    V = _np_fft(G, isign)
    ref = V[np.ix_(*[port._band(N[d], plan.n_up[d]) for d in range(dim)])] * _scale(
        _decs(N, plan.n_up, eps, 2.0), N)
    err = port.rel_l2(out.cpu().numpy(), ref)
    assert err <= FP32_FFT, err


def test_pruned_3d_batch_and_full_transform(rng):
    """The pruned 3-D FFT inside whole transforms: a batch of 3 vectors
    (scratch per vector) through type 2 and type 1, against the fp64
    restatement of the pipeline."""
    from mlx_nufft_b200 import Type1PlanND, Type2PlanND
    N, M, eps = (32, 64, 32), 60_000, 1e-6
    x = [rng.uniform(-np.pi, np.pi, M) for _ in range(3)]
    p2 = Type2PlanND(tuple(x), N, eps=eps)
    assert p2._plan.info().fft_own == 1
    fs = rng.standard_normal((3,) + N) + 1j * rng.standard_normal((3,) + N)
    cs = p2.execute_batch(fs)
    for v in range(3):
        assert port.rel_l2(cs[v], port.nufft_t2(x, fs[v], eps, -1)) <= 2e-5
    p1 = Type1PlanND(tuple(x), N, eps=eps)
    assert p1._plan.info().fft_own == 1
    c3 = rng.standard_normal((3, M)) + 1j * rng.standard_normal((3, M))
    fk = p1.execute_batch(c3)
    for v in range(3):
        assert port.rel_l2(fk[v], port.nufft_t1(x, c3[v], N, eps, +1)) <= 2e-5
