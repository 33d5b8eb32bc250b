"""Generate the golden fixtures in tests/golden/ from the REFERENCE's own CPU
code (martinlachaine/mlx-nufft v0.1.3).

Run in the build container, where the reference checkout is available:

    python tests/golden/make_golden.py <path-to-reference-checkout>

The reference package imports MLX in mlx_nufft/__init__.py, which is not
installable here; its numpy-only modules (mlx_nufft/sizing.py,
mlx_nufft/ref_t3.py, harness/gen.py) are imported through a stub package
object whose __path__ points at the checkout, so __init__.py never runs.
Nothing in the fixtures is computed by this repository's code: every array
comes from the reference functions named beside it.  The fixtures travel
with the repo; the GPU box never needs the reference checkout.
"""

import os
import sys
import types

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))


def load_reference(root):
    for name, sub in (("mlx_nufft", "mlx_nufft"), ("harness", "harness")):
        mod = types.ModuleType(name)
        mod.__path__ = [os.path.join(root, sub)]
        sys.modules[name] = mod
    from mlx_nufft import sizing, ref_t3          # noqa: E402
    from harness import gen                      # noqa: E402
    return sizing, ref_t3, gen


def make_sizing(sizing):
    eps_list = np.array([1e-1, 3e-2, 1e-2, 1e-3, 3e-4, 1e-4, 1e-5, 5e-6, 1e-6,
                         3e-7, 1e-7, 1e-8, 1e-9, 1e-10, 1e-12, 1e-14])
    sigmas = np.array([2.0, 1.25, 1.1, 1.5, 3.0, 4.0])
    ws = np.zeros((eps_list.size, sigmas.size), dtype=np.int64)
    betas = np.zeros_like(ws, dtype=np.float64)
    for i, e in enumerate(eps_list):
        for j, s in enumerate(sigmas):
            ws[i, j], betas[i, j] = sizing.kernel_params(float(e), float(s))
    n235_in = np.arange(0, 4000)
    n235 = np.array([sizing.next235even(int(n)) for n in n235_in])
    kft_wb = []
    kft_xi = np.linspace(-np.pi, np.pi, 41)
    kft_val = []
    for e, s in ((1e-6, 2.0), (1e-5, 2.0), (1e-5, 1.25), (1e-6, 1.25),
                 (1e-3, 2.0), (1e-9, 2.0)):
        w, b = sizing.kernel_params(e, s)
        kft_wb.append((w, b))
        kft_val.append(sizing.kernel_ft(kft_xi, b, w))
    nhg_in = np.array([(20.0, 10.0, 1.25, 9), (0.0, 0.0, 1.25, 9),
                       (5.0, 0.0, 1.25, 7), (0.0, 3.0, 2.0, 7),
                       (7.17e-4, 1.2e7, 1.25, 9), (30.0, 30.0, 1.25, 10),
                       (1.0, 1.0, 2.0, 2), (100.0, 0.01, 1.5, 6)])
    nhg_out = np.array([sizing.set_nhg_type3(S, X, s, int(w))
                        for S, X, s, w in nhg_in])
    np.savez_compressed(os.path.join(HERE, "sizing.npz"),
                        eps=eps_list, sigma=sigmas, w=ws, beta=betas,
                        n235_in=n235_in, n235=n235,
                        kft_wb=np.array(kft_wb), kft_xi=kft_xi,
                        kft_val=np.array(kft_val),
                        nhg_in=nhg_in, nhg_out=nhg_out)


def make_t3(ref_t3, gen):
    cases = []
    rng = np.random.default_rng(2024)
    # cfg-5 geometry (X=10, S=20) at a small point count
    P, M = 800, 300
    cases.append(dict(x=tuple(rng.uniform(-10, 10, P) for _ in range(3)),
                      s=tuple(rng.uniform(-20, 20, M) for _ in range(3)),
                      eps=1e-5, isign=+1))
    # small extents, eps=1e-6, isign -1
    P, M = 1000, 400
    cases.append(dict(x=tuple(rng.uniform(-2, 2, P) for _ in range(3)),
                      s=tuple(rng.uniform(-3, 3, M) for _ in range(3)),
                      eps=1e-6, isign=-1))
    # the reference's anisotropic generator (large coordinate dynamic range)
    prob = gen.gen_anisotropic(N=12, P=300, lat=0.02, seed=5)
    cases.append(dict(x=prob["x"], s=prob["s"], c=prob["c"], eps=1e-5,
                      isign=+1))
    out = {}
    for i, cs in enumerate(cases):
        x, s = cs["x"], cs["s"]
        P = x[0].size
        c = cs.get("c")
        if c is None:
            c = rng.standard_normal(P) + 1j * rng.standard_normal(P)
        plan = ref_t3.RefT3Plan(x, s, eps=cs["eps"], isign=cs["isign"],
                                flags=ref_t3.FULL64)
        f = plan.execute(c)
        fd = gen.direct_sum(x, c, s, isign=cs["isign"])
        # the reference's fp32 pipeline with crit64 geometry (fp64 coords
        # and phases, fp32 spread/FFT/interp/deconvolution): the accuracy
        # floor its GPU path is designed to (ref_t3.py:29-48)
        crit32 = ref_t3.Flags(coords64=True, phases64=True, spread64=False,
                              fft64=False, interp64=False, deconv64=False)
        f32 = ref_t3.RefT3Plan(x, s, eps=cs["eps"], isign=cs["isign"],
                               flags=crit32).execute(c)
        pre = f"c{i}_"
        out.update({pre + "x": np.stack(x), pre + "s": np.stack(s),
                    pre + "c": c, pre + "eps": cs["eps"],
                    pre + "isign": cs["isign"], pre + "out": f,
                    pre + "out32": f32,
                    pre + "direct": fd, pre + "nf": np.array(plan.nf),
                    pre + "n_up": np.array(plan.n_up), pre + "w": plan.w,
                    pre + "beta": plan.beta, pre + "C": np.array(plan.C),
                    pre + "D": np.array(plan.D), pre + "gam": np.array(plan.gam),
                    pre + "i1": np.stack(plan.i1), pre + "fr": np.stack(plan.fr),
                    pre + "t_i1": np.stack(plan.t_i1),
                    pre + "t_fr": np.stack(plan.t_fr),
                    pre + "prephase": plan.prephase, pre + "post": plan.post,
                    pre + "mode_dec0": plan.mode_dec[0],
                    pre + "mode_dec1": plan.mode_dec[1],
                    pre + "mode_dec2": plan.mode_dec[2]})
    out["ncases"] = len(cases)
    np.savez_compressed(os.path.join(HERE, "t3_ref.npz"), **out)


def make_direct(gen):
    """Exact sums from the reference's direct_sum oracle (3-D signature;
    lower dimensions embedded with zero coordinates as the reference's API
    does, mlx_nufft/api.py:118-122)."""
    rng = np.random.default_rng(77)
    out = {}
    # type-1 style: sources = points, targets = the integer mode lattice
    for dim, N, M, isign in ((1, (40,), 500, +1), (2, (12, 9), 400, -1),
                             (3, (6, 5, 4), 300, +1)):
        x = [rng.uniform(-np.pi, np.pi, M) for _ in range(dim)]
        c = rng.standard_normal(M) + 1j * rng.standard_normal(M)
        ks = np.meshgrid(*[np.arange(-(n // 2), n - n // 2) for n in N],
                         indexing="ij")
        ks = [k.ravel().astype(np.float64) for k in ks]
        z = np.zeros(M)
        zk = np.zeros(ks[0].size)
        f = gen.direct_sum(tuple(x) + (z,) * (3 - dim), c,
                           tuple(ks) + (zk,) * (3 - dim), isign=isign)
        tag = f"t1_{dim}d_"
        out.update({tag + "x": np.stack(x), tag + "c": c, tag + "N": np.array(N),
                    tag + "isign": isign, tag + "f": f.reshape(N)})
        # type-2 style: sources = mode lattice with strengths fk, targets = x
        fk = rng.standard_normal(N) + 1j * rng.standard_normal(N)
        cj = gen.direct_sum(tuple(ks) + (zk,) * (3 - dim), fk.ravel(),
                            tuple(x) + (z,) * (3 - dim), isign=-isign)
        tag = f"t2_{dim}d_"
        out.update({tag + "x": np.stack(x), tag + "f": fk, tag + "N": np.array(N),
                    tag + "isign": -isign, tag + "c": cj})
    np.savez_compressed(os.path.join(HERE, "direct.npz"), **out)


def make_quickstart():
    """The reference's known-answer self-check (examples/quickstart.py:52-73):
    1-D type 1, M=2000, N=64, seed 2, exact DFT as the answer."""
    rng = np.random.default_rng(2)
    M, N = 2_000, 64
    x = rng.uniform(-np.pi, np.pi, M)
    c = rng.standard_normal(M) + 1j * rng.standard_normal(M)
    k = np.arange(-(N // 2), N - N // 2)
    f_exact = (c[None, :] * np.exp(1j * k[:, None] * x[None, :])).sum(axis=1)
    np.savez_compressed(os.path.join(HERE, "quickstart.npz"), x=x, c=c, N=N,
                        f_exact=f_exact, eps=1e-6)


def make_gen(gen):
    x, n_modes, M = gen.uniform_points(2, 16, rho=1.0, dist="rand", seed=3)
    xc, _, Mc = gen.uniform_points(3, 8, rho=0.5, dist="cluster", seed=4)
    g = gen.gen_generic(N=6, P=50, seed=1, X=3.0, S=2.0)
    a = gen.gen_anisotropic(N=6, P=40, lat=1.5, seed=0)
    np.savez_compressed(
        os.path.join(HERE, "gen.npz"),
        rand_x=np.stack(x), rand_M=M, cl_x=np.stack(xc), cl_M=Mc,
        gen_x=np.stack(g["x"]), gen_s=np.stack(g["s"]), gen_c=g["c"],
        an_x=np.stack(a["x"]), an_s=np.stack(a["s"]), an_c=a["c"])


def main():
    if len(sys.argv) != 2:
        sys.exit("usage: python tests/golden/make_golden.py <path of the "
                 "mlx-nufft v0.1.3 source tree>")
    root = sys.argv[1]
    sizing, ref_t3, gen = load_reference(root)
    make_sizing(sizing)
    make_gen(gen)
    make_direct(gen)
    make_quickstart()
    make_t3(ref_t3, gen)
    for f in sorted(os.listdir(HERE)):
        if f.endswith(".npz"):
            print(f, os.path.getsize(os.path.join(HERE, f)))


if __name__ == "__main__":
    main()
