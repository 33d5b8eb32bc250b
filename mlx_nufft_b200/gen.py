"""Synthetic problem generators (host numpy, seeded).

uniform_points / gen_generic / gen_anisotropic restate the reference's
harness generators (harness/gen.py:15-90) so benchmarks and parity tests
draw the same kind of inputs; `config(k)` builds the five benchmark
workloads (cfg 1..5, plus the standalone expi input for cfg 5) with their
stated shapes, distributions and seeds.  `scale` shrinks the point counts
for quick runs without changing anything else.
"""

import numpy as np

PI = np.pi


def uniform_points(dim, N, rho=1.0, dist="rand", sigma=2.0, seed=0):
    """Points for a type-1/2 problem at density rho = M / (sigma^dim N^dim)
    (harness/gen.py:62-90): 'rand' uniform on [-pi, pi)^dim, 'cluster' in a
    box of 8 fine-grid cells at the domain corner."""
    rng = np.random.default_rng(seed)
    M = int(round(rho * (sigma ** dim) * (N ** dim)))
    if dist == "rand":
        x = [rng.uniform(-np.pi, np.pi, M) for _ in range(dim)]
    elif dist == "cluster":
        h = 2.0 * np.pi / (sigma * N)
        x = [(-np.pi + rng.uniform(0.0, 8.0 * h, M)) for _ in range(dim)]
    else:
        raise ValueError(f"unknown dist {dist!r}")
    return [v.astype(np.float64) for v in x], (N,) * dim, M


def gen_generic(N=1024, P=100_000, seed=0, X=30.0, S=20.0):
    """Isotropic type 3: P sources in [-X, X]^3, N^2 targets in [-S, S]^3
    (harness/gen.py:46-59)."""
    rng = np.random.default_rng(seed)
    M = N * N
    x = tuple(rng.uniform(-X, X, P) for _ in range(3))
    s = tuple(rng.uniform(-S, S, M) for _ in range(3))
    a = rng.uniform(0.2, 1.0, P)
    th = rng.uniform(0, 2 * np.pi, P)
    return dict(x=x, c=a * np.exp(1j * th), s=s,
                meta=dict(N=N, P=P, X=X, S=S, seed=seed, geom="generic"))


def gen_anisotropic(N=1024, P=100_000, lat=1.5, seed=0):
    """Anisotropic type 3 with a large coordinate dynamic range: two wide
    source axes of order 1e7 against target extents of order 1e-4, and a
    thin third axis (harness/gen.py:15-43; the constants only set the
    per-axis dynamic ranges)."""
    rng = np.random.default_rng(seed)
    s0 = 520e-9
    k0 = 2.0 * np.pi / s0
    A = 7.17e-4
    u = rng.uniform(-lat, lat, P)
    v = rng.uniform(-lat, lat, P)
    d = rng.uniform(1.2, 6.0, P)
    tau = 1.0 / d
    amp = rng.uniform(0.2, 1.0, P)
    th = rng.uniform(0, 2 * np.pi, P)
    c = (amp * np.exp(1j * th) / (1j * s0 * d)
         * np.exp(1j * 0.5 * k0 * tau * (u * u + v * v))).astype(np.complex128)
    x = (-k0 * tau * v, -k0 * tau * u, 0.5 * k0 * tau)
    p = A / N
    r = (np.arange(N) - N / 2) * p
    GY, GX = np.meshgrid(r, r, indexing="ij")
    s = (GY.ravel(), GX.ravel(), (GX * GX + GY * GY).ravel())
    return dict(x=x, c=c, s=s,
                meta=dict(N=N, P=P, lat=lat, seed=seed, geom="anisotropic"))


def _cnormal(rng, shape, dtype):
    return (rng.standard_normal(shape) + 1j * rng.standard_normal(shape)).astype(dtype)


CONFIG_NAMES = {
    1: "2D type-1 M=1e5 N=256^2 eps=1e-6",
    2: "1D type-2 N=2^20 M=1e7 eps=1e-6",
    3: "3D type-1 batch n_trans=8 M=1e7 N=128^3 eps=1e-5",
    4: "3D type-2 clustered M=5e7 N=256^3 eps=1e-6",
    5: "3D type-3 1e6 sources -> 1e6 targets eps=1e-5",
    6: "expi 1e7 phases in [-1e6, 1e6]",
}


def config(k, scale=1.0, seed=0):
    """Benchmark workload k (1..5; 6 = the standalone expi of cfg 5; 7..12 =
    the reference's type-3 paper suite, PAPER_T3).

    Returns a dict with keys: type, dim, eps, isign, x (list of fp64
    coordinate arrays), data (strengths or modes), and n_modes / s / phi as
    applicable.  `scale` multiplies the point counts (tests use < 1)."""
    rng = np.random.default_rng(seed)

    def m(n):
        return max(1, int(round(n * scale)))

    if k == 1:
        # examples/quickstart.py:21-30 demo_basic, seed 0
        M = m(100_000)
        x = rng.uniform(-np.pi, np.pi, M)
        y = rng.uniform(-np.pi, np.pi, M)
        c = rng.standard_normal(M) + 1j * rng.standard_normal(M)
        return dict(type=1, dim=2, eps=1e-6, isign=+1, x=[x, y], data=c,
                    n_modes=(256, 256), name=CONFIG_NAMES[1])
    if k == 2:
        N = 1_048_576
        f = _cnormal(rng, N, np.complex64)
        M = m(10_000_000)
        x = rng.uniform(-np.pi, np.pi, M)
        return dict(type=2, dim=1, eps=1e-6, isign=-1, x=[x], data=f,
                    n_modes=(N,), name=CONFIG_NAMES[2])
    if k == 3:
        M = m(10_000_000)
        x = [rng.uniform(-np.pi, np.pi, M) for _ in range(3)]
        cs = _cnormal(rng, (8, M), np.complex64)
        return dict(type=1, dim=3, eps=1e-5, isign=+1, x=x, data=cs,
                    n_modes=(128, 128, 128), n_trans=8, name=CONFIG_NAMES[3])
    if k == 4:
        f = _cnormal(rng, (256, 256, 256), np.complex64)
        M = m(50_000_000)
        h = M // 2
        xu = [rng.uniform(-np.pi, np.pi, h) for _ in range(3)]
        xg = [np.mod(rng.normal(0.0, 0.3, M - h) + np.pi, 2 * np.pi) - np.pi
              for _ in range(3)]
        x = [np.concatenate([a, b]) for a, b in zip(xu, xg)]
        return dict(type=2, dim=3, eps=1e-6, isign=-1, x=x, data=f,
                    n_modes=(256, 256, 256), name=CONFIG_NAMES[4])
    if k == 5:
        P = m(1_000_000)
        Mt = m(1_000_000)
        x = [rng.uniform(-10, 10, P) for _ in range(3)]
        c = _cnormal(rng, P, np.complex64)
        s = [rng.uniform(-20, 20, Mt) for _ in range(3)]
        return dict(type=3, dim=3, eps=1e-5, isign=+1, x=x, data=c, s=s,
                    name=CONFIG_NAMES[5])
    if k == 6:
        n = m(10_000_000)
        return dict(type=0, phi=rng.uniform(-1e6, 1e6, n), isign=+1,
                    name=CONFIG_NAMES[6])
    if k in PAPER_T3:
        # the reference's type-3 acceptance / paper suite, 1e6 sources
        # (harness/run_acceptance.py:25-41, 99-128; mlx-nufft.pdf Table I)
        geom, N = PAPER_T3[k]
        P = m(1_000_000)
        prob = (gen_generic(N=N, P=P, seed=seed) if geom == "generic"
                else gen_anisotropic(N=N, P=P, lat=1.5, seed=seed))
        return dict(type=3, dim=3, eps=3e-5 if geom == "generic" else 1e-5,
                    isign=+1, x=list(prob["x"]), data=prob["c"],
                    s=list(prob["s"]),
                    name=f"3D type-3 {geom} N={N} ({N * N} targets) P=1e6")
    raise ValueError(f"unknown config {k}")


# bench configs 7..12: (geometry, N) of the reference's type-3 paper suite
PAPER_T3 = {7: ("generic", 512), 8: ("generic", 1024), 9: ("generic", 2048),
            10: ("anisotropic", 512), 11: ("anisotropic", 1024),
            12: ("anisotropic", 2048)}
