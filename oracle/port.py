"""numpy restatement of the reference's CPU NUFFT algorithms (fp64 oracle).

TEST INFRASTRUCTURE ONLY (see oracle/__init__.py).  Each function cites the
reference file:line it restates.  The type-1/2 pipelines have no CPU
counterpart in the reference (it validates them against CPU finufft, which
is not installed); they restate the reference's GPU pipeline conventions
(mlx_nufft/nd.py) with every stage in fp64, in the structure of the
reference's own CPU type-3 oracle (mlx_nufft/ref_t3.py:156-221).
"""

import numpy as np

PI = np.pi


# --------------------------------------------------------------------------
# sizing -- mlx_nufft/sizing.py

def next235even(n):
    """sizing.py:13-25"""
    n = max(int(n), 2)
    if n % 2:
        n += 1
    while True:
        m = n
        for p in (2, 3, 5):
            while m % p == 0:
                m //= p
        if m == 1:
            return n
        n += 2


def kernel_params(eps, upsampfac):
    """sizing.py:28-50"""
    if upsampfac == 2.0:
        ns = int(np.ceil(-np.log10(eps / 10.0)))
    else:
        ns = int(np.ceil(-np.log(eps) / (PI * np.sqrt(1.0 - 1.0 / upsampfac))))
    ns = max(2, min(ns, 16))
    b = {2: 2.20, 3: 2.26, 4: 2.38}.get(ns, 2.30)
    if upsampfac != 2.0:
        b = 0.97 * PI * (1.0 - 1.0 / (2.0 * upsampfac))
    return ns, b * ns


def es_kernel(d, beta, w):
    """sizing.py:53-65: exp(beta (sqrt(1 - (2d/w)^2) - 1)), 0 outside."""
    z2 = (2.0 * np.asarray(d, dtype=np.float64) / w) ** 2
    out = np.zeros_like(z2)
    inside = z2 <= 1.0
    out[inside] = np.exp(beta * (np.sqrt(1.0 - z2[inside]) - 1.0))
    return out


def kernel_ft(xi, beta, w, nquad=128):
    """sizing.py:74-85: 2 * int_0^{w/2} psi(d) cos(xi d) dd, Gauss-Legendre."""
    xi = np.atleast_1d(np.asarray(xi, dtype=np.float64))
    nodes, weights = np.polynomial.legendre.leggauss(nquad)
    d = 0.5 * (nodes + 1.0) * (w / 2.0)
    wq = weights * (w / 4.0)
    return 2.0 * (wq * es_kernel(d, beta, w)) @ np.cos(np.outer(d, xi))


def set_nhg_type3(S, X, upsampfac, w):
    """sizing.py:88-111"""
    nss = w + 1
    Xsafe, Ssafe = X, S
    if X == 0.0:
        if S == 0.0:
            Xsafe, Ssafe = 1.0, 1.0
        else:
            Xsafe = max(Xsafe, 1.0 / S)
    else:
        Ssafe = max(Ssafe, 1.0 / X)
    nf = int(2.0 * upsampfac * Ssafe * Xsafe / PI + nss)
    if nf < 2 * w:
        nf = 2 * w
    nf = next235even(nf)
    return nf, 2.0 * PI / nf, nf / (2.0 * upsampfac * Ssafe)


def fine_grid_sizes(N, eps, upsampfac=2.0):
    """n_up per dimension for types 1/2 (nd.py:120-125)."""
    w, beta = kernel_params(eps, upsampfac)
    return w, beta, [next235even(max(2 * w, int(np.ceil(upsampfac * n))))
                     for n in N]


# --------------------------------------------------------------------------
# crit64 cell / fraction split

def cells_fold(x, n_up, w, prec="crit64"):
    """Type-1/2 cells (nd.py:152-165): xi = mod(x, 2pi)/h, i1 = ceil(xi - w/2),
    fr = xi - i1 (returned in fp64 and as the fp32 the GPU stores)."""
    rdt = np.float64 if prec == "crit64" else np.float32
    h = 2.0 * PI / n_up
    xi = np.mod(np.asarray(x, dtype=np.float64), 2.0 * PI).astype(rdt) / rdt(h)
    i1 = np.ceil(xi - rdt(w / 2.0)).astype(np.int32)
    fr64 = (xi - i1.astype(rdt)).astype(np.float64)
    return i1, fr64, fr64.astype(np.float32)


def normalize_cells(i1, n, w):
    """Shift i1 by a multiple of n so i1 + w//2 is in [0, n) (periodic grid;
    the device stores this form)."""
    b = np.mod(i1.astype(np.int64) + w // 2, n)
    return (b - w // 2).astype(np.int32)


# --------------------------------------------------------------------------
# fp64 spread / interp on a periodic grid

def _weights(fr, w, beta):
    l = np.arange(w, dtype=np.float64)
    return es_kernel(l[None, :] - np.asarray(fr, dtype=np.float64)[:, None],
                     beta, w)


def spread(i1s, frs, c, n, w, beta, chunk=4096):
    """sum_j c_j prod_d psi(l_d - fr_jd) onto cells (i1_jd + l_d) mod n_d."""
    dim = len(n)
    ncell = int(np.prod(n))
    gre = np.zeros(ncell)
    gim = np.zeros(ncell)
    c = np.asarray(c, dtype=np.complex128)
    for a0 in range(0, c.size, chunk):
        sl = slice(a0, min(a0 + chunk, c.size))
        vals = c[sl]
        flat = np.zeros(vals.size, dtype=np.int64)
        wt = np.ones(vals.size)
        for d in range(dim):
            W = _weights(frs[d][sl], w, beta)                     # (m, w)
            I = np.mod(i1s[d][sl, None].astype(np.int64) + np.arange(w), n[d])
            flat = flat.reshape(flat.shape + (1,)) * n[d] + I.reshape(
                (I.shape[0],) + (1,) * d + (w,))
            wt = wt.reshape(wt.shape + (1,)) * W.reshape(
                (W.shape[0],) + (1,) * d + (w,))
        v = vals.reshape((-1,) + (1,) * dim) * wt
        gre += np.bincount(flat.ravel(), weights=v.real.ravel(), minlength=ncell)
        gim += np.bincount(flat.ravel(), weights=v.imag.ravel(), minlength=ncell)
    return (gre + 1j * gim).reshape(n)


def interp(G, i1s, frs, w, beta, chunk=4096):
    """out_j = sum_taps G[(i1 + l) mod n] prod_d psi(l_d - fr_jd)."""
    n = G.shape
    dim = len(n)
    M = len(i1s[0])
    out = np.zeros(M, dtype=np.complex128)
    Gf = G.ravel()
    for a0 in range(0, M, chunk):
        sl = slice(a0, min(a0 + chunk, M))
        m = sl.stop - sl.start
        flat = np.zeros(m, dtype=np.int64)
        wt = np.ones(m)
        for d in range(dim):
            W = _weights(frs[d][sl], w, beta)
            I = np.mod(i1s[d][sl, None].astype(np.int64) + np.arange(w), n[d])
            flat = flat.reshape(flat.shape + (1,)) * n[d] + I.reshape(
                (m,) + (1,) * d + (w,))
            wt = wt.reshape(wt.shape + (1,)) * W.reshape((m,) + (1,) * d + (w,))
        out[sl] = (Gf[flat] * wt).reshape(m, -1).sum(axis=1)
    return out


def _fft(H, isign):
    if isign > 0:
        return np.fft.ifftn(H) * float(np.prod(H.shape))
    return np.fft.fftn(H)


def _band(N, n):
    """FFT-order fine-grid index of modes k in [-N//2, N - N//2)."""
    k = np.arange(-(N // 2), N - N // 2)
    return np.mod(k, n)


# --------------------------------------------------------------------------
# types 1 / 2 (conventions of nd.py, all stages fp64)

def nufft_t1(x, c, N, eps, isign=+1, upsampfac=2.0):
    """f[k] = sum_j c_j exp(i isign k.x_j), modeord=0 (nd.py:581-625)."""
    x = [np.asarray(v, dtype=np.float64).ravel() for v in x]
    N = tuple(int(v) for v in N)
    w, beta, nup = fine_grid_sizes(N, eps, upsampfac)
    i1s, frs = [], []
    for d in range(len(x)):
        i1, fr64, _ = cells_fold(x[d], nup[d], w)
        i1s.append(i1)
        frs.append(fr64)
    G = spread(i1s, frs, c, nup, w, beta)
    V = _fft(G, isign)
    out = V[np.ix_(*[_band(N[d], nup[d]) for d in range(len(N))])]
    for d in range(len(N)):
        k = np.arange(-(N[d] // 2), N[d] - N[d] // 2, dtype=np.float64)
        dec = 1.0 / kernel_ft(2.0 * PI * k / nup[d], beta, w)
        out = out * dec.reshape((1,) * d + (-1,) + (1,) * (len(N) - d - 1))
    return out


def nufft_t2(x, f, eps, isign=-1, upsampfac=2.0):
    """c_j = sum_k f[k] exp(i isign k.x_j), modeord=0 (nd.py:1075-1119)."""
    x = [np.asarray(v, dtype=np.float64).ravel() for v in x]
    f = np.asarray(f, dtype=np.complex128)
    N = f.shape
    w, beta, nup = fine_grid_sizes(N, eps, upsampfac)
    g = f.copy()
    for d in range(len(N)):
        k = np.arange(-(N[d] // 2), N[d] - N[d] // 2, dtype=np.float64)
        dec = 1.0 / kernel_ft(2.0 * PI * k / nup[d], beta, w)
        g = g * dec.reshape((1,) * d + (-1,) + (1,) * (len(N) - d - 1))
    H = np.zeros(nup, dtype=np.complex128)
    H[np.ix_(*[_band(N[d], nup[d]) for d in range(len(N))])] = g
    V = _fft(H, isign)
    i1s, frs = [], []
    for d in range(len(x)):
        i1, fr64, _ = cells_fold(x[d], nup[d], w)
        i1s.append(i1)
        frs.append(fr64)
    return interp(V, i1s, frs, w, beta)


# --------------------------------------------------------------------------
# type 3 (ref_t3.py:53-221 with FULL64 flags, any dimension)

class T3Geometry:
    """Sizing, cells and phases of the reference's type-3 plan
    (ref_t3.py:53-153; gpu_t3.py:288-441, 474-493 for the device layout)."""

    def __init__(self, x, s, eps=1e-5, isign=+1, upsampfac=1.25,
                 source_extent=None):
        x = [np.asarray(v, dtype=np.float64).ravel() for v in x]
        s = [np.asarray(v, dtype=np.float64).ravel() for v in s]
        self.dim = len(x)
        self.isign = +1 if isign >= 0 else -1
        self.w, self.beta = kernel_params(eps, upsampfac)
        w = self.w
        self.nf, self.h, self.gam, self.C, self.D = [], [], [], [], []
        for d in range(self.dim):
            if source_extent is not None:
                xlo, xhi = map(float, source_extent[d])
            else:
                xlo, xhi = float(x[d].min()), float(x[d].max())
            self.C.append(0.5 * (xlo + xhi))
            self.D.append(0.5 * (s[d].min() + s[d].max()))
            X = 0.5 * (xhi - xlo)
            S = 0.5 * (s[d].max() - s[d].min())
            nf, h, gam = set_nhg_type3(S, X, upsampfac, w)
            self.nf.append(nf)
            self.h.append(h)
            self.gam.append(gam)
        self.n_up = [next235even(int(np.ceil(upsampfac * nf))) for nf in self.nf]
        # sources: xi = (x - C)/gam/h + nf/2
        self.i1, self.fr = [], []
        for d in range(self.dim):
            xi = (x[d] - self.C[d]) / self.gam[d] / self.h[d] + self.nf[d] / 2.0
            i1 = np.ceil(xi - w / 2.0).astype(np.int64)
            self.i1.append(i1)
            self.fr.append(xi - i1)
        # targets: theta = (s - D) h gam ; lam = theta/(2pi/n_up) + n_up/2
        self.t_i1, self.t_fr, self.theta = [], [], []
        for d in range(self.dim):
            th = (s[d] - self.D[d]) * (self.h[d] * self.gam[d])
            self.theta.append(th)
            lam = th / (2.0 * PI / self.n_up[d]) + self.n_up[d] / 2.0
            i1 = np.ceil(lam - w / 2.0).astype(np.int64)
            self.t_i1.append(i1)
            self.t_fr.append(lam - i1)
        pre = sum(self.D[d] * x[d] for d in range(self.dim))
        post = sum(self.C[d] * (s[d] - self.D[d]) for d in range(self.dim))
        self.prephase = np.exp(1j * self.isign * pre)
        tdec = np.ones(s[0].size)
        for d in range(self.dim):
            tdec *= kernel_ft(self.theta[d], self.beta, w)
        self.post = np.exp(1j * self.isign * post) / tdec
        self.mode_dec = []
        for d in range(self.dim):
            q = np.arange(-self.nf[d] // 2, self.nf[d] // 2, dtype=np.float64)
            self.mode_dec.append(((-1.0) ** np.abs(q)) /
                                 kernel_ft(2.0 * PI * q / self.n_up[d],
                                           self.beta, w))


def nufft_t3(x, c, s, eps=1e-5, isign=+1, upsampfac=1.25, geom=None):
    """f_k = sum_j c_j exp(i isign s_k.x_j) by the reference's type-3
    algorithm in fp64 (ref_t3.py:156-221)."""
    g = geom or T3Geometry(x, s, eps, isign, upsampfac)
    cp = np.asarray(c, dtype=np.complex128) * g.prephase
    B = spread(g.i1, g.fr, cp, g.nf, g.w, g.beta)
    dec = np.ones(g.nf)
    for d in range(g.dim):
        dec = dec * g.mode_dec[d].reshape((1,) * d + (-1,) + (1,) * (g.dim - d - 1))
    H = np.zeros(g.n_up, dtype=np.complex128)
    H[np.ix_(*[np.mod(np.arange(-g.nf[d] // 2, g.nf[d] // 2), g.n_up[d])
               for d in range(g.dim)])] = B * dec
    V = _fft(H, g.isign)
    return interp(V, g.t_i1, g.t_fr, g.w, g.beta) * g.post


def _kernel_1d_f32(fr, w, beta):
    """ref_t3.py:140-154 with dtype float32: the fp32 ES weights."""
    f32 = np.float32
    l = np.arange(w, dtype=f32)
    d = l[None, :] - np.asarray(fr, dtype=f32)[:, None]
    z2 = (f32(2.0 / w) * d) ** 2
    out = np.exp(f32(beta) * (np.sqrt(np.maximum(f32(1.0) - z2, f32(0.0)))
                              - f32(1.0)))
    out[z2 > 1.0] = 0.0
    return out


def nufft_t3_fp32(x, c, s, eps=1e-5, isign=+1, upsampfac=1.25, chunk=2048):
    """The reference's fp32 type-3 pipeline with crit64 geometry: fp64
    coordinates and phases, fp32 spread / FFT / interp / deconvolution
    (ref_t3.py:156-221 executed with Flags(coords64=True, phases64=True,
    spread64=False, fft64=False, interp64=False, deconv64=False)).  Its
    error against the exact sum is the accuracy floor an fp32 device
    pipeline of this algorithm has on the given inputs."""
    g = T3Geometry(x, s, eps, isign, upsampfac)
    dim, w = g.dim, g.w
    cp = (np.asarray(c, dtype=np.complex128) * g.prephase).astype(np.complex64)
    fr = [v.astype(np.float32) for v in g.fr]
    B = np.zeros(int(np.prod(g.nf)), dtype=np.complex64)
    P = cp.size
    for a0 in range(0, P, chunk):
        sl = slice(a0, min(a0 + chunk, P))
        m = sl.stop - sl.start
        vals = cp[sl].reshape((m,) + (1,) * dim)
        flat = np.zeros((m,) + (1,) * dim, dtype=np.int64)
        for d in range(dim):
            shp = (m,) + (1,) * d + (w,) + (1,) * (dim - d - 1)
            vals = vals * _kernel_1d_f32(fr[d][sl], w, g.beta).reshape(shp)
            idx = (g.i1[d][sl, None] + np.arange(w)) % g.nf[d]
            flat = flat * g.nf[d] + idx.reshape(shp)
        np.add.at(B, flat.ravel(), vals.ravel())
    B = B.reshape(g.nf)
    dec = np.ones(g.nf, dtype=np.float32)
    for d in range(dim):
        dec = dec * g.mode_dec[d].astype(np.float32).reshape(
            (1,) * d + (-1,) + (1,) * (dim - d - 1))
    H = np.zeros(g.n_up, dtype=np.complex64)
    H[np.ix_(*[np.mod(np.arange(-g.nf[d] // 2, g.nf[d] // 2), g.n_up[d])
               for d in range(dim)])] = (B * dec).astype(np.complex64)
    if g.isign > 0:
        V = np.fft.ifftn(H) * int(np.prod(g.n_up))
    else:
        V = np.fft.fftn(H)
    V = V.astype(np.complex64).ravel()
    t_fr = [v.astype(np.float32) for v in g.t_fr]
    M = g.t_i1[0].size
    out = np.zeros(M, dtype=np.complex64)
    for a0 in range(0, M, chunk):
        sl = slice(a0, min(a0 + chunk, M))
        m = sl.stop - sl.start
        wgt = np.ones((m,) + (1,) * dim, dtype=np.float32)
        flat = np.zeros((m,) + (1,) * dim, dtype=np.int64)
        for d in range(dim):
            shp = (m,) + (1,) * d + (w,) + (1,) * (dim - d - 1)
            wgt = wgt * _kernel_1d_f32(t_fr[d][sl], w, g.beta).reshape(shp)
            idx = (g.t_i1[d][sl, None] + np.arange(w)) % g.n_up[d]
            flat = flat * g.n_up[d] + idx.reshape(shp)
        out[sl] = (V[flat] * wgt).sum(axis=tuple(range(1, dim + 1)))
    return out * g.post.astype(np.complex64)


# --------------------------------------------------------------------------
# exact direct sums (harness/gen.py:93-119) and error metric (gen.py:122-125)

def direct_sum(x, c, s, isign=+1, idx=None, chunk=None):
    """f[k] = sum_j c_j exp(i isign s_k . x_j) in fp64, any dimension."""
    x = [np.asarray(v, dtype=np.float64).ravel() for v in x]
    s = [np.asarray(v, dtype=np.float64).ravel() for v in s]
    if idx is not None:
        s = [v[idx] for v in s]
    c = np.asarray(c, dtype=np.complex128).ravel()
    M = s[0].size
    if chunk is None:
        chunk = max(8, int(2e7 / max(x[0].size, 1)))
    out = np.empty(M, dtype=np.complex128)
    for a0 in range(0, M, chunk):
        sl = slice(a0, min(a0 + chunk, M))
        ph = sum(np.outer(s[d][sl], x[d]) for d in range(len(x)))
        out[sl] = np.exp(1j * isign * ph) @ c
    return out


def mode_lattice(N, idx=None):
    """Integer mode coordinates k_d (modeord=0, C order) as 'targets'."""
    grids = np.meshgrid(*[np.arange(-(n // 2), n - n // 2) for n in N],
                        indexing="ij")
    ks = [g.ravel().astype(np.float64) for g in grids]
    if idx is not None:
        ks = [k[idx] for k in ks]
    return ks


def direct_t1(x, c, N, isign=+1, idx=None):
    """Exact type 1 at (a subset of) the modes, flat C-order."""
    return direct_sum(x, c, mode_lattice(N, idx), isign)


def direct_t2(x, f, isign=-1, idx=None):
    """Exact type 2 at (a subset of) the points."""
    f = np.asarray(f)
    ks = mode_lattice(f.shape)
    xs = [np.asarray(v, dtype=np.float64).ravel() for v in x]
    if idx is not None:
        xs = [v[idx] for v in xs]
    return direct_sum(ks, f.ravel(), xs, isign)


def rel_l2(u, ref):
    u = np.asarray(u).ravel()
    ref = np.asarray(ref).ravel()
    return float(np.linalg.norm(u - ref) / np.linalg.norm(ref))


def expi_ref(phi, isign=1):
    """fp64 host reference of expi (harness/test_expi.py:34-37)."""
    return np.exp(1j * (1 if isign >= 0 else -1) * np.asarray(phi, dtype=np.float64))
