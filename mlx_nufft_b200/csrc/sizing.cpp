// sizing.cpp -- host fp64 numerics of the NUFFT plan: kernel width/shape,
// fine-grid sizes and the kernel Fourier transform.  Each function restates
// the algorithm of the reference's mlx_nufft/sizing.py (itself FINUFFT's
// setup_spreader / set_nhg_type3) so that grid sizes and kernel shapes agree
// exactly with the reference.
#include <algorithm>
#include <cmath>
#include <vector>

#include "internal.h"

namespace nufft {

// Smallest even n' >= n whose prime factors are all in {2, 3, 5}.
// mlx_nufft/sizing.py:13-25
int64_t next235even(int64_t n) {
    if (n < 2) n = 2;
    if (n % 2) n += 1;
    for (;; n += 2) {
        int64_t m = n;
        while (m % 2 == 0) m /= 2;
        while (m % 3 == 0) m /= 3;
        while (m % 5 == 0) m /= 5;
        if (m == 1) return n;
    }
}

// ES width w and shape beta for tolerance eps at upsampling sigma.
// mlx_nufft/sizing.py:28-50
void kernel_params(double eps, double upsampfac, int* w, double* beta) {
    int ns;
    if (upsampfac == 2.0)
        ns = (int)std::ceil(-std::log10(eps / 10.0));
    else
        ns = (int)std::ceil(-std::log(eps) /
                            (kPi * std::sqrt(1.0 - 1.0 / upsampfac)));
    if (ns < 2) ns = 2;
    if (ns > 16) ns = 16;
    double betaoverns = 2.30;
    if (ns == 2) betaoverns = 2.20;
    else if (ns == 3) betaoverns = 2.26;
    else if (ns == 4) betaoverns = 2.38;
    if (upsampfac != 2.0)
        betaoverns = 0.97 * kPi * (1.0 - 1.0 / (2.0 * upsampfac));
    *w = ns;
    *beta = betaoverns * ns;
}

namespace {

// Gauss-Legendre nodes/weights on [-1, 1] (ascending nodes), by Newton's
// method on the three-term Legendre recurrence.
void gauss_legendre(int n, std::vector<double>* x, std::vector<double>* wt) {
    x->assign(n, 0.0);
    wt->assign(n, 0.0);
    for (int i = 0; i < (n + 1) / 2; ++i) {
        double z = std::cos(kPi * (i + 0.75) / (n + 0.5));
        double dp = 0.0;
        for (int it = 0; it < 100; ++it) {
            double p0 = 1.0, p1 = z;
            for (int k = 2; k <= n; ++k) {
                double p2 = ((2.0 * k - 1.0) * z * p1 - (k - 1.0) * p0) / k;
                p0 = p1;
                p1 = p2;
            }
            dp = n * (z * p1 - p0) / (z * z - 1.0);
            double dz = p1 / dp;
            z -= dz;
            if (std::fabs(dz) < 1e-16) break;
        }
        {   // weight from the converged node
            double p0 = 1.0, p1 = z;
            for (int k = 2; k <= n; ++k) {
                double p2 = ((2.0 * k - 1.0) * z * p1 - (k - 1.0) * p0) / k;
                p0 = p1;
                p1 = p2;
            }
            dp = n * (z * p1 - p0) / (z * z - 1.0);
        }
        double wi = 2.0 / ((1.0 - z * z) * dp * dp);
        (*x)[n - 1 - i] = z;
        (*x)[i] = -z;
        (*wt)[i] = wi;
        (*wt)[n - 1 - i] = wi;
    }
}

double es_kernel64(double d, double beta, int w) {
    double z = 2.0 * d / w;
    double z2 = z * z;
    if (z2 > 1.0) return 0.0;
    return std::exp(beta * (std::sqrt(1.0 - z2) - 1.0));
}

}  // namespace

// Nodes d_q in [0, w/2] and weights a_q (quadrature weight times kernel
// value) so that phihat(xi) = 2 * sum_q a_q cos(xi * d_q).
// mlx_nufft/sizing.py:74-85 (nquad = 128)
void kernel_ft_nodes(double beta, int w, std::vector<double>* d,
                     std::vector<double>* a) {
    const int nq = 128;
    std::vector<double> x, wt;
    gauss_legendre(nq, &x, &wt);
    d->resize(nq);
    a->resize(nq);
    for (int q = 0; q < nq; ++q) {
        (*d)[q] = 0.5 * (x[q] + 1.0) * (w / 2.0);
        (*a)[q] = wt[q] * (w / 4.0) * es_kernel64((*d)[q], beta, w);
    }
}

double kernel_ft(double xi, double beta, int w) {
    std::vector<double> d, a;
    kernel_ft_nodes(beta, w, &d, &a);
    double s = 0.0;
    for (size_t q = 0; q < d.size(); ++q) s += a[q] * std::cos(xi * d[q]);
    return 2.0 * s;
}

// Piecewise-polynomial form of the ES kernel used by the device kernels
// (the "Horner" evaluation of FINUFFT, Barnett, Magland & af Klinteberg,
// SIAM J. Sci. Comput. 41 (2019)): for a point with fraction fr in
// (w/2 - 1, w/2], tap l has weight psi(l - fr) = sum_k c[k][l] t^k with
// t = fr - (w/2 - 1/2) in (-1/2, 1/2].  Each tap's polynomial is the
// degree-`deg` interpolant at Chebyshev nodes of [-1/2, 1/2], computed in
// fp64 and converted to the monomial basis.  Its error is at the level of
// the kernel's edge value exp(-beta) (~3e-8 for w = 7), below the kernel's
// own truncation error.
void es_poly_coeffs(int w, double beta, int deg, float* coef) {
    const int n = deg + 1;
    std::vector<double> s(n), a(n), mono(n), Tm1(n), T(n), Tn(n);
    for (int i = 0; i < n; ++i) s[i] = std::cos(kPi * (i + 0.5) / n);
    for (int l = 0; l < w; ++l) {
        // Chebyshev coefficients of y(s) = psi(l - (w/2 - 1/2) - s/2)
        for (int j = 0; j < n; ++j) {
            double acc = 0.0;
            for (int i = 0; i < n; ++i) {
                const double d = l - (w / 2.0 - 0.5) - 0.5 * s[i];
                acc += es_kernel64(d, beta, w) * std::cos(j * kPi * (i + 0.5) / n);
            }
            a[j] = 2.0 / n * acc;
        }
        a[0] *= 0.5;
        // sum_j a_j T_j(s) in the monomial basis of s
        std::fill(mono.begin(), mono.end(), 0.0);
        std::fill(Tm1.begin(), Tm1.end(), 0.0);
        std::fill(T.begin(), T.end(), 0.0);
        Tm1[0] = 1.0;
        mono[0] = a[0];
        if (n > 1) {
            T[1] = 1.0;
            mono[1] += a[1];
        }
        for (int j = 2; j < n; ++j) {
            std::fill(Tn.begin(), Tn.end(), 0.0);
            for (int k = 0; k + 1 < n; ++k) Tn[k + 1] = 2.0 * T[k];
            for (int k = 0; k < n; ++k) Tn[k] -= Tm1[k];
            for (int k = 0; k < n; ++k) mono[k] += a[j] * Tn[k];
            Tm1.swap(T);
            T.swap(Tn);
        }
        // s = 2t
        double scale = 1.0;
        for (int k = 0; k < n; ++k) {
            coef[k * w + l] = (float)(mono[k] * scale);
            scale *= 2.0;
        }
    }
}

EsPoly make_es_poly(int w, double beta) {
    EsPoly p{};
    if (w < 2 || w > kMaxW) return p;
    const int deg = es_degree(w);
    std::vector<float> c((size_t)(deg + 1) * w);
    es_poly_coeffs(w, beta, deg, c.data());
    for (int k = 0; k <= deg; ++k)
        for (int l = 0; l < w; ++l) p.c[k][l] = c[(size_t)k * w + l];
    return p;
}

// Type-3 spread-grid size nf, spacing h and scale gam for one dimension.
// mlx_nufft/sizing.py:88-111
void set_nhg_type3(double S, double X, double upsampfac, int w, int64_t* nf,
                   double* h, double* gam) {
    int nss = w + 1;
    double Xsafe = X, Ssafe = S;
    if (X == 0.0) {
        if (S == 0.0) {
            Xsafe = 1.0;
            Ssafe = 1.0;
        } else {
            Xsafe = std::max(Xsafe, 1.0 / S);
        }
    } else {
        Ssafe = std::max(Ssafe, 1.0 / X);
    }
    double nfd = 2.0 * upsampfac * Ssafe * Xsafe / kPi + nss;
    int64_t n = (int64_t)nfd;
    if (n < 2 * w) n = 2 * w;
    n = next235even(n);
    *nf = n;
    *h = 2.0 * kPi / n;
    *gam = n / (2.0 * upsampfac * Ssafe);
}

}  // namespace nufft
