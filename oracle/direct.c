/* direct.c -- TEST INFRASTRUCTURE ONLY: exact fp64 direct NUFFT sum.
 *
 *   out[k] = sum_j c[j] exp(i * isign * sum_d s_d[k] x_d[j])
 *
 * The same sum as the reference's harness/gen.py:93-119 (direct_sum), any
 * dimension 1..3, parallel over targets with OpenMP.  Used by the parity
 * tests as the exact answer on target subsets of full-size problems, and
 * never by the product library.
 */
#include <math.h>
#include <stdint.h>

void oracle_direct_sum(int dim, int64_t M, const double* x0, const double* x1,
                       const double* x2, const double* cre, const double* cim,
                       int64_t N, const double* s0, const double* s1,
                       const double* s2, int isign, double* ore, double* oim) {
    const double sg = isign >= 0 ? 1.0 : -1.0;
#pragma omp parallel for schedule(dynamic, 4)
    for (int64_t k = 0; k < N; ++k) {
        const double a0 = s0[k];
        const double a1 = dim > 1 ? s1[k] : 0.0;
        const double a2 = dim > 2 ? s2[k] : 0.0;
        double sr = 0.0, si = 0.0;
        for (int64_t j = 0; j < M; ++j) {
            double ph = a0 * x0[j];
            if (dim > 1) ph += a1 * x1[j];
            if (dim > 2) ph += a2 * x2[j];
            const double sn = sin(sg * ph), cs = cos(sg * ph);
            sr += cre[j] * cs - cim[j] * sn;
            si += cre[j] * sn + cim[j] * cs;
        }
        ore[k] = sr;
        oim[k] = si;
    }
}
