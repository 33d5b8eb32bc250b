// deconv.cu -- fused mode-copy / deconvolution kernels and expi.
//
// crop (type 1, mlx_nufft/nd.py:416-435): FFT-ordered fine grid -> modeord=0
//   mode box, times the per-dimension correction 1/phihat(2 pi k / n).
// pad (type 2 nd.py:878-906, type 3 gpu_t3.py:629-651): mode box times the
//   correction into the zero-padded FFT-ordered fine grid (zeros written too,
//   so no separate memset pass).
// Both sweep the innermost (contiguous) dimension with consecutive threads,
// so every global access is coalesced; a CTA covers part of one long row or
// several whole short rows (RowSplit), so thin innermost dimensions do not
// leave most threads idle.  The outer-dimension correction factor is formed
// once per row.
//
// expi (mlx_nufft/dfmath.py:29-134): the reference forms the phase in
// double-single and reduces it mod 2 pi before fp32 cos/sin.  B200 has
// native fp64, so the components are summed in fp64 and reduced with a
// two-constant Cody-Waite step (2 pi = kTwoPi + kTwoPiLo, the product
// k * kTwoPi taken exactly by fma); the O(1) residual is split into a float
// pair and evaluated with sincosf plus a first-order correction for the low
// part.
#include <algorithm>

#include "internal.h"
#include "spreadinterp.cuh"   // NUFFT_DIM_SWITCH

namespace nufft {

struct DecPtrs {
    const float* d[3];
};

// Extents of a box and of the fine grid, innermost dimension last.
struct BoxGrid {
    int dim;
    int N[3];      // mode box (1 for unused leading dims)
    int n[3];      // fine grid
    int64_t K;     // prod N
    int64_t ncells;  // prod n
};

// Map an "outer" row index (all dims but the last) to per-dim indices.
// Kernels are templated on DIM so that every index is a compile-time
// constant (a runtime dimension count put these arrays, and the parameter
// structs they index, in local memory).
template <int DIM>
__device__ __forceinline__ void split_row(int64_t row, const BoxGrid& bg,
                                          bool modes, int (&idx)[3]) {
#pragma unroll
    for (int d = DIM - 2; d >= 0; --d) {
        const int ext = modes ? bg.N[d] : bg.n[d];
        idx[d] = (int)(row % ext);
        row /= ext;
    }
}

// Type-1 crop: fk[v][m] = grid[v][r(m)] * prod_d dec_d[m_d], with
// r_d = m_d - N_d/2 (+ n_d if negative).
__device__ __forceinline__ float2 to_f2(float2 v) { return v; }
__device__ __forceinline__ float2 to_f2(double2 v) {
    return make_float2((float)v.x, (float)v.y);
}

// Work split shared by crop and pad: a CTA covers `chunks` blocks of 256
// consecutive innermost elements of one row, or, when a row is shorter than
// the CTA, `rows` whole rows (so short innermost dimensions -- a thin axis
// of a type-3 grid -- still fill the CTA).  Element e of row `row`:
struct RowSplit {
    int per_row;     // elements (or element pairs) per row
    int rows;        // rows per CTA (>= 1)
    int chunks;      // CTAs per row (>= 1)
};

__device__ __forceinline__ bool row_elem(const RowSplit& rs, int64_t* row, int* e) {
    if (rs.rows > 1) {
        const int lr = (int)threadIdx.x / rs.per_row;
        *row = (int64_t)blockIdx.x * rs.rows + lr;
        *e = (int)threadIdx.x - lr * rs.per_row;
        return lr < rs.rows;
    }
    *row = blockIdx.x / rs.chunks;
    *e = (int)(blockIdx.x % rs.chunks) * blockDim.x + threadIdx.x;
    return *e < rs.per_row;
}

template <int DIM, typename G>
__global__ void __launch_bounds__(256)
k_crop(const G* __restrict__ grid, float2* __restrict__ fk, DecPtrs dec,
       BoxGrid bg, RowSplit rs, int64_t nrows) {
    constexpr int L = DIM - 1;                // innermost dim index
    int64_t row;
    int m_in;
    if (!row_elem(rs, &row, &m_in) || row >= nrows) return;
    const int v = blockIdx.y;
    int m[3] = {0, 0, 0};
    split_row<DIM>(row, bg, true, m);
    int64_t rrow = 0;
    float dout = 1.0f;
#pragma unroll
    for (int d = 0; d < L; ++d) {
        int r = m[d] - bg.N[d] / 2;
        if (r < 0) r += bg.n[d];
        rrow = rrow * bg.n[d] + r;
        dout = (d == 0) ? dec.d[0][m[0]] : dout * dec.d[d][m[d]];
    }
    int r = m_in - bg.N[L] / 2;
    if (r < 0) r += bg.n[L];
    const float dd = (L == 0) ? dec.d[0][m_in] : dout * dec.d[L][m_in];
    const float2 g = to_f2(grid[v * bg.ncells + rrow * bg.n[L] + r]);
    fk[v * bg.K + row * bg.N[L] + m_in] = make_float2(g.x * dd, g.y * dd);
}

__global__ void __launch_bounds__(256)
k_widen(const float2* __restrict__ in, double2* __restrict__ out, int64_t n) {
    const int64_t j = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
    if (j < n) {
        const float2 v = in[j];
        out[j] = make_double2(v.x, v.y);
    }
}

// Pad: H[v][r] = f[v][m(r)] * prod dec if every dim is in band, else 0.
// In-band test (nd.py:894-901): q = r - n if r >= n - N/2; band is
// -N/2 <= q < N - N/2; m = q + N/2.
// Each thread writes two consecutive fine cells with one 16-byte store
// (fine-grid extents are even, so rows stay 16-byte aligned).
__device__ __forceinline__ void store_pair(float2* p, float4 v) {
    *reinterpret_cast<float4*>(p) = v;
}
__device__ __forceinline__ void store_pair(double2* p, float4 v) {
    p[0] = make_double2(v.x, v.y);
    p[1] = make_double2(v.z, v.w);
}

template <int DIM, typename H_T>
__global__ void __launch_bounds__(256)
k_pad(const float2* __restrict__ f, H_T* __restrict__ H, DecPtrs dec,
      BoxGrid bg, RowSplit rs, int64_t nrows) {
    constexpr int L = DIM - 1;
    int64_t row;
    int pair;
    if (!row_elem(rs, &row, &pair) || row >= nrows) return;
    const int r0 = 2 * pair;
    const int v = blockIdx.y;
    int r[3] = {0, 0, 0};
    split_row<DIM>(row, bg, false, r);
    bool inband = true;
    int64_t mrow = 0;
    float dout = 1.0f;
#pragma unroll
    for (int d = 0; d < L; ++d) {
        int q = r[d];
        if (q >= bg.n[d] - bg.N[d] / 2) q -= bg.n[d];
        const int md = q + bg.N[d] / 2;
        inband &= (md >= 0) && (md < bg.N[d]);
        if (inband) {
            mrow = mrow * bg.N[d] + md;
            dout = (d == 0) ? dec.d[0][md] : dout * dec.d[d][md];
        }
    }
    float4 out = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    if (inband) {
        const float2* frow = f + v * bg.K + mrow * bg.N[L];
        const int lo = bg.n[L] - bg.N[L] / 2;     // first negative-mode cell
        int q0 = r0;
        if (q0 >= lo) q0 -= bg.n[L];
        const int m0 = q0 + bg.N[L] / 2;          // mode of cell r0
        const float* dl = dec.d[L];
        if (m0 >= 0 && m0 + 1 < bg.N[L] && r0 + 1 != lo &&
            (reinterpret_cast<uintptr_t>(frow + m0) & 15) == 0 &&
            (reinterpret_cast<uintptr_t>(dl + m0) & 7) == 0) {
            // both cells in band with consecutive modes whose addresses
            // are aligned (the caller's array may be 8-byte aligned only):
            // one 16-byte strength load, one 8-byte correction load
            const float4 g = __ldg(reinterpret_cast<const float4*>(frow + m0));
            float2 dd = __ldg(reinterpret_cast<const float2*>(dl + m0));
            if (L != 0) { dd.x *= dout; dd.y *= dout; }
            out = make_float4(g.x * dd.x, g.y * dd.x, g.z * dd.y, g.w * dd.y);
        } else {
#pragma unroll
            for (int e = 0; e < 2; ++e) {
                int q = r0 + e;
                if (q >= lo) q -= bg.n[L];
                const int mi = q + bg.N[L] / 2;
                if (mi >= 0 && mi < bg.N[L]) {
                    const float dd = (L == 0) ? __ldg(dl + mi) : dout * __ldg(dl + mi);
                    const float2 g = __ldg(frow + mi);
                    if (e == 0) { out.x = g.x * dd; out.y = g.y * dd; }
                    else        { out.z = g.x * dd; out.w = g.y * dd; }
                }
            }
        }
    }
    store_pair(H + v * bg.ncells + row * bg.n[L] + r0, out);
}

namespace {

BoxGrid make_boxgrid(int dim, const int64_t* N, const int64_t* n) {
    BoxGrid bg{};
    bg.dim = dim;
    bg.K = 1;
    bg.ncells = 1;
    for (int d = 0; d < 3; ++d) {
        bg.N[d] = d < dim ? (int)N[d] : 1;
        bg.n[d] = d < dim ? (int)n[d] : 1;
    }
    for (int d = 0; d < dim; ++d) {
        bg.K *= N[d];
        bg.ncells *= n[d];
    }
    return bg;
}

// CTAs and work split for rows of `per_row` elements (256 threads).
RowSplit make_split(int per_row, int64_t nrows, int64_t* blocks) {
    RowSplit rs{};
    rs.per_row = per_row;
    if (per_row <= 128) {
        rs.rows = 256 / per_row;
        rs.chunks = 1;
        *blocks = (nrows + rs.rows - 1) / rs.rows;
    } else {
        rs.rows = 1;
        rs.chunks = (per_row + 255) / 256;
        *blocks = nrows * rs.chunks;
    }
    return rs;
}

DecPtrs make_dec(const float* const* dec) {
    DecPtrs dp{};
    for (int d = 0; d < 3; ++d) dp.d[d] = dec[d];
    return dp;
}

}  // namespace

void launch_crop(int dim, const int64_t* N, const int64_t* n,
                 const float* const* dec, const void* grid, bool grid64,
                 float2* fk, int nvec, cudaStream_t st) {
    const BoxGrid bg = make_boxgrid(dim, N, n);
    const int inner = bg.N[dim - 1];
    const int64_t rows = bg.K / inner;
    int64_t blocks = 0;
    const RowSplit rs = make_split(inner, rows, &blocks);
    if (blocks > 0x7fffffffLL) fail(-1, "mode box too large");
    for (int v0 = 0; v0 < nvec; v0 += 65535) {
        const int nv = std::min(65535, nvec - v0);
        dim3 g((unsigned)blocks, (unsigned)nv);
        NUFFT_DIM_SWITCH(dim, {
            if (grid64)
                k_crop<DIM><<<g, 256, 0, st>>>((const double2*)grid + v0 * bg.ncells,
                                               fk + v0 * bg.K, make_dec(dec), bg, rs,
                                               rows);
            else
                k_crop<DIM><<<g, 256, 0, st>>>((const float2*)grid + v0 * bg.ncells,
                                               fk + v0 * bg.K, make_dec(dec), bg, rs,
                                               rows);
        });
        NUFFT_LAUNCH("k_crop");
    }
}

void launch_pad(int dim, const int64_t* N, const int64_t* n,
                const float* const* dec, const float2* f, void* H,
                bool grid64, int nvec, cudaStream_t st) {
    const BoxGrid bg = make_boxgrid(dim, N, n);
    const int inner = bg.n[dim - 1];
    if (inner % 2) fail(-1, "fine-grid extents must be even");
    const int64_t rows = bg.ncells / inner;
    int64_t blocks = 0;
    const RowSplit rs = make_split(inner / 2, rows, &blocks);
    if (blocks > 0x7fffffffLL) fail(-1, "fine grid too large");
    for (int v0 = 0; v0 < nvec; v0 += 65535) {
        const int nv = std::min(65535, nvec - v0);
        dim3 g((unsigned)blocks, (unsigned)nv);
        NUFFT_DIM_SWITCH(dim, {
            if (grid64)
                k_pad<DIM><<<g, 256, 0, st>>>(f + v0 * bg.K, (double2*)H + v0 * bg.ncells,
                                              make_dec(dec), bg, rs, rows);
            else
                k_pad<DIM><<<g, 256, 0, st>>>(f + v0 * bg.K, (float2*)H + v0 * bg.ncells,
                                              make_dec(dec), bg, rs, rows);
        });
        NUFFT_LAUNCH("k_pad");
    }
}

void launch_widen(const float2* in, double2* out, int64_t n, cudaStream_t st) {
    if (n <= 0) return;
    k_widen<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(in, out, n);
    NUFFT_LAUNCH("k_widen");
}

// ---------------------------------------------------------------------
constexpr int kMaxExpiComps = 64;
struct ExpiComps {
    const double* p[kMaxExpiComps];
};

__device__ __forceinline__ float2 expi_one(double phi, float sgn) {
    const double k = rint(phi * (1.0 / kTwoPi));
    double r = fma(-k, kTwoPi, phi);
    r = fma(-k, kTwoPiLo, r);
    const float hi = (float)r;
    const float lo = (float)(r - (double)hi);
    float s, c;
    sincosf(hi, &s, &c);
    const float sr = fmaf(c, lo, s);     // sin(hi + lo) to first order
    const float cr = fmaf(-s, lo, c);    // cos(hi + lo) to first order
    return make_float2(cr, sgn * sr);
}

// E (even) consecutive elements per thread: 16-byte loads per component
// and 16-byte stores (every component and the output 16-byte aligned); the
// elements past the last full group run one by one.
#ifndef NUFFT_EXPI_PER
#define NUFFT_EXPI_PER 4
#endif
constexpr int kExpiPer = NUFFT_EXPI_PER;

__global__ void __launch_bounds__(256)
k_expi2(ExpiComps comps, int ncomp, int64_t n, float sgn,
        float2* __restrict__ out) {
    constexpr int E = kExpiPer;
    const int64_t j = E * (blockIdx.x * (int64_t)blockDim.x + threadIdx.x);
    if (j >= n) return;
    if (j + E <= n) {
        double phi[E];
#pragma unroll
        for (int e = 0; e < E; ++e) phi[e] = 0.0;
        for (int c = 0; c < ncomp; ++c) {
#pragma unroll
            for (int e = 0; e < E; e += 2) {
                const double2 v =
                    __ldg(reinterpret_cast<const double2*>(comps.p[c] + j + e));
                phi[e] += v.x;
                phi[e + 1] += v.y;
            }
        }
#pragma unroll
        for (int e = 0; e < E; e += 2) {
            const float2 a = expi_one(phi[e], sgn), b = expi_one(phi[e + 1], sgn);
            *reinterpret_cast<float4*>(out + j + e) = make_float4(a.x, a.y, b.x, b.y);
        }
    } else {
        for (int64_t i = j; i < n; ++i) {
            double phi = 0.0;
            for (int c = 0; c < ncomp; ++c) phi += __ldg(comps.p[c] + i);
            out[i] = expi_one(phi, sgn);
        }
    }
}

__global__ void __launch_bounds__(256)
k_expi(ExpiComps comps, int ncomp, int64_t n, float sgn,
       float2* __restrict__ out) {
    const int64_t j = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
    if (j >= n) return;
    double phi = 0.0;
    for (int c = 0; c < ncomp; ++c) phi += __ldg(comps.p[c] + j);
    out[j] = expi_one(phi, sgn);
}

void launch_expi(int ncomp, const double* const* comps, int64_t n, int isign,
                 float2* out, cudaStream_t st) {
    if (ncomp < 1 || ncomp > kMaxExpiComps)
        fail(-1, "expi: between 1 and 64 phase components are supported");
    if (n <= 0) return;
    ExpiComps cp{};
    for (int c = 0; c < ncomp; ++c) cp.p[c] = comps[c];
    const float sgn = isign >= 0 ? 1.0f : -1.0f;
    bool aligned = (reinterpret_cast<uintptr_t>(out) & 15) == 0;
    for (int c = 0; c < ncomp; ++c)
        aligned &= (reinterpret_cast<uintptr_t>(comps[c]) & 15) == 0;
    if (aligned) {
        const int64_t blocks = ((n + kExpiPer - 1) / kExpiPer + 255) / 256;
        k_expi2<<<(unsigned)blocks, 256, 0, st>>>(cp, ncomp, n, sgn, out);
        NUFFT_LAUNCH("k_expi2");
    } else {
        const int64_t blocks = (n + 255) / 256;
        k_expi<<<(unsigned)blocks, 256, 0, st>>>(cp, ncomp, n, sgn, out);
        NUFFT_LAUNCH("k_expi");
    }
}

}  // namespace nufft
