// points.cu -- device setpts: coordinate rescale to (cell, fraction),
// counting-sort by bin, subproblem tables, and the type-3 pre/post phases.
//
// The reference does this on the host in numpy fp64 ("crit64",
// mlx_nufft/nd.py:152-181, 298-372; mlx_nufft/gpu_t3.py:344-377, 474-501)
// or with a double-single Metal kernel plus mx.argsort (nd.py:43-91,
// 191-243; gpu_t3.py:237-276, 508-555).  B200 has native fp64, so every
// rescale below is the reference's fp64 expression evaluated with the same
// operations in the same order (IEEE-exact fmod, correctly rounded + - * /,
// ceil), which makes the cell index bit-identical to the host fp64 path.
// The sort is a counting sort: one atomic histogram pass that also records
// each point's rank inside its bin, an exclusive scan of the bin counts,
// and a scatter -- O(M) with two coalesced reads of the coordinates.
#include <algorithm>
#include <utility>
#include <cmath>
#include <cstdio>
#include <cstdlib>

#include "internal.h"

namespace nufft {

struct Coords {
    const double* p[3];
};

// (i1, fr) of coordinate x in dimension d, plus the bin-normalised cell
// index: i1 is shifted by a multiple of the grid size so that
// i1 + w/2 lies in [0, n) (the grid is periodic, so this changes no tap).
__device__ __forceinline__ void cell_of(const CellParams& cp, int d, double x,
                                        int* i1n, float* fr, int* ib,
                                        bool* bad) {
    if (!isfinite(x)) {
        *bad = true;
        x = 0.0;
    }
    int i1;
    if (cp.kind == CELL_FOLD) {
        // xi = mod(x, 2pi) / h ; numpy's float mod: fmod, then + 2pi when
        // the remainder is negative (nd.py:162)
        double r = fmod(x, kTwoPi);
        if (r < 0.0) r += kTwoPi;
        if (!cp.fp32) {
            double xi = r / cp.h[d];
            double i1d = ceil(xi - cp.halfw_d);
            i1 = (int)i1d;
            *fr = (float)(xi - i1d);
        } else {
            float xi = (float)r / (float)cp.h[d];
            float i1f = ceilf(xi - (float)cp.halfw_d);
            i1 = (int)i1f;
            *fr = xi - i1f;
        }
    } else if (cp.kind == CELL_T3SRC) {
        // xi = (x - C) / gam / h + nf/2  (gpu_t3.py:486-490)
        if (!cp.fp32) {
            double xi = (x - cp.a[d]) / cp.b[d] / cp.h[d] + cp.c[d];
            double i1d = ceil(xi - cp.halfw_d);
            i1 = (int)i1d;
            *fr = (float)(xi - i1d);
        } else {
            float xi = ((float)x - (float)cp.a[d]) / (float)cp.b[d] /
                           (float)cp.h[d] + (float)cp.c[d];
            float i1f = ceilf(xi - (float)cp.halfw_d);
            i1 = (int)i1f;
            *fr = xi - i1f;
        }
    } else {
        // theta = (s - D) * (h*gam); lam = theta / (2pi/n_up) + n_up/2
        // (gpu_t3.py:357-366)
        if (!cp.fp32) {
            double th = (x - cp.a[d]) * cp.b[d];
            double lam = th / cp.c[d] + cp.e[d];
            double i1d = ceil(lam - cp.halfw_d);
            i1 = (int)i1d;
            *fr = (float)(lam - i1d);
        } else {
            float th = ((float)x - (float)cp.a[d]) * (float)cp.b[d];
            float lam = th / (float)cp.c[d] + (float)cp.e[d];
            float i1f = ceilf(lam - (float)cp.halfw_d);
            i1 = (int)i1f;
            *fr = lam - i1f;
        }
    }
    // periodic normalisation for binning
    int64_t n = cp.n[d];
    int64_t b = ((int64_t)i1 + cp.halfw) % n;
    if (b < 0) b += n;
    *ib = (int)b;
    *i1n = (int)(b - cp.halfw);
}

template <int DIM>
__global__ void k_cells_direct(int64_t M, Coords X, CellParams cp, int2* c0,
                               int2* c1, int2* c2, int* err) {
    int64_t j = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
    if (j >= M) return;
    bool bad = false;
    int2* out[3] = {c0, c1, c2};
#pragma unroll
    for (int d = 0; d < DIM; ++d) {
        int i1, ib;
        float fr;
        cell_of(cp, d, X.p[d][j], &i1, &fr, &ib, &bad);
        out[d][j] = make_int2(i1, __float_as_int(fr));
    }
    if (bad) atomicOr(err, 1);
}

template <int DIM>
__global__ void k_bin_count(int64_t M, Coords X, CellParams cp,
                            uint32_t* key_of, uint32_t* rank_of,
                            uint32_t* count, int* err) {
    int64_t j = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
    if (j >= M) return;
    bool bad = false;
    uint32_t key = cp.chunk ? (uint32_t)(j / cp.chunk) : 0u;
#pragma unroll
    for (int d = 0; d < DIM; ++d) {
        int i1, ib;
        float fr;
        cell_of(cp, d, X.p[d][j], &i1, &fr, &ib, &bad);
        key = key * (uint32_t)cp.nb[d] + (uint32_t)(ib / cp.m[d]);
    }
    if (bad) atomicOr(err, 1);
    key_of[j] = key;
    rank_of[j] = atomicAdd(&count[key], 1u);
}

template <int DIM>
__global__ void k_bin_scatter(int64_t M, Coords X, CellParams cp,
                              const uint32_t* key_of, const uint32_t* rank_of,
                              const uint32_t* start, int2* c0, int2* c1,
                              int2* c2, uint32_t* perm) {
    int64_t j = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
    if (j >= M) return;
    bool bad = false;
    uint32_t pos = start[key_of[j]] + rank_of[j];
    int2* out[3] = {c0, c1, c2};
#pragma unroll
    for (int d = 0; d < DIM; ++d) {
        int i1, ib;
        float fr;
        cell_of(cp, d, X.p[d][j], &i1, &fr, &ib, &bad);
        out[d][pos] = make_int2(i1, __float_as_int(fr));
    }
    perm[pos] = (uint32_t)j;
}

// Single-CTA exclusive scan (uint32, in place allowed) with the total in
// *total.  Only used at setpts time on bin / subproblem counts.
__global__ void __launch_bounds__(1024)
k_scan(const uint32_t* in, uint32_t* out, int64_t n, uint32_t* total) {
    __shared__ uint32_t sums[1024];
    const int t = threadIdx.x;
    const int64_t chunk = (n + 1023) / 1024;
    const int64_t b = t * chunk;
    const int64_t e = min(n, b + chunk);
    uint32_t s = 0;
    for (int64_t i = b; i < e; ++i) s += in[i];
    sums[t] = s;
    __syncthreads();
    for (int off = 1; off < 1024; off <<= 1) {
        uint32_t v = (t >= off) ? sums[t - off] : 0u;
        __syncthreads();
        sums[t] += v;
        __syncthreads();
    }
    uint32_t run = t ? sums[t - 1] : 0u;
    for (int64_t i = b; i < e; ++i) {
        uint32_t v = in[i];
        out[i] = run;
        run += v;
    }
    if (t == 1023) *total = sums[1023];
}

__global__ void k_sub_count(const uint32_t* count, int64_t nbins, int msub,
                            uint32_t* nsubs) {
    int64_t b = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
    if (b >= nbins) return;
    nsubs[b] = (count[b] + (uint32_t)msub - 1u) / (uint32_t)msub;
}

// Full (msub-point) and partial subproblems of each sort key.
__global__ void k_sub_split(const uint32_t* count, int64_t nbins, int msub,
                            uint32_t* nfull, uint32_t* npart) {
    int64_t b = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
    if (b >= nbins) return;
    nfull[b] = count[b] / (uint32_t)msub;
    npart[b] = (count[b] % (uint32_t)msub) != 0u ? 1u : 0u;
}

// Subproblem table: one entry per <= msub points of a sort key; the entry
// carries the spatial bin (key mod the number of spatial bins).  With
// partofs (interpolation point sets) the full subproblems come first (in
// key order, at fullofs[b]), then the partial ones (at *nfull_total +
// partofs[b]): the persistent kernels take subproblems in table order, so
// the longest ones (a dense bin's msub-point pieces) start early instead of
// running alone at the end of a launch.  Without it (spreading, whose tile
// flushes of neighbouring bins share L2 lines) the table is in key order,
// bin b's subproblems at fullofs[b] on.
__global__ void k_sub_fill(const uint32_t* count, const uint32_t* start,
                           const uint32_t* fullofs, const uint32_t* partofs,
                           const uint32_t* nfull_total, int64_t nbins,
                           int64_t nbins_spatial, int msub, int4* subs) {
    int64_t b = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
    if (b >= nbins) return;
    const uint32_t n = count[b];
    const uint32_t nf = n / (uint32_t)msub;
    const int spatial = (int)(b % nbins_spatial);
    for (uint32_t k = 0; k * (uint32_t)msub < n; ++k) {
        const uint32_t s = start[b] + k * (uint32_t)msub;
        const uint32_t c = min((uint32_t)msub, n - k * (uint32_t)msub);
        const uint32_t pos = (!partofs || k < nf) ? fullofs[b] + k
                                                  : *nfull_total + partofs[b];
        subs[pos] = make_int4((int)s, (int)c, spatial, 0);
    }
}

// Block-wide exclusive scan of a[0..n) in place (a CTA of 256 threads, each
// owning a contiguous run); returns the total.  warp_tot: 8 words.
__device__ uint32_t block_exclusive_scan(uint32_t* a, int n, uint32_t* warp_tot) {
    const int per = (n + blockDim.x - 1) / blockDim.x;
    const int b = threadIdx.x * per, e = min(n, b + per);
    uint32_t run = 0;
    for (int q = b; q < e; ++q) run += a[q];
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
    uint32_t incl = run;
#pragma unroll
    for (int k = 1; k < 32; k <<= 1) {
        const uint32_t v = __shfl_up_sync(0xffffffffu, incl, k);
        if (lane >= k) incl += v;
    }
    if (lane == 31) warp_tot[wid] = incl;
    __syncthreads();
    uint32_t before = incl - run, total = 0;
    for (int w = 0; w < (int)(blockDim.x >> 5); ++w) {
        if (w < wid) before += warp_tot[w];
        total += warp_tot[w];
    }
    for (int q = b; q < e; ++q) {
        const uint32_t v = a[q];
        a[q] = before;
        before += v;
    }
    __syncthreads();
    return total;
}

// Ranks inside residue classes: entries e = 0..n-1 hold a residue in bits
// 0..3 of key[e] (bits 17 and up are kept as they are); afterwards bits
// 4..16 hold k, the number of earlier entries of the same residue (n <=
// 8192), and rcount[r] counts the entries of residue r.  A ballot
// multi-split over 256 entries at a time.
__device__ void residue_ranks(uint32_t* key, int n, uint32_t* rcount,
                              uint32_t (*wres)[16]) {
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
    if (threadIdx.x < 16) rcount[threadIdx.x] = 0u;
    for (int base = 0; base < n; base += blockDim.x) {
        if (threadIdx.x < 128) wres[threadIdx.x >> 4][threadIdx.x & 15] = 0u;
        __syncthreads();
        const int pe = base + threadIdx.x;
        const bool act = pe < n;
        const uint32_t kv = act ? key[pe] : 16u;
        const uint32_t r = act ? (kv & 15u) : 16u;        // 16: no residue
        const unsigned mask = __match_any_sync(0xffffffffu, r);
        const uint32_t below = (uint32_t)__popc(mask & ((1u << lane) - 1u));
        if (act && below == 0) wres[wid][r] = (uint32_t)__popc(mask);
        __syncthreads();
        if (act) {
            uint32_t k = rcount[r] + below;
            for (int w = 0; w < wid; ++w) k += wres[w][r];
            key[pe] = (kv & ~0x1ffffu) | r | (k << 4);
        }
        __syncthreads();
        if (threadIdx.x < 16) {
            uint32_t s = 0;
            for (int w = 0; w < 8; ++w) s += wres[w][threadIdx.x];
            rcount[threadIdx.x] += s;
        }
        __syncthreads();
    }
}

// Greedy grouping of a subproblem's n points into rows of 16 consecutive
// output positions (the half-warps of the interpolation kernels, one point
// per lane) with as few repeated residues per row as the residue counts
// allow: a row costs as many shared-memory wavefronts per tap load as its
// most repeated residue, so the total is at least max(rows, max_r n_r).
// Each row takes one point from each residue that has points left, largest
// remainders first, passing over them again while the row has room (a
// residue repeats in a row only once fewer than 16 residues remain).
//
// While all 16 residues have points and rows are full, every row takes
// residue r into slot r: that happens for the first m = min(min_r n_r,
// n / 16) rows only, so the k-th point of residue r with k < m goes to
// position 16 k + r (computed by the caller).  This warp (lane r < 16
// owning residue r, rcount[r] points in their rank order k) deals the rest
// row by row and writes pos[rpre[r] + k - m] for k >= m, rpre being the
// exclusive prefix of n_r - m (also written, with *s_m = m).
__device__ void deal_rows(const uint32_t* rcount, uint32_t* rpre, uint32_t* pos,
                          int n, int* s_m) {
    const unsigned full = 0xffffffffu;
    const int lane = threadIdx.x & 31;
    const bool own = lane < 16;
    const int nr = own ? (int)rcount[lane] : 0;
    int m = 0;
    if (__popc(__ballot_sync(full, own && nr > 0)) == 16) {
        int mn = own ? nr : 0x7fffffff;
#pragma unroll
        for (int d = 16; d > 0; d >>= 1) mn = min(mn, __shfl_xor_sync(full, mn, d));
        m = min(mn, n / 16);
    }
    const int nt = own ? nr - m : 0;
    int pre = nt;
#pragma unroll
    for (int d = 1; d < 32; d <<= 1) {
        const int v = __shfl_up_sync(full, pre, d);
        if (lane >= d) pre += v;
    }
    pre -= nt;
    if (own) rpre[lane] = (uint32_t)pre;
    if (lane == 0) *s_m = m;
    int taken = 0;                       // tail points of this residue dealt
    for (int g = m, placed = 16 * m; placed < n; ++g) {
        const int cap = min(16, n - 16 * g);
        int t = 0, need = cap;
        while (need > 0) {
            const int r2 = nt - taken - t;
            const bool av = own && r2 > 0;
            const unsigned am = __ballot_sync(full, av);
            const int c = __popc(am);
            if (c == 0) break;           // never: rows hold no more than the points left
            if (c <= need) {
                t += av ? 1 : 0;
                need -= c;
            } else {
                int rank = 0;            // among available residues, r2 descending
                for (int j = 0; j < 16; ++j) {
                    const int rj = __shfl_sync(full, r2, j);
                    rank += (((am >> j) & 1u) && (rj > r2 || (rj == r2 && j < lane))) ? 1 : 0;
                }
                if (av && rank < need) t += 1;
                need = 0;
            }
        }
        int sp = t;                      // slot of this residue's first point in the row
#pragma unroll
        for (int d = 1; d < 32; d <<= 1) {
            const int v = __shfl_up_sync(full, sp, d);
            if (lane >= d) sp += v;
        }
        sp -= t;
        if (own)
            for (int i = 0; i < t; ++i) pos[pre + taken + i] = (uint32_t)(16 * g + sp + i);
        taken += t;
        placed += cap;
    }
}

// Order the points of every subproblem by their cell inside the bin
// (row-major, last dimension fastest, the tile's memory order), and -- when
// cp.rs is set -- deal them round-robin over the 16 bank residues of their
// first tap in the interpolation kernel's shared tile.  One CTA per
// subproblem:
//  1. shared histogram over the bin's cells with per-point ranks and a
//     block-wide exclusive scan give each point its cell-order position c;
//  2. (interleave) residue r = (sum_d l_d rs[d]) mod 16 of the point's
//     tile index; k = rank of the point among the residue-r points in cell
//     order (a ballot multi-split);
//  3. one warp deals the residues into rows of 16 output positions (a
//     half-warp of the interpolation kernels, one point per lane) with
//     distinct residues wherever the counts allow (deal_rows), so the
//     lanes' 8-byte tap loads hit distinct bank pairs.
// Shared memory: (cells per bin + 2 msub) x 4 bytes with the residue
// order (the per-point slots are reused for the dealt positions once each
// cell-order entry carries its point's index), (cells per bin + msub) x 4
// without.
template <int DIM>
__global__ void __launch_bounds__(256)
k_sub_sort(const int4* __restrict__ subs, CellParams cp, int mcells, int msub,
           const int2* __restrict__ i0, const int2* __restrict__ i1,
           const int2* __restrict__ i2, const uint32_t* __restrict__ pin,
           int2* __restrict__ o0, int2* __restrict__ o1, int2* __restrict__ o2,
           uint32_t* __restrict__ pout) {
    extern __shared__ uint32_t sm[];
    uint32_t* hist = sm;              // mcells counters, then starts
    uint32_t* slot = sm + mcells;     // per point: local cell | rank << 16
    // per cell-order position: residue | point << 17, then with k << 4 too
    uint32_t* kres = slot + msub;
    uint32_t* pos = slot;             // then: per (residue, rank) output position
    __shared__ uint32_t warp_tot[8];
    __shared__ uint32_t rcount[16];
    __shared__ uint32_t rpre[16];
    __shared__ int s_m;
    __shared__ uint32_t wres[8][16];
    const bool inter = cp.rs[0] != 0 || cp.rs[1] != 0 || cp.rs[2] != 0;
    const int4 sb = subs[blockIdx.x];
    const int start = sb.x, cnt = sb.y;
    int o[3] = {0, 0, 0};
    {
        int bin = sb.z;
#pragma unroll
        for (int d = DIM - 1; d >= 0; --d) {
            o[d] = (bin % cp.nb[d]) * cp.m[d] - cp.halfw;
            bin /= cp.nb[d];
        }
    }
    const int2* in[3] = {i0, i1, i2};
    auto residue = [&](int t) {
        int tix = 0;
#pragma unroll
        for (int d = 0; d < DIM; ++d) {
            int l = in[d][start + t].x - o[d];
            l = min(max(l, 0), cp.m[d] - 1);
            tix += l * cp.rs[d];
        }
        return (uint32_t)tix & 15u;
    };
    for (int q = threadIdx.x; q < mcells; q += blockDim.x) hist[q] = 0u;
    __syncthreads();
    for (int t = threadIdx.x; t < cnt; t += blockDim.x) {
        uint32_t loc = 0;
#pragma unroll
        for (int d = 0; d < DIM; ++d) {
            int l = in[d][start + t].x - o[d];
            l = min(max(l, 0), cp.m[d] - 1);   // setpts output is in range
            loc = loc * (uint32_t)cp.m[d] + (uint32_t)l;
        }
        const uint32_t r = atomicAdd(hist + loc, 1u);
        slot[t] = loc | (r << 16);
    }
    __syncthreads();
    block_exclusive_scan(hist, mcells, warp_tot);
    int2* out[3] = {o0, o1, o2};
    auto put = [&](int t, int pos) {
#pragma unroll
        for (int d = 0; d < DIM; ++d) out[d][start + pos] = in[d][start + t];
        pout[start + pos] = pin[start + t];
    };
    if (!inter) {
        for (int t = threadIdx.x; t < cnt; t += blockDim.x) {
            const uint32_t sl = slot[t];
            put(t, (int)(hist[sl & 0xffffu] + (sl >> 16)));
        }
        return;
    }
    // cell-order position c of every point: its residue and index there
    for (int t = threadIdx.x; t < cnt; t += blockDim.x) {
        const uint32_t sl = slot[t];
        const uint32_t c = hist[sl & 0xffffu] + (sl >> 16);
        kres[c] = residue(t) | ((uint32_t)t << 17);
    }
    __syncthreads();
    residue_ranks(kres, cnt, rcount, wres);   // (also orders slot[] reads before pos[] writes)
    if (threadIdx.x < 32) deal_rows(rcount, rpre, pos, cnt, &s_m);
    __syncthreads();
    const uint32_t m = (uint32_t)s_m;
    for (int c = threadIdx.x; c < cnt; c += blockDim.x) {
        const uint32_t kr = kres[c], r = kr & 15u, k = (kr >> 4) & 0x1fffu;
        put((int)(kr >> 17), (int)(k < m ? 16u * k + r : pos[rpre[r] + k - m]));
    }
}

// Type-3 phases, written in sorted order (position j reads caller index
// perm[j]).
//  mode 1: prephase e^{i isign sum_d D_d x_d}            (gpu_t3.py:491-493)
//  mode 2: post e^{i isign sum_d C_d (s_d - D_d)} / prod_d phihat(theta_d)
//          with theta_d = (s_d - D_d) * (h_d gam_d)       (gpu_t3.py:368-377)
template <int DIM>
__global__ void k_phase(int64_t M, Coords X, const uint32_t* perm,
                        PhaseParams pp, CellParams cp, float2* phase) {
    int64_t j = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
    if (j >= M) return;
    int64_t src = perm ? (int64_t)perm[j] : j;
    double ang;
    if (!pp.fp32) {
        ang = 0.0;
#pragma unroll
        for (int d = 0; d < DIM; ++d) {
            double v = X.p[d][src];
            ang += (pp.mode == 1) ? pp.D[d] * v : pp.C[d] * (v - pp.D[d]);
        }
    } else {
        float a = 0.0f;
#pragma unroll
        for (int d = 0; d < DIM; ++d) {
            float v = (float)X.p[d][src];
            a += (pp.mode == 1) ? (float)pp.D[d] * v
                                : (float)pp.C[d] * (v - (float)pp.D[d]);
        }
        ang = (double)a;
    }
    double sn, cs;
    sincos((double)pp.isign * ang, &sn, &cs);
    if (pp.mode == 2) {
        double tdec = 1.0;
#pragma unroll
        for (int d = 0; d < DIM; ++d) {
            double s = X.p[d][src];
            double th;
            if (!cp.fp32)
                th = (s - cp.a[d]) * cp.b[d];
            else
                th = (double)(((float)s - (float)cp.a[d]) * (float)cp.b[d]);
            double acc = 0.0;
            for (int q = 0; q < pp.nq; ++q) acc += pp.fta[q] * cos(th * pp.ftd[q]);
            tdec *= 2.0 * acc;
        }
        cs /= tdec;
        sn /= tdec;
    }
    phase[j] = make_float2((float)cs, (float)sn);
}

// Partial min/max of up to 6 arrays: partial[blk][2*i] = min, [2*i+1] = max.
struct Arr6 {
    const double* p[6];
};
__global__ void k_minmax(int n, Arr6 A, int64_t M, double* partial) {
    __shared__ double smin[6][256], smax[6][256];
    const int t = threadIdx.x;
    for (int i = 0; i < n; ++i) {
        double lo = INFINITY, hi = -INFINITY;
        for (int64_t j = blockIdx.x * (int64_t)blockDim.x + t; j < M;
             j += (int64_t)gridDim.x * blockDim.x) {
            double v = A.p[i][j];
            lo = fmin(lo, v);
            hi = fmax(hi, v);
        }
        smin[i][t] = lo;
        smax[i][t] = hi;
    }
    __syncthreads();
    for (int s = 128; s > 0; s >>= 1) {
        if (t < s)
            for (int i = 0; i < n; ++i) {
                smin[i][t] = fmin(smin[i][t], smin[i][t + s]);
                smax[i][t] = fmax(smax[i][t], smax[i][t + s]);
            }
        __syncthreads();
    }
    if (t == 0)
        for (int i = 0; i < n; ++i) {
            partial[blockIdx.x * 2 * n + 2 * i] = smin[i][0];
            partial[blockIdx.x * 2 * n + 2 * i + 1] = smax[i][0];
        }
}

void device_minmax(int n, const double* const* arrs, int64_t M, double* out,
                   cudaStream_t st) {
    Arr6 A{};
    for (int i = 0; i < n; ++i) A.p[i] = arrs[i];
    int blocks = (int)std::min<int64_t>(512, (M + 255) / 256);
    if (blocks < 1) blocks = 1;
    double* d_part = (double*)dmalloc(sizeof(double) * blocks * 2 * n, "minmax");
    k_minmax<<<blocks, 256, 0, st>>>(n, A, M, d_part);
    NUFFT_LAUNCH("k_minmax");
    std::vector<double> h(blocks * 2 * n);
    NUFFT_CUDA(cudaMemcpyAsync(h.data(), d_part, sizeof(double) * h.size(),
                               cudaMemcpyDeviceToHost, st));
    NUFFT_CUDA(cudaStreamSynchronize(st));
    dfree(d_part);
    for (int i = 0; i < n; ++i) {
        double lo = INFINITY, hi = -INFINITY;
        for (int b = 0; b < blocks; ++b) {
            lo = std::min(lo, h[b * 2 * n + 2 * i]);
            hi = std::max(hi, h[b * 2 * n + 2 * i + 1]);
        }
        out[2 * i] = lo;
        out[2 * i + 1] = hi;
    }
}

void free_pointset(PointSet* ps) {
    for (int d = 0; d < 3; ++d) {
        dfree(ps->cell[d]);
        ps->cell[d] = nullptr;
    }
    dfree(ps->perm);
    dfree(ps->subs);
    dfree(ps->phase);
    dfree(ps->sched);
    dfree(ps->scratch);
    for (int d = 0; d < 3; ++d) {
        dfree(ps->cell_alt[d]);
        ps->cell_alt[d] = nullptr;
    }
    dfree(ps->perm_alt);
    ps->scratch = nullptr;
    ps->scratch_bytes = 0;
    ps->perm_alt = nullptr;
    ps->perm = nullptr;
    ps->subs = nullptr;
    ps->phase = nullptr;
    ps->sched = nullptr;
    ps->cap = ps->subcap = ps->M = ps->nsub = 0;
}

namespace {

// Cell order inside every subproblem (k_sub_sort) into fresh arrays, which
// then replace the point set's cells and permutation.  NUFFT_SUB_SORT
// (tuning): 0 off, 1 plain cell order, 2 (default) residue interleave when
// the plan gave the tile strides.
template <int DIM>
void sub_sort(PointSet* ps, const CellParams& cp, int msub, cudaStream_t st) {
    static const char* env = std::getenv("NUFFT_SUB_SORT");
    const int mode = (env && *env) ? std::atoi(env) : 2;
    if (mode == 0) return;
    CellParams c2 = cp;
    if (mode == 1) c2.rs[0] = c2.rs[1] = c2.rs[2] = 0;
    const bool inter = c2.rs[0] != 0 || c2.rs[1] != 0 || c2.rs[2] != 0;
    int mcells = 1;
    for (int d = 0; d < DIM; ++d) mcells *= cp.m[d];
    // 16-bit slot fields; 13-bit rank and point fields of the residue keys
    if (mcells > 65536 || msub > 65536 || (inter && msub > 8192)) return;
    const size_t smem = sizeof(uint32_t) *
                        ((size_t)mcells + (size_t)msub * (inter ? 2 : 1));
    // opt in beyond the default dynamic limit (the kernel also has about
    // 0.6 KB of static shared memory)
    if (smem > 40 * 1024) {
        NUFFT_CUDA(cudaFuncSetAttribute((const void*)k_sub_sort<DIM>,
                                        cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        (int)smem));
    }
    // second buffers, kept in the point set and swapped with the primary ones
    if (!ps->perm_alt) {
        for (int d = 0; d < DIM; ++d)
            ps->cell_alt[d] = (int2*)dmalloc(sizeof(int2) * (ps->cap + kPointSlack),
                                             "sorted cells");
        ps->perm_alt = (uint32_t*)dmalloc(4 * (ps->cap + kPointSlack), "sorted permutation");
    }
    k_sub_sort<DIM><<<(unsigned)ps->nsub, 256, smem, st>>>(
        ps->subs, c2, mcells, msub, ps->cell[0], ps->cell[1], ps->cell[2], ps->perm,
        ps->cell_alt[0], ps->cell_alt[1], ps->cell_alt[2], ps->perm_alt);
    NUFFT_LAUNCH("k_sub_sort");
    for (int d = 0; d < DIM; ++d) std::swap(ps->cell[d], ps->cell_alt[d]);
    std::swap(ps->perm, ps->perm_alt);
}

template <int DIM>
void build_impl(PointSet* ps, const CellParams& cp, int64_t M,
                const double* const* coords, bool sort, bool tiled, int msub,
                bool cell_order, const PhaseParams& pp, int* d_err,
                cudaStream_t st) {
    Coords X{};
    for (int d = 0; d < DIM; ++d) X.p[d] = coords[d];
    const int bs = 256;
    const int64_t grid = (M + bs - 1) / bs;
    if (!sort) {
        k_cells_direct<DIM><<<(unsigned)grid, bs, 0, st>>>(
            M, X, cp, ps->cell[0], ps->cell[1], ps->cell[2], d_err);
        NUFFT_LAUNCH("k_cells_direct");
    } else {
        int64_t nbins_sp = 1;
        for (int d = 0; d < DIM; ++d) nbins_sp *= cp.nb[d];
        const int64_t nchunks = cp.chunk ? (M + cp.chunk - 1) / cp.chunk : 1;
        const int64_t nbins = nbins_sp * nchunks;
        if (nbins > (int64_t)0x7fffffffLL) fail(-1, "too many bins");
        // sort scratch: keys and ranks per point, four arrays per sort key,
        // the scan total; one allocation kept in the point set
        auto al = [](size_t b) { return (b + 255) & ~(size_t)255; };
        const size_t pb = al(4 * (size_t)M), kb = al(4 * (size_t)(nbins + 1));
        const size_t need = 2 * pb + 6 * kb + 256;
        if (need > ps->scratch_bytes) {
            dfree(ps->scratch);       // previous setpts synchronised its stream
            ps->scratch = nullptr;
            ps->scratch_bytes = 0;
            ps->scratch = dmalloc(need + need / 4, "sort scratch");
            ps->scratch_bytes = need + need / 4;
        }
        char* sp = (char*)ps->scratch;
        uint32_t* key_of = (uint32_t*)sp;
        uint32_t* rank_of = (uint32_t*)(sp + pb);
        uint32_t* count = (uint32_t*)(sp + 2 * pb);
        uint32_t* start = (uint32_t*)(sp + 2 * pb + kb);
        uint32_t* nsubs = (uint32_t*)(sp + 2 * pb + 2 * kb);
        uint32_t* subofs = (uint32_t*)(sp + 2 * pb + 3 * kb);
        uint32_t* npart = (uint32_t*)(sp + 2 * pb + 4 * kb);
        uint32_t* partofs = (uint32_t*)(sp + 2 * pb + 5 * kb);
        uint32_t* tot = (uint32_t*)(sp + 2 * pb + 6 * kb);   // [0] subproblems, [1] full ones
        NUFFT_CUDA(cudaMemsetAsync(count, 0, 4 * (nbins + 1), st));
        k_bin_count<DIM><<<(unsigned)grid, bs, 0, st>>>(M, X, cp, key_of,
                                                       rank_of, count, d_err);
        NUFFT_LAUNCH("k_bin_count");
        k_scan<<<1, 1024, 0, st>>>(count, start, nbins, tot);
        NUFFT_LAUNCH("k_scan");
        k_bin_scatter<DIM><<<(unsigned)grid, bs, 0, st>>>(
            M, X, cp, key_of, rank_of, start, ps->cell[0], ps->cell[1],
            ps->cell[2], ps->perm);
        NUFFT_LAUNCH("k_bin_scatter");
        ps->nsub = 0;
        if (tiled) {
            const unsigned gb = (unsigned)((nbins + 255) / 256);
            k_sub_count<<<gb, 256, 0, st>>>(count, nbins, msub, nsubs);
            NUFFT_LAUNCH("k_sub_count");
            k_scan<<<1, 1024, 0, st>>>(nsubs, subofs, nbins, tot);
            NUFFT_LAUNCH("k_scan");
            uint32_t h_tot = 0;
            NUFFT_CUDA(cudaMemcpyAsync(&h_tot, tot, 4, cudaMemcpyDeviceToHost, st));
            NUFFT_CUDA(cudaStreamSynchronize(st));
            if ((int64_t)h_tot > ps->subcap) {
                dfree(ps->subs);
                ps->subs = nullptr;
                ps->subcap = 0;
                ps->subs = (int4*)dmalloc(sizeof(int4) * std::max<int64_t>(h_tot, 1),
                                          "subproblems");
                ps->subcap = std::max<int64_t>(h_tot, 1);
            }
            if (cell_order) {
                // interpolation: full subproblems first; offsets of full and
                // partial ones (nsubs / subofs reused for the full counts
                // and offsets)
                k_sub_split<<<gb, 256, 0, st>>>(count, nbins, msub, nsubs, npart);
                NUFFT_LAUNCH("k_sub_split");
                k_scan<<<1, 1024, 0, st>>>(nsubs, subofs, nbins, tot + 1);
                NUFFT_LAUNCH("k_scan");
                k_scan<<<1, 1024, 0, st>>>(npart, partofs, nbins, tot + 2);
                NUFFT_LAUNCH("k_scan");
            }
            k_sub_fill<<<gb, 256, 0, st>>>(count, start, subofs,
                                           cell_order ? partofs : nullptr, tot + 1, nbins,
                                           nbins_sp, msub, ps->subs);
            NUFFT_LAUNCH("k_sub_fill");
            ps->nsub = h_tot;
            if (h_tot > 0 && cell_order && DIM != 2)
                sub_sort<DIM>(ps, cp, msub, st);
        }
        NUFFT_CUDA(cudaStreamSynchronize(st));   // scratch free for reuse
    }
    if (pp.mode) {
        k_phase<DIM><<<(unsigned)grid, bs, 0, st>>>(
            M, X, sort ? ps->perm : nullptr, pp, cp, ps->phase);
        NUFFT_LAUNCH("k_phase");
    }
}

}  // namespace

void build_pointset(PointSet* ps, const CellParams& cp, int64_t M,
                    const double* const* coords, bool sort, bool tiled,
                    int msub, bool cell_order, const PhaseParams& pp,
                    int* d_err, cudaStream_t st) {
    if (M < 1) fail(-1, "at least one nonuniform point is required");
    if (M >= (int64_t)0x7fffffffLL)
        fail(-1, "at most 2^31-1 nonuniform points per plan");
    if (M > ps->cap || (sort && !ps->perm) || (pp.mode && !ps->phase)) {
        free_pointset(ps);
        for (int d = 0; d < cp.dim; ++d)
            ps->cell[d] = (int2*)dmalloc(sizeof(int2) * (M + kPointSlack), "point cells");
        ps->perm = (uint32_t*)dmalloc(4 * (M + kPointSlack), "point permutation");
        if (pp.mode)
            ps->phase = (float2*)dmalloc(sizeof(float2) * (M + kPointSlack), "phases");
        ps->sched = (int*)dmalloc(2 * sizeof(int), "scheduler");
        NUFFT_CUDA(cudaMemsetAsync(ps->sched, 0, 2 * sizeof(int), st));
        ps->cap = M;
    }
    ps->dim = cp.dim;
    ps->M = M;
    ps->msub = msub;
    ps->sorted = sort;
    ps->tiled = tiled && sort;
    switch (cp.dim) {
        case 1: build_impl<1>(ps, cp, M, coords, sort, tiled, msub, cell_order, pp, d_err, st); break;
        case 2: build_impl<2>(ps, cp, M, coords, sort, tiled, msub, cell_order, pp, d_err, st); break;
        case 3: build_impl<3>(ps, cp, M, coords, sort, tiled, msub, cell_order, pp, d_err, st); break;
        default: fail(-1, "dim must be 1, 2 or 3");
    }
}

}  // namespace nufft
