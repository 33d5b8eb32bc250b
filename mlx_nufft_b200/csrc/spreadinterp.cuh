// spreadinterp.cuh -- exponential-of-semicircle (ES) spreading and
// interpolation kernels for sm_100a, shared by spread.cu and interp.cu.
//
// Two families, chosen per point set at setpts time:
//  * tiled (the reference's "output-driven" OD path, mlx_nufft/nd.py:492-579
//    and 974-1073): points are counting-sorted by bin; one CTA owns one
//    subproblem (<= msub points of one bin) and works on a shared-memory
//    tile covering the bin plus the kernel halo (bin + w - 1 cells per
//    dimension, periodically wrapped).  Spread accumulates into the tile
//    with shared-memory atomics and flushes it with one vector (float2)
//    global atomic per touched cell; interp loads the tile once and gathers.
//  * global (the reference's "GM" path, nd.py:437-490, 908-972): one thread
//    per point reading / atomically updating the fine grid directly; used
//    for small point counts and when the grid is L2-resident.
//
// The ES kernel psi(d) = exp(beta (sqrt(1 - (2d/w)^2) - 1)) is evaluated in
// fp32 with the accurate expf/sqrtf (no fast-math), as the reference does
// with metal::precise (mlx_nufft/gpu_t3.py:30-37).
#pragma once

#include <cuda_runtime.h>

#include "internal.h"

namespace nufft {

struct CellPtrs {
    const int2* d[3];
};

__device__ __forceinline__ float es_weight(float d, float c2w, float beta) {
    float z = d * c2w;
    float t = fmaxf(1.0f - z * z, 0.0f);
    return expf(beta * (sqrtf(t) - 1.0f));
}

__device__ __forceinline__ float2 cmul(float2 a, float2 b) {
    return make_float2(a.x * b.x - a.y * b.y, a.x * b.y + a.y * b.x);
}

__device__ __forceinline__ int wrap1(int x, int n) {
    x -= (x >= n) ? n : 0;
    x += (x < 0) ? n : 0;
    return x;
}

__device__ __forceinline__ int wrapmod(int x, int n) {
    x %= n;
    return x < 0 ? x + n : x;
}

// Tile origin (global cell of tile index 0) of bin `bin` (row-major over nb).
template <int DIM>
__device__ __forceinline__ void bin_origin(int bin, const TileGeom& tg,
                                           int* o) {
#pragma unroll
    for (int d = DIM - 1; d >= 0; --d) {
        int b = bin % tg.nb[d];
        bin /= tg.nb[d];
        o[d] = b * tg.m[d] - tg.halfw;
    }
}

// Global linear cell of tile index q, with periodic wrap.
template <int DIM>
__device__ __forceinline__ int64_t tile_to_global(int q, const int* o,
                                                  const TileGeom& tg) {
    int p[3];
#pragma unroll
    for (int d = DIM - 1; d >= 0; --d) {
        p[d] = q % tg.T[d];
        q /= tg.T[d];
    }
    int64_t g = 0;
#pragma unroll
    for (int d = 0; d < DIM; ++d)
        g = g * tg.n[d] + wrapmod(o[d] + p[d], tg.n[d]);
    return g;
}

// ES weights of one point in every dimension; returns false if the point's
// cell is not inside the bin (never for consistent setpts output; guards
// the shared-memory indexing).
template <int DIM, int W>
__device__ __forceinline__ bool point_weights(const CellPtrs& cells, int64_t j,
                                              const int* o, const TileGeom& tg,
                                              float (&wgt)[DIM][W],
                                              int (&l0)[DIM]) {
    bool ok = true;
#pragma unroll
    for (int d = 0; d < DIM; ++d) {
        int2 cl = __ldg(cells.d[d] + j);
        l0[d] = cl.x - o[d];
        ok &= (unsigned)l0[d] < (unsigned)tg.m[d];
        float fr = __int_as_float(cl.y);
#pragma unroll
        for (int l = 0; l < W; ++l)
            wgt[d][l] = es_weight((float)l - fr, tg.c2w, tg.beta);
    }
    return ok;
}

// --------------------------------------------------------------------
// tiled spread: grid[v] += sum_j c[v][perm j] * phase_j * psi-tensor
template <int DIM, int W>
__global__ void __launch_bounds__(256)
k_spread_tiled(const float2* __restrict__ c, int64_t cstride, int nvg,
               const uint32_t* __restrict__ perm, CellPtrs cells,
               const float2* __restrict__ phase, const int4* __restrict__ subs,
               float2* __restrict__ grid, TileGeom tg) {
    extern __shared__ float2 tile[];
    const int4 sb = subs[blockIdx.x];
    const int start = sb.x, cnt = sb.y;
    int o[3] = {0, 0, 0};
    bin_origin<DIM>(sb.z, tg, o);
    const int T = tg.tcells;
    for (int q = threadIdx.x; q < nvg * T; q += blockDim.x)
        tile[q] = make_float2(0.0f, 0.0f);
    __syncthreads();
    for (int t = threadIdx.x; t < cnt; t += blockDim.x) {
        const int64_t j = start + t;
        const int64_t src = perm ? (int64_t)__ldg(perm + j) : j;
        float wgt[DIM][W];
        int l0[DIM];
        if (!point_weights<DIM, W>(cells, j, o, tg, wgt, l0)) continue;
        const float2 ph = phase ? __ldg(phase + j) : make_float2(1.0f, 0.0f);
        for (int v = 0; v < nvg; ++v) {
            float2 cv = __ldg(c + v * cstride + src);
            if (phase) cv = cmul(cv, ph);
            float* tv = reinterpret_cast<float*>(tile + v * T);
            if (DIM == 1) {
#pragma unroll
                for (int a = 0; a < W; ++a) {
                    const int q = 2 * (l0[0] + a);
                    atomicAdd(tv + q, cv.x * wgt[0][a]);
                    atomicAdd(tv + q + 1, cv.y * wgt[0][a]);
                }
            } else if (DIM == 2) {
#pragma unroll
                for (int a = 0; a < W; ++a) {
                    const float2 ca = make_float2(cv.x * wgt[0][a], cv.y * wgt[0][a]);
                    const int row = (l0[0] + a) * tg.T[1] + l0[DIM > 1 ? 1 : 0];
#pragma unroll
                    for (int b = 0; b < W; ++b) {
                        const int q = 2 * (row + b);
                        atomicAdd(tv + q, ca.x * wgt[DIM > 1 ? 1 : 0][b]);
                        atomicAdd(tv + q + 1, ca.y * wgt[DIM > 1 ? 1 : 0][b]);
                    }
                }
            } else {
#pragma unroll 1
                for (int a = 0; a < W; ++a) {
#pragma unroll
                    for (int b = 0; b < W; ++b) {
                        const float wab = wgt[0][a] * wgt[DIM > 1 ? 1 : 0][b];
                        const float2 cab = make_float2(cv.x * wab, cv.y * wab);
                        const int base =
                            ((l0[0] + a) * tg.T[1] + l0[DIM > 1 ? 1 : 0] + b) *
                                tg.T[DIM > 2 ? 2 : 0] + l0[DIM > 2 ? 2 : 0];
#pragma unroll
                        for (int k = 0; k < W; ++k) {
                            const int q = 2 * (base + k);
                            atomicAdd(tv + q, cab.x * wgt[DIM > 2 ? 2 : 0][k]);
                            atomicAdd(tv + q + 1, cab.y * wgt[DIM > 2 ? 2 : 0][k]);
                        }
                    }
                }
            }
        }
    }
    __syncthreads();
    for (int q = threadIdx.x; q < T; q += blockDim.x) {
        const int64_t g = tile_to_global<DIM>(q, o, tg);
        for (int v = 0; v < nvg; ++v) {
            const float2 val = tile[v * T + q];
            if (val.x != 0.0f || val.y != 0.0f)
                atomicAdd(grid + v * tg.ncells + g, val);
        }
    }
}

// --------------------------------------------------------------------
// tiled interp: out[v][perm j] = phase_j * sum taps tile[v] * psi-tensor
template <int DIM, int W>
__global__ void __launch_bounds__(256)
k_interp_tiled(const float2* __restrict__ grid, int nvg,
               const uint32_t* __restrict__ perm, CellPtrs cells,
               const float2* __restrict__ phase, const int4* __restrict__ subs,
               float2* __restrict__ out, int64_t ostride, TileGeom tg) {
    extern __shared__ float2 tile[];
    const int4 sb = subs[blockIdx.x];
    const int start = sb.x, cnt = sb.y;
    int o[3] = {0, 0, 0};
    bin_origin<DIM>(sb.z, tg, o);
    const int T = tg.tcells;
    for (int q = threadIdx.x; q < T; q += blockDim.x) {
        const int64_t g = tile_to_global<DIM>(q, o, tg);
        for (int v = 0; v < nvg; ++v)
            tile[v * T + q] = __ldg(grid + v * tg.ncells + g);
    }
    __syncthreads();
    for (int t = threadIdx.x; t < cnt; t += blockDim.x) {
        const int64_t j = start + t;
        const int64_t dst = perm ? (int64_t)__ldg(perm + j) : j;
        float wgt[DIM][W];
        int l0[DIM];
        const bool ok = point_weights<DIM, W>(cells, j, o, tg, wgt, l0);
        const float2 ph = phase ? __ldg(phase + j) : make_float2(1.0f, 0.0f);
        for (int v = 0; v < nvg; ++v) {
            const float2* tv = tile + v * T;
            float2 acc = make_float2(0.0f, 0.0f);
            if (ok) {
                if (DIM == 1) {
#pragma unroll
                    for (int a = 0; a < W; ++a) {
                        const float2 g = tv[l0[0] + a];
                        acc.x = fmaf(g.x, wgt[0][a], acc.x);
                        acc.y = fmaf(g.y, wgt[0][a], acc.y);
                    }
                } else if (DIM == 2) {
#pragma unroll
                    for (int a = 0; a < W; ++a) {
                        const int row = (l0[0] + a) * tg.T[1] + l0[DIM > 1 ? 1 : 0];
                        float2 s = make_float2(0.0f, 0.0f);
#pragma unroll
                        for (int b = 0; b < W; ++b) {
                            const float2 g = tv[row + b];
                            s.x = fmaf(g.x, wgt[DIM > 1 ? 1 : 0][b], s.x);
                            s.y = fmaf(g.y, wgt[DIM > 1 ? 1 : 0][b], s.y);
                        }
                        acc.x = fmaf(s.x, wgt[0][a], acc.x);
                        acc.y = fmaf(s.y, wgt[0][a], acc.y);
                    }
                } else {
#pragma unroll 1
                    for (int a = 0; a < W; ++a) {
#pragma unroll
                        for (int b = 0; b < W; ++b) {
                            const float wab = wgt[0][a] * wgt[DIM > 1 ? 1 : 0][b];
                            const int base =
                                ((l0[0] + a) * tg.T[1] + l0[DIM > 1 ? 1 : 0] + b) *
                                    tg.T[DIM > 2 ? 2 : 0] + l0[DIM > 2 ? 2 : 0];
                            float2 s = make_float2(0.0f, 0.0f);
#pragma unroll
                            for (int k = 0; k < W; ++k) {
                                const float2 g = tv[base + k];
                                s.x = fmaf(g.x, wgt[DIM > 2 ? 2 : 0][k], s.x);
                                s.y = fmaf(g.y, wgt[DIM > 2 ? 2 : 0][k], s.y);
                            }
                            acc.x = fmaf(s.x, wab, acc.x);
                            acc.y = fmaf(s.y, wab, acc.y);
                        }
                    }
                }
                if (phase) acc = cmul(acc, ph);
            }
            out[v * ostride + dst] = acc;
        }
    }
}

// --------------------------------------------------------------------
// global-memory variants: one thread per point (sorted or caller order).
template <int DIM, int W>
__device__ __forceinline__ void global_taps(const CellPtrs& cells, int64_t j,
                                            const TileGeom& tg,
                                            float (&wgt)[DIM][W],
                                            int (&idx)[DIM][W]) {
#pragma unroll
    for (int d = 0; d < DIM; ++d) {
        int2 cl = __ldg(cells.d[d] + j);
        float fr = __int_as_float(cl.y);
#pragma unroll
        for (int l = 0; l < W; ++l) {
            wgt[d][l] = es_weight((float)l - fr, tg.c2w, tg.beta);
            idx[d][l] = wrap1(cl.x + l, tg.n[d]);
        }
    }
}

template <int DIM, int W>
__global__ void __launch_bounds__(256)
k_spread_global(const float2* __restrict__ c, int64_t cstride, int nvec,
                const uint32_t* __restrict__ perm, CellPtrs cells,
                const float2* __restrict__ phase, int64_t M,
                float2* __restrict__ grid, TileGeom tg) {
    const int64_t j = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
    if (j >= M) return;
    const int64_t src = perm ? (int64_t)__ldg(perm + j) : j;
    float wgt[DIM][W];
    int idx[DIM][W];
    global_taps<DIM, W>(cells, j, tg, wgt, idx);
    const float2 ph = phase ? __ldg(phase + j) : make_float2(1.0f, 0.0f);
    for (int v = 0; v < nvec; ++v) {
        float2 cv = __ldg(c + v * cstride + src);
        if (phase) cv = cmul(cv, ph);
        float2* gv = grid + v * tg.ncells;
        if (DIM == 1) {
#pragma unroll
            for (int a = 0; a < W; ++a)
                atomicAdd(gv + idx[0][a],
                          make_float2(cv.x * wgt[0][a], cv.y * wgt[0][a]));
        } else if (DIM == 2) {
#pragma unroll
            for (int a = 0; a < W; ++a) {
                const int64_t row = (int64_t)idx[0][a] * tg.n[1];
#pragma unroll
                for (int b = 0; b < W; ++b) {
                    const float wab = wgt[0][a] * wgt[DIM > 1 ? 1 : 0][b];
                    atomicAdd(gv + row + idx[DIM > 1 ? 1 : 0][b],
                              make_float2(cv.x * wab, cv.y * wab));
                }
            }
        } else {
#pragma unroll 1
            for (int a = 0; a < W; ++a) {
#pragma unroll
                for (int b = 0; b < W; ++b) {
                    const float wab = wgt[0][a] * wgt[DIM > 1 ? 1 : 0][b];
                    const int64_t base =
                        ((int64_t)idx[0][a] * tg.n[1] + idx[DIM > 1 ? 1 : 0][b]) *
                        tg.n[DIM > 2 ? 2 : 0];
#pragma unroll
                    for (int k = 0; k < W; ++k) {
                        const float wk = wab * wgt[DIM > 2 ? 2 : 0][k];
                        atomicAdd(gv + base + idx[DIM > 2 ? 2 : 0][k],
                                  make_float2(cv.x * wk, cv.y * wk));
                    }
                }
            }
        }
    }
}

template <int DIM, int W>
__global__ void __launch_bounds__(256)
k_interp_global(const float2* __restrict__ grid, int nvec,
                const uint32_t* __restrict__ perm, CellPtrs cells,
                const float2* __restrict__ phase, int64_t M,
                float2* __restrict__ out, int64_t ostride, TileGeom tg) {
    const int64_t j = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
    if (j >= M) return;
    const int64_t dst = perm ? (int64_t)__ldg(perm + j) : j;
    float wgt[DIM][W];
    int idx[DIM][W];
    global_taps<DIM, W>(cells, j, tg, wgt, idx);
    const float2 ph = phase ? __ldg(phase + j) : make_float2(1.0f, 0.0f);
    for (int v = 0; v < nvec; ++v) {
        const float2* gv = grid + v * tg.ncells;
        float2 acc = make_float2(0.0f, 0.0f);
        if (DIM == 1) {
#pragma unroll
            for (int a = 0; a < W; ++a) {
                const float2 g = __ldg(gv + idx[0][a]);
                acc.x = fmaf(g.x, wgt[0][a], acc.x);
                acc.y = fmaf(g.y, wgt[0][a], acc.y);
            }
        } else if (DIM == 2) {
#pragma unroll
            for (int a = 0; a < W; ++a) {
                const int64_t row = (int64_t)idx[0][a] * tg.n[1];
                float2 s = make_float2(0.0f, 0.0f);
#pragma unroll
                for (int b = 0; b < W; ++b) {
                    const float2 g = __ldg(gv + row + idx[DIM > 1 ? 1 : 0][b]);
                    s.x = fmaf(g.x, wgt[DIM > 1 ? 1 : 0][b], s.x);
                    s.y = fmaf(g.y, wgt[DIM > 1 ? 1 : 0][b], s.y);
                }
                acc.x = fmaf(s.x, wgt[0][a], acc.x);
                acc.y = fmaf(s.y, wgt[0][a], acc.y);
            }
        } else {
#pragma unroll 1
            for (int a = 0; a < W; ++a) {
#pragma unroll
                for (int b = 0; b < W; ++b) {
                    const float wab = wgt[0][a] * wgt[DIM > 1 ? 1 : 0][b];
                    const int64_t base =
                        ((int64_t)idx[0][a] * tg.n[1] + idx[DIM > 1 ? 1 : 0][b]) *
                        tg.n[DIM > 2 ? 2 : 0];
                    float2 s = make_float2(0.0f, 0.0f);
#pragma unroll
                    for (int k = 0; k < W; ++k) {
                        const float2 g = __ldg(gv + base + idx[DIM > 2 ? 2 : 0][k]);
                        s.x = fmaf(g.x, wgt[DIM > 2 ? 2 : 0][k], s.x);
                        s.y = fmaf(g.y, wgt[DIM > 2 ? 2 : 0][k], s.y);
                    }
                    acc.x = fmaf(s.x, wab, acc.x);
                    acc.y = fmaf(s.y, wab, acc.y);
                }
            }
        }
        if (phase) acc = cmul(acc, ph);
        out[v * ostride + dst] = acc;
    }
}

// Compile-time dispatch over the kernel width 2..16 and the dimension.
#define NUFFT_WIDTH_SWITCH(w, ...)                                     \
    switch (w) {                                                       \
        case 2: { constexpr int W = 2; __VA_ARGS__; } break;           \
        case 3: { constexpr int W = 3; __VA_ARGS__; } break;           \
        case 4: { constexpr int W = 4; __VA_ARGS__; } break;           \
        case 5: { constexpr int W = 5; __VA_ARGS__; } break;           \
        case 6: { constexpr int W = 6; __VA_ARGS__; } break;           \
        case 7: { constexpr int W = 7; __VA_ARGS__; } break;           \
        case 8: { constexpr int W = 8; __VA_ARGS__; } break;           \
        case 9: { constexpr int W = 9; __VA_ARGS__; } break;           \
        case 10: { constexpr int W = 10; __VA_ARGS__; } break;         \
        case 11: { constexpr int W = 11; __VA_ARGS__; } break;         \
        case 12: { constexpr int W = 12; __VA_ARGS__; } break;         \
        case 13: { constexpr int W = 13; __VA_ARGS__; } break;         \
        case 14: { constexpr int W = 14; __VA_ARGS__; } break;         \
        case 15: { constexpr int W = 15; __VA_ARGS__; } break;         \
        case 16: { constexpr int W = 16; __VA_ARGS__; } break;         \
        default: fail(-1, "kernel width must be in [2, 16]");          \
    }

#define NUFFT_DIM_SWITCH(dim, ...)                                     \
    switch (dim) {                                                     \
        case 1: { constexpr int DIM = 1; __VA_ARGS__; } break;         \
        case 2: { constexpr int DIM = 2; __VA_ARGS__; } break;         \
        case 3: { constexpr int DIM = 3; __VA_ARGS__; } break;         \
        default: fail(-1, "dim must be 1, 2 or 3");                    \
    }

inline CellPtrs cell_ptrs(const PointSet& ps) {
    CellPtrs cp{};
    for (int d = 0; d < 3; ++d) cp.d[d] = ps.cell[d];
    return cp;
}

// Raise a kernel's dynamic shared-memory limit to `bytes` when it exceeds
// the 48 KB default (host-side attribute call, cached per kernel).
void ensure_smem(const void* kernel, size_t bytes);

}  // namespace nufft
