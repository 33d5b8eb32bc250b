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
// Kernel weights: the reference evaluates psi(d) = exp(beta (sqrt(1 -
// (2d/w)^2) - 1)) with fp32 exp/sqrt per tap (mlx_nufft/gpu_t3.py:30-37).
// Here the W weights of a point come from per-tap polynomials in the
// point's fraction (es_weights, coefficients fitted in fp64 at plan time,
// sizing.cpp es_poly_coeffs): W*(W+2) FMAs with constant-bank operands,
// within ~1e-7 of the exact kernel.
//
// The x-weights of 3-D loops live in registers and are rotated once per
// rolled outer iteration, so no weight array is ever indexed dynamically
// (no local-memory stack frame).
#pragma once

#include <cuda_runtime.h>

#include "internal.h"

namespace nufft {

struct CellPtrs {
    const int2* d[3];
};

// Wait for the grid this one depends on (programmatic dependent launch;
// a no-op for a normal launch).
__device__ __forceinline__ void grid_dep_wait() {
    asm volatile("griddepcontrol.wait;" ::: "memory");
}

// Exact ES kernel in fp32 (reference form, kept for checks).
__device__ __forceinline__ float es_weight(float d, float c2w, float beta) {
    float z = d * c2w;
    float t = fmaxf(1.0f - z * z, 0.0f);
    return expf(beta * (sqrtf(t) - 1.0f));
}

// All W weights psi(l - fr), l = 0..W-1, from the plan's per-tap
// polynomials p_l(t), t = fr - (W/2 - 1/2).  The ES kernel is even, so
// p_{W-1-l}(t) = p_l(-t): splitting p_l(t) = E_l(t^2) + t O_l(t^2) gives
// both mirrored taps from one Horner pass each over the even and the odd
// coefficients (about half the FMAs of W separate evaluations).  The
// middle tap of an odd width is even in t and uses E alone.
template <int W>
__device__ __forceinline__ void es_weights(float fr, const EsPoly& P,
                                           float* wt) {
    constexpr int D = es_degree(W);
    constexpr int KE = D - (D & 1);          // highest even power
    constexpr int KO = D - 1 + (D & 1);      // highest odd power
    const float t = fr - (0.5f * W - 0.5f);
    const float u = t * t;
#pragma unroll
    for (int l = 0; l < (W + 1) / 2; ++l) {
        float e = P.c[KE][l];
#pragma unroll
        for (int k = KE - 2; k >= 0; k -= 2) e = fmaf(e, u, P.c[k][l]);
        if (2 * l + 1 == W) {
            wt[l] = e;
        } else {
            float o = P.c[KO][l];
#pragma unroll
            for (int k = KO - 2; k >= 1; k -= 2) o = fmaf(o, u, P.c[k][l]);
            wt[l] = fmaf(t, o, e);
            wt[W - 1 - l] = fmaf(-t, o, e);
        }
    }
}

// Weights by the plan's evaluation method: per-tap polynomials (keval 1)
// or the exact exp/sqrt form of the reference (keval 0).
template <int W>
__device__ __forceinline__ void kernel_weights(float fr, const TileGeom& tg,
                                               float* wt) {
    if (tg.keval) {
        es_weights<W>(fr, tg.poly, wt);
    } else {
#pragma unroll
        for (int l = 0; l < W; ++l)
            wt[l] = es_weight((float)l - fr, tg.c2w, tg.beta);
    }
}

// L2 evict-last policy for scattered output stores: a sorted-order interp
// writes each caller-order output sector from several subproblems at
// different times; keeping those lines resident lets L2 merge the partial
// sectors instead of write-allocating each one from DRAM.
__device__ __forceinline__ uint64_t l2_evict_last_policy() {
    uint64_t pol;
    asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;"
                 : "=l"(pol));
    return pol;
}

__device__ __forceinline__ void st_keep(float2* p, float2 v, uint64_t pol) {
    asm volatile("st.global.L2::cache_hint.v2.f32 [%0], {%1, %2}, %3;"
                 :: "l"(p), "f"(v.x), "f"(v.y), "l"(pol) : "memory");
}

// Fine-grid element loads: the grid is complex64 (float2) or, with the
// fp64 FFT mode, complex128 (double2); either way the taps are fp32.
__device__ __forceinline__ float2 load_cell(const float2* p) { return __ldg(p); }
__device__ __forceinline__ float2 load_cell(const double2* p) {
    const double2 v = __ldg(p);
    return make_float2((float)v.x, (float)v.y);
}

// Cyclic left rotation by one (compile-time indices only).
template <int W, typename T>
__device__ __forceinline__ void rotate(T* a) {
    const T first = a[0];
#pragma unroll
    for (int l = 0; l < W - 1; ++l) a[l] = a[l + 1];
    a[W - 1] = first;
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

// Periodic wrap of a tile coordinate: one compare in the common case
// (tile cells lie within one period of [0, n)), remainder otherwise.
__device__ __forceinline__ int wrap_tile(int x, int n) {
    return ((unsigned)x < (unsigned)n) ? x : wrapmod(x, n);
}

// Global linear cell of tile index q (row-major over T, last dimension
// fastest), with periodic wrap.  q / T[d] by multiply-high with the
// plan's reciprocal tdiv[d] = ceil(2^32 / T[d]) (exact for q T[d] < 2^32).
// 3-D: in the grid's stored layout (halo offsets lo, extents P; without a
// halo lo = 0 and P = n).
template <int DIM>
__device__ __forceinline__ int64_t tile_to_global(int q, const int* o,
                                                  const TileGeom& tg) {
    if constexpr (DIM == 1) {
        return wrap_tile(o[0] + q, tg.n[0]);
    } else if constexpr (DIM == 2) {
        const int r = (int)__umulhi((unsigned)q, tg.tdiv[1]);
        const int x = q - r * tg.T[1];
        return (int64_t)wrap_tile(o[0] + r, tg.n[0]) * tg.n[1] +
               wrap_tile(o[1] + x, tg.n[1]);
    } else {
        const int r = (int)__umulhi((unsigned)q, tg.tdiv[2]);
        const int x = q - r * tg.T[2];
        const int z = (int)__umulhi((unsigned)r, tg.tdiv[1]);
        const int y = r - z * tg.T[1];
        return ((int64_t)(wrap_tile(o[0] + z, tg.n[0]) + tg.lo[0]) * tg.P[1] +
                wrap_tile(o[1] + y, tg.n[1]) + tg.lo[1]) * tg.P[2] +
               wrap_tile(o[2] + x, tg.n[2]) + tg.lo[2];
    }
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
        kernel_weights<W>(__int_as_float(cl.y), tg, wgt[d]);
    }
    return ok;
}

// --------------------------------------------------------------------
// shared-tile accumulate / gather of one point (cv already weighted by the
// point's phase).  tv: interleaved complex tile as floats.
template <int DIM, int W>
__device__ __forceinline__ void tile_add(float* tv, const TileGeom& tg,
                                         const int (&l0)[DIM],
                                         float (&wgt)[DIM][W], float2 cv) {
    if constexpr (DIM == 1) {
#pragma unroll
        for (int a = 0; a < W; ++a) {
            const int q = 2 * (l0[0] + a);
            atomicAdd(tv + q, cv.x * wgt[0][a]);
            atomicAdd(tv + q + 1, cv.y * wgt[0][a]);
        }
    } else if constexpr (DIM == 2) {
#pragma unroll
        for (int a = 0; a < W; ++a) {
            const float2 ca = make_float2(cv.x * wgt[0][a], cv.y * wgt[0][a]);
            const int row = (l0[0] + a) * tg.T[1] + l0[1];
#pragma unroll
            for (int b = 0; b < W; ++b) {
                const int q = 2 * (row + b);
                atomicAdd(tv + q, ca.x * wgt[1][b]);
                atomicAdd(tv + q + 1, ca.y * wgt[1][b]);
            }
        }
    } else {
        const int plane = tg.T[1] * tg.T[2];
        int base = l0[0] * plane + l0[1] * tg.T[2] + l0[2];
#pragma unroll 1
        for (int a = 0; a < W; ++a, base += plane) {
            const float wa = wgt[0][0];
            const float2 ca = make_float2(cv.x * wa, cv.y * wa);
#pragma unroll
            for (int b = 0; b < W; ++b) {
                const float2 cab = make_float2(ca.x * wgt[1][b], ca.y * wgt[1][b]);
                const int q0 = 2 * (base + b * tg.T[2]);
#pragma unroll
                for (int k = 0; k < W; ++k) {
                    atomicAdd(tv + q0 + 2 * k, cab.x * wgt[2][k]);
                    atomicAdd(tv + q0 + 2 * k + 1, cab.y * wgt[2][k]);
                }
            }
            rotate<W>(wgt[0]);
        }
    }
}

template <int DIM, int W>
__device__ __forceinline__ float2 tile_gather(const float2* tv,
                                              const TileGeom& tg,
                                              const int (&l0)[DIM],
                                              float (&wgt)[DIM][W]) {
    float2 acc = make_float2(0.0f, 0.0f);
    if constexpr (DIM == 1) {
#pragma unroll
        for (int a = 0; a < W; ++a) {
            const float2 g = tv[l0[0] + a];
            acc.x = fmaf(g.x, wgt[0][a], acc.x);
            acc.y = fmaf(g.y, wgt[0][a], acc.y);
        }
    } else if constexpr (DIM == 2) {
#pragma unroll
        for (int a = 0; a < W; ++a) {
            const int row = (l0[0] + a) * tg.T[1] + l0[1];
            float2 s = make_float2(0.0f, 0.0f);
#pragma unroll
            for (int b = 0; b < W; ++b) {
                const float2 g = tv[row + b];
                s.x = fmaf(g.x, wgt[1][b], s.x);
                s.y = fmaf(g.y, wgt[1][b], s.y);
            }
            acc.x = fmaf(s.x, wgt[0][a], acc.x);
            acc.y = fmaf(s.y, wgt[0][a], acc.y);
        }
    } else {
        const int plane = tg.T[1] * tg.T[2];
        int base = l0[0] * plane + l0[1] * tg.T[2] + l0[2];
#pragma unroll 1
        for (int a = 0; a < W; ++a, base += plane) {
            float2 sa = make_float2(0.0f, 0.0f);
#pragma unroll
            for (int b = 0; b < W; ++b) {
                const float2* row = tv + base + b * tg.T[2];
                float2 s = make_float2(0.0f, 0.0f);
#pragma unroll
                for (int k = 0; k < W; ++k) {
                    const float2 g = row[k];
                    s.x = fmaf(g.x, wgt[2][k], s.x);
                    s.y = fmaf(g.y, wgt[2][k], s.y);
                }
                sa.x = fmaf(s.x, wgt[1][b], sa.x);
                sa.y = fmaf(s.y, wgt[1][b], sa.y);
            }
            acc.x = fmaf(sa.x, wgt[0][0], acc.x);
            acc.y = fmaf(sa.y, wgt[0][0], acc.y);
            rotate<W>(wgt[0]);
        }
    }
    return acc;
}

// --------------------------------------------------------------------
// Dynamic subproblem scheduler of the persistent tiled kernels.  sched[0]
// hands out subproblem indices; sched[1] counts CTAs that found no more
// work; the last such CTA resets both, so the next launch on the stream
// starts from zero without a memset.
__device__ __forceinline__ int next_subproblem(int* sched, int* s_sub) {
    if (threadIdx.x == 0) *s_sub = atomicAdd(&sched[0], 1);
    __syncthreads();
    return *s_sub;
}

__device__ __forceinline__ void scheduler_done(int* sched) {
    if (threadIdx.x == 0) {
        __threadfence();
        if (atomicAdd(&sched[1], 1) == (int)gridDim.x - 1) {
            atomicExch(&sched[0], 0);
            atomicExch(&sched[1], 0);
        }
    }
}

// Points of a subproblem are processed in batches of U per thread: the
// loads of a whole batch (cells, permutation, phase: streamed once, so
// cache-streaming hints) are issued before any of its math, keeping U
// independent DRAM requests in flight per thread.
#ifndef NUFFT_U_1D
#define NUFFT_U_1D 4
#endif
template <int DIM>
__host__ __device__ constexpr int batch_u() {
    return DIM == 3 ? 2 : (DIM == 1 ? NUFFT_U_1D : 4);
}

// --------------------------------------------------------------------
// tiled spread, 3-D: plane-owned shared tile, no shared-memory atomics.
//
// Float atomicAdd on shared memory is a load / compare-and-swap loop on this
// GPU (8 conflict-free lane-ops per clock per SM, far fewer when a CTA's
// warps update one small tile).  Here warp k of the CTA owns the tile
// planes z (dimension 0) with z mod 8 == k, and only warp k ever writes
// them, so a plain shared load / FMA / store cannot race: a point touches
// W <= 8 consecutive planes, i.e. at most one plane per warp (W > 8: at
// most two), and within a plane the lanes take distinct (y, x) taps.
// __syncwarp() orders one point's stores before the next point's loads.
// The in-plane taps are spread over the lanes by the plan's table
// (TileGeom::tapmap) with the shared rows padded to stride S2, so the 16
// accesses of each half-warp fall on distinct bank pairs.
//
// Points are staged 128 at a time: one thread per point computes its tile
// offset, its 3 x W kernel weights and its NV strengths (times the phase)
// into shared memory; then every warp walks the staged points and updates
// its plane of each.  The flush adds the tile to the fine grid with one
// float2 global atomic per touched cell.
constexpr int kPlaneWarps = 8;
constexpr int kPlaneChunk = 128;

// Static shared memory of k_spread_planes<W, NV, PRE> (bytes, within 64).
__host__ __device__ constexpr size_t plane_static_bytes(int W, int NV, bool pre) {
    return (size_t)kPlaneChunk *
               (8 + 4 * (pre ? W : 3 * W) +
                4 * (pre ? (((W * W) & 1) ? W * W : W * W + 1) : 1) + 8 * NV) +
           64;
}

// Vector pairs (NUFFT_PLANE_PAIR, default 1; an even NV): the tile holds
// two vectors per 16-byte cell ([NV/2][T0][T1][S4] float4), so a tap round
// is one 16-byte load / store per pair instead of one 8-byte one per
// vector: a quarter of the load / store instructions saved, and a round
// with few active lanes (W^2 mod 32 taps) moves half the wavefronts.
#ifndef NUFFT_PLANE_PAIR
#define NUFFT_PLANE_PAIR 1
#endif

template <int W, int NV, bool PRE>
__global__ void __launch_bounds__(32 * kPlaneWarps)
k_spread_planes(const float2* __restrict__ c, int64_t cstride,
                const uint32_t* __restrict__ perm, CellPtrs cells,
                const float2* __restrict__ phase, const int4* __restrict__ subs,
                int nsub, int* __restrict__ sched, float2* __restrict__ grid,
                TileGeom tg) {
    constexpr int W2 = W * W;
    constexpr int NR = (W2 + 31) / 32;               // rounds per plane
    static_assert(NR <= kMaxTapRounds, "tap table too small");
    constexpr bool PAIR = NUFFT_PLANE_PAIR && NV % 2 == 0;
    constexpr int NT = PAIR ? NV / 2 : NV;           // tiles (vector pairs or vectors)
    // PRE: the staging thread also forms the W^2 in-plane weight products,
    // so a lane reads one product per round instead of two factors (rows of
    // an odd stride: the staging stores are conflict-free); it costs
    // 4 W^2 bytes of shared memory per staged point
    static_assert(!PRE || W <= 8, "weight products staged for W <= 8 only");
    constexpr int WS = PRE ? ((W2 & 1) ? W2 : W2 + 1) : 1;
    extern __shared__ __align__(16) float2 tile[];   // [NV][T0][T1][S2] or pairs
    float4* tile4 = reinterpret_cast<float4*>(tile); // [NV/2][T0][T1][S4]
    __shared__ int2 s_pos[kPlaneChunk];              // (l0z or -1, in-plane offset)
    __shared__ float s_w[kPlaneChunk][PRE ? W : 3 * W];
    __shared__ float s_wyx[kPlaneChunk][WS];
    __shared__ __align__(16) float2 s_c[kPlaneChunk][NV];
    __shared__ int s_sub;
    const int T = tg.tcells;
    const int S2 = PAIR ? tg.S4 : tg.S2, TT = tg.T[1] * S2;
    const int TS = tg.T[0] * TT;                     // padded cells per tile
    const uint8_t* tapmap = PAIR ? tg.tapmap4 : tg.tapmap;
    const int wid = threadIdx.x >> 5;
    // this lane's (y, x) tap in each round: its offset inside a plane and
    // its index b * W + k among the in-plane taps
    int rb[NR], rk[NR], roff[NR];
    bool ract[NR];
#pragma unroll
    for (int r = 0; r < NR; ++r) {
        const int m = tapmap[r * 32 + (threadIdx.x & 31)];
        ract[r] = m != 0xff;
        rb[r] = ract[r] ? (m >> 4) : 0;
        rk[r] = ract[r] ? (m & 15) : 0;
        roff[r] = rb[r] * S2 + rk[r];
    }
    for (;;) {
        const int sub = next_subproblem(sched, &s_sub);    // (syncs)
        if (sub >= nsub) break;
        const int4 sb = subs[sub];
        const int start = sb.x, cnt = sb.y;
        int o[3] = {0, 0, 0};
        bin_origin<3>(sb.z, tg, o);
        // The staging thread's global loads are issued early: cells,
        // permutation and phase of the next chunk before this chunk's taps,
        // its strengths (through the permutation) before the barrier that
        // waits for the taps of the other warps.  With one vector (PF off)
        // the next chunk's loads wait for its own staging: the registers
        // they would hold across the taps cost the kernel a resident CTA.
        int2 pcl[3];
        int64_t psrc = 0;
        float2 pph = make_float2(1.0f, 0.0f);
        auto fetch = [&](int cb) {
            if (threadIdx.x < min(kPlaneChunk, cnt - cb)) {
                const int64_t j = start + cb + threadIdx.x;
#pragma unroll
                for (int d = 0; d < 3; ++d) pcl[d] = __ldg(cells.d[d] + j);
                psrc = perm ? (int64_t)__ldg(perm + j) : j;
                if (phase) pph = __ldg(phase + j);
            }
        };
        constexpr bool PF = NV >= 2;
        if constexpr (PF) fetch(0);
        for (int q = threadIdx.x; q < NV * TS; q += blockDim.x)
            tile[q] = make_float2(0.0f, 0.0f);
        for (int c0 = 0; c0 < cnt; c0 += kPlaneChunk) {
            const int n = min(kPlaneChunk, cnt - c0);
            float2 pcv[NV];
            if constexpr (PF) {
                if (threadIdx.x < n) {
#pragma unroll
                    for (int v = 0; v < NV; ++v) pcv[v] = __ldg(c + v * cstride + psrc);
                }
            }
            __syncthreads();      // tile zeroed / previous chunk consumed
            if (threadIdx.x < n) {
                const int p = threadIdx.x;
                if constexpr (!PF) {
                    fetch(c0);
#pragma unroll
                    for (int v = 0; v < NV; ++v) pcv[v] = __ldg(c + v * cstride + psrc);
                }
                int l0[3];
                bool ok = true;
                float wt[3][W];
#pragma unroll
                for (int d = 0; d < 3; ++d) {
                    const int2 cl = pcl[d];
                    l0[d] = cl.x - o[d];
                    ok &= (unsigned)l0[d] < (unsigned)tg.m[d];
                    kernel_weights<W>(__int_as_float(cl.y), tg, wt[d]);
                }
                if constexpr (PRE) {
#pragma unroll
                    for (int l = 0; l < W; ++l) s_w[p][l] = wt[0][l];
#pragma unroll
                    for (int b = 0; b < W; ++b)
#pragma unroll
                        for (int k = 0; k < W; ++k) s_wyx[p][b * W + k] = wt[1][b] * wt[2][k];
                } else {
#pragma unroll
                    for (int d = 0; d < 3; ++d)
#pragma unroll
                        for (int l = 0; l < W; ++l) s_w[p][d * W + l] = wt[d][l];
                }
                // l0z = -1 marks a point outside the bin (never for
                // consistent setpts output): every warp skips it
                s_pos[p] = make_int2(ok ? l0[0] : -1, l0[1] * S2 + l0[2]);
#pragma unroll
                for (int v = 0; v < NV; ++v) s_c[p][v] = phase ? cmul(pcv[v], pph) : pcv[v];
            }
            __syncthreads();
            if (PF && c0 + kPlaneChunk < cnt) fetch(c0 + kPlaneChunk);
            for (int p = 0; p < n; ++p) {
                const int2 pos = s_pos[p];
                const int l0z = pos.x;
                if (l0z < 0) continue;
                // planes z = l0z + a owned by this warp: a = (wid - l0z) mod 8
                for (int a = (wid - l0z) & (kPlaneWarps - 1); a < W; a += kPlaneWarps) {
                    const float wa = s_w[p][a];
                    const int base = (l0z + a) * TT + pos.y;
                    float2 cv[NV];
                    if constexpr (NV % 2 == 0) {
                        const float4* c4 = reinterpret_cast<const float4*>(&s_c[p][0]);
#pragma unroll
                        for (int v = 0; v < NV / 2; ++v) {
                            const float4 q = c4[v];
                            cv[2 * v] = make_float2(q.x * wa, q.y * wa);
                            cv[2 * v + 1] = make_float2(q.z * wa, q.w * wa);
                        }
                    } else {
#pragma unroll
                        for (int v = 0; v < NV; ++v) {
                            const float2 cc = s_c[p][v];
                            cv[v] = make_float2(cc.x * wa, cc.y * wa);
                        }
                    }
                    float wr[NR];
                    int q[NR];
#pragma unroll
                    for (int r = 0; r < NR; ++r) {
                        if constexpr (PRE)
                            wr[r] = s_wyx[p][rb[r] * W + rk[r]];
                        else
                            wr[r] = s_w[p][W + rb[r]] * s_w[p][2 * W + rk[r]];
                        q[r] = base + roff[r];
                    }
                    if constexpr (PAIR) {
                        float4 g[NR][NT];
#pragma unroll
                        for (int r = 0; r < NR; ++r)
                            if (ract[r])
#pragma unroll
                                for (int v = 0; v < NT; ++v) g[r][v] = tile4[v * TS + q[r]];
#pragma unroll
                        for (int r = 0; r < NR; ++r)
                            if (ract[r])
#pragma unroll
                                for (int v = 0; v < NT; ++v) {
                                    g[r][v].x = fmaf(cv[2 * v].x, wr[r], g[r][v].x);
                                    g[r][v].y = fmaf(cv[2 * v].y, wr[r], g[r][v].y);
                                    g[r][v].z = fmaf(cv[2 * v + 1].x, wr[r], g[r][v].z);
                                    g[r][v].w = fmaf(cv[2 * v + 1].y, wr[r], g[r][v].w);
                                    tile4[v * TS + q[r]] = g[r][v];
                                }
                    } else {
                        float2 g[NR][NV];
#pragma unroll
                        for (int r = 0; r < NR; ++r)
                            if (ract[r])
#pragma unroll
                                for (int v = 0; v < NV; ++v) g[r][v] = tile[v * TS + q[r]];
#pragma unroll
                        for (int r = 0; r < NR; ++r)
                            if (ract[r])
#pragma unroll
                                for (int v = 0; v < NV; ++v) {
                                    g[r][v].x = fmaf(cv[v].x, wr[r], g[r][v].x);
                                    g[r][v].y = fmaf(cv[v].y, wr[r], g[r][v].y);
                                    tile[v * TS + q[r]] = g[r][v];
                                }
                    }
                }
                __syncwarp();
            }
        }
        __syncthreads();
        for (int q = threadIdx.x; q < T; q += blockDim.x) {
            const int64_t g = tile_to_global<3>(q, o, tg);
            // shared index of tile cell q: row q / T2 at stride S2
            const int row = (int)__umulhi((unsigned)q, tg.tdiv[2]);
            const int sq = row * S2 + (q - row * tg.T[2]);
            if constexpr (PAIR) {
#pragma unroll
                for (int v = 0; v < NT; ++v) {
                    const float4 val = tile4[v * TS + sq];
                    if (val.x != 0.0f || val.y != 0.0f)
                        atomicAdd(grid + 2 * v * tg.ncells + g, make_float2(val.x, val.y));
                    if (val.z != 0.0f || val.w != 0.0f)
                        atomicAdd(grid + (2 * v + 1) * tg.ncells + g, make_float2(val.z, val.w));
                }
            } else {
#pragma unroll
                for (int v = 0; v < NV; ++v) {
                    const float2 val = tile[v * TS + sq];
                    if (val.x != 0.0f || val.y != 0.0f)
                        atomicAdd(grid + v * tg.ncells + g, val);
                }
            }
        }
    }
    scheduler_done(sched);
}

// Resident CTAs per SM the tiled interpolation is compiled for: caps its
// registers at 64 so four 256-thread CTAs fit an SM (its tile needs at
// most a quarter of the shared memory).
#ifndef NUFFT_INTERP_MINB
#define NUFFT_INTERP_MINB 4
#endif

// --------------------------------------------------------------------
// tiled spread, 1-D / 2-D: grid[v] += sum_j c[v][perm j] * phase_j *
// psi(taps); one thread per point, float shared atomics into an
// interleaved tile (a 1-D / 2-D point has few taps, and this is the
// fastest form measured for them).
template <int DIM, int W>
__global__ void __launch_bounds__(256)
k_spread_tiled(const float2* __restrict__ c, int64_t cstride, int nvg,
               const uint32_t* __restrict__ perm, CellPtrs cells,
               const float2* __restrict__ phase, const int4* __restrict__ subs,
               int nsub, int* __restrict__ sched, float2* __restrict__ grid,
               TileGeom tg) {
    extern __shared__ float2 tile[];
    __shared__ int s_sub;
    constexpr int U = batch_u<DIM>();
    const int T = tg.tcells;
    for (;;) {
        const int sub = next_subproblem(sched, &s_sub);
        if (sub >= nsub) break;
        const int4 sb = subs[sub];
        const int start = sb.x, cnt = sb.y;
        int o[3] = {0, 0, 0};
        bin_origin<DIM>(sb.z, tg, o);
        for (int q = threadIdx.x; q < nvg * T; q += blockDim.x)
            tile[q] = make_float2(0.0f, 0.0f);
        __syncthreads();
        {
        for (int base = 0; base < cnt; base += U * blockDim.x) {
            int2 cl[U][DIM];
            int64_t src[U];
            float2 ph[U];
#pragma unroll
            for (int u = 0; u < U; ++u) {
                const int t = base + u * blockDim.x + threadIdx.x;
                const int64_t j = start + min(t, cnt - 1);
#pragma unroll
                for (int d = 0; d < DIM; ++d) cl[u][d] = __ldcs(cells.d[d] + j);
                src[u] = perm ? (int64_t)__ldcs(perm + j) : j;
                ph[u] = phase ? __ldcs(phase + j) : make_float2(1.0f, 0.0f);
            }
#pragma unroll
            for (int u = 0; u < U; ++u) {
                if (base + u * (int)blockDim.x + (int)threadIdx.x >= cnt) break;
                float wgt[DIM][W];
                int l0[DIM];
                bool ok = true;
#pragma unroll
                for (int d = 0; d < DIM; ++d) {
                    l0[d] = cl[u][d].x - o[d];
                    ok &= (unsigned)l0[d] < (unsigned)tg.m[d];
                    kernel_weights<W>(__int_as_float(cl[u][d].y), tg, wgt[d]);
                }
                if (!ok) continue;
                for (int v = 0; v < nvg; ++v) {
                    float2 cv = __ldg(c + v * cstride + src[u]);
                    if (phase) cv = cmul(cv, ph[u]);
                    tile_add<DIM, W>(reinterpret_cast<float*>(tile + v * T), tg,
                                     l0, wgt, cv);
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
        __syncthreads();
    }
    scheduler_done(sched);
}

// --------------------------------------------------------------------
// tiled interp: out[v][perm j] = phase_j * sum taps tile[v] * psi-tensor
template <int DIM, int W, typename G>
__global__ void __launch_bounds__(256, NUFFT_INTERP_MINB)
k_interp_tiled(const G* __restrict__ grid, int nvg,
               const uint32_t* __restrict__ perm, CellPtrs cells,
               const float2* __restrict__ phase, const int4* __restrict__ subs,
               int nsub, int* __restrict__ sched, float2* __restrict__ out,
               int64_t ostride, TileGeom tg) {
    extern __shared__ float2 tile[];
    __shared__ int s_sub;
    constexpr int U = batch_u<DIM>();
    const int T = tg.tcells;
    const uint64_t pol = l2_evict_last_policy();
    for (;;) {
        const int sub = next_subproblem(sched, &s_sub);
        if (sub >= nsub) break;
        const int4 sb = subs[sub];
        const int start = sb.x, cnt = sb.y;
        int o[3] = {0, 0, 0};
        bin_origin<DIM>(sb.z, tg, o);
        for (int q = threadIdx.x; q < T; q += blockDim.x) {
            const int64_t g = tile_to_global<DIM>(q, o, tg);
            for (int v = 0; v < nvg; ++v)
                tile[v * T + q] = load_cell(grid + v * tg.pcells + g);
        }
        __syncthreads();
        for (int base = 0; base < cnt; base += U * blockDim.x) {
            int2 cl[U][DIM];
            int64_t dst[U];
            float2 ph[U];
#pragma unroll
            for (int u = 0; u < U; ++u) {
                const int t = base + u * blockDim.x + threadIdx.x;
                const int64_t j = start + min(t, cnt - 1);
#pragma unroll
                for (int d = 0; d < DIM; ++d) cl[u][d] = __ldcs(cells.d[d] + j);
                dst[u] = perm ? (int64_t)__ldcs(perm + j) : j;
                ph[u] = phase ? __ldcs(phase + j) : make_float2(1.0f, 0.0f);
            }
#pragma unroll
            for (int u = 0; u < U; ++u) {
                if (base + u * (int)blockDim.x + (int)threadIdx.x >= cnt) break;
                float wgt[DIM][W];
                int l0[DIM];
                bool ok = true;
#pragma unroll
                for (int d = 0; d < DIM; ++d) {
                    l0[d] = cl[u][d].x - o[d];
                    ok &= (unsigned)l0[d] < (unsigned)tg.m[d];
                    kernel_weights<W>(__int_as_float(cl[u][d].y), tg, wgt[d]);
                }
                for (int v = 0; v < nvg; ++v) {
                    float2 acc = make_float2(0.0f, 0.0f);
                    if (ok) {
                        acc = tile_gather<DIM, W>(tile + v * T, tg, l0, wgt);
                        if (phase) acc = cmul(acc, ph[u]);
                    }
                    if (perm)
                        st_keep(out + v * ostride + dst[u], acc, pol);
                    else
                        out[v * ostride + dst[u]] = acc;
                }
            }
        }
        __syncthreads();
    }
    scheduler_done(sched);
}

// --------------------------------------------------------------------
// global-memory variants: one thread per point (sorted or caller order).
// Tap indices are in the grid's stored layout (lo, P; 3-D grids may carry
// a periodic halo).
template <int DIM, int W>
__device__ __forceinline__ void global_taps(const CellPtrs& cells, int64_t j,
                                            const TileGeom& tg,
                                            float (&wgt)[DIM][W],
                                            int (&idx)[DIM][W]) {
#pragma unroll
    for (int d = 0; d < DIM; ++d) {
        int2 cl = __ldg(cells.d[d] + j);
        kernel_weights<W>(__int_as_float(cl.y), tg, wgt[d]);
#pragma unroll
        for (int l = 0; l < W; ++l) idx[d][l] = wrap1(cl.x + l, tg.n[d]) + tg.lo[d];
    }
}

// grid[...] += cv * psi-tensor with global float2 atomics
template <int DIM, int W>
__device__ __forceinline__ void global_add(float2* gv, const TileGeom& tg,
                                           float (&wgt)[DIM][W],
                                           int (&idx)[DIM][W], float2 cv) {
    if constexpr (DIM == 1) {
#pragma unroll
        for (int a = 0; a < W; ++a)
            atomicAdd(gv + idx[0][a], make_float2(cv.x * wgt[0][a], cv.y * wgt[0][a]));
    } else if constexpr (DIM == 2) {
#pragma unroll
        for (int a = 0; a < W; ++a) {
            const int64_t row = (int64_t)idx[0][a] * tg.n[1];
#pragma unroll
            for (int b = 0; b < W; ++b) {
                const float wab = wgt[0][a] * wgt[1][b];
                atomicAdd(gv + row + idx[1][b], make_float2(cv.x * wab, cv.y * wab));
            }
        }
    } else {
#pragma unroll 1
        for (int a = 0; a < W; ++a) {
            const int64_t plane = (int64_t)idx[0][0] * tg.P[1];
            const float wa = wgt[0][0];
#pragma unroll
            for (int b = 0; b < W; ++b) {
                const float wab = wa * wgt[1][b];
                const int64_t base = (plane + idx[1][b]) * tg.P[2];
#pragma unroll
                for (int k = 0; k < W; ++k) {
                    const float wk = wab * wgt[2][k];
                    atomicAdd(gv + base + idx[2][k], make_float2(cv.x * wk, cv.y * wk));
                }
            }
            rotate<W>(wgt[0]);
            rotate<W>(idx[0]);
        }
    }
}

template <int DIM, int W, typename G>
__device__ __forceinline__ float2 global_gather(const G* gv,
                                                const TileGeom& tg,
                                                float (&wgt)[DIM][W],
                                                int (&idx)[DIM][W]) {
    float2 acc = make_float2(0.0f, 0.0f);
    if constexpr (DIM == 1) {
#pragma unroll
        for (int a = 0; a < W; ++a) {
            const float2 g = load_cell(gv + idx[0][a]);
            acc.x = fmaf(g.x, wgt[0][a], acc.x);
            acc.y = fmaf(g.y, wgt[0][a], acc.y);
        }
    } else if constexpr (DIM == 2) {
#pragma unroll
        for (int a = 0; a < W; ++a) {
            const int64_t row = (int64_t)idx[0][a] * tg.n[1];
            float2 s = make_float2(0.0f, 0.0f);
#pragma unroll
            for (int b = 0; b < W; ++b) {
                const float2 g = load_cell(gv + row + idx[1][b]);
                s.x = fmaf(g.x, wgt[1][b], s.x);
                s.y = fmaf(g.y, wgt[1][b], s.y);
            }
            acc.x = fmaf(s.x, wgt[0][a], acc.x);
            acc.y = fmaf(s.y, wgt[0][a], acc.y);
        }
    } else {
#pragma unroll 1
        for (int a = 0; a < W; ++a) {
            const int64_t plane = (int64_t)idx[0][0] * tg.P[1];
            float2 sa = make_float2(0.0f, 0.0f);
#pragma unroll
            for (int b = 0; b < W; ++b) {
                const G* row = gv + (plane + idx[1][b]) * tg.P[2];
                float2 s = make_float2(0.0f, 0.0f);
#pragma unroll
                for (int k = 0; k < W; ++k) {
                    const float2 g = load_cell(row + idx[2][k]);
                    s.x = fmaf(g.x, wgt[2][k], s.x);
                    s.y = fmaf(g.y, wgt[2][k], s.y);
                }
                sa.x = fmaf(s.x, wgt[1][b], sa.x);
                sa.y = fmaf(s.y, wgt[1][b], sa.y);
            }
            acc.x = fmaf(sa.x, wgt[0][0], acc.x);
            acc.y = fmaf(sa.y, wgt[0][0], acc.y);
            rotate<W>(wgt[0]);
            rotate<W>(idx[0]);
        }
    }
    return acc;
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
        global_add<DIM, W>(grid + v * tg.ncells, tg, wgt, idx, cv);
    }
}

template <int DIM, int W, typename G>
__global__ void __launch_bounds__(256)
k_interp_global(const G* __restrict__ grid, int nvec,
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
        float2 acc = global_gather<DIM, W, G>(grid + v * tg.pcells, tg, wgt, idx);
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

}  // namespace nufft
