// interp_tma.cu -- 3-D tiled interpolation with TMA-staged, double-buffered
// grid tiles (types 2 and 3, complex64 fine grid).
//
// The plain tiled kernel (k_interp_tiled) loads each subproblem's tile with
// per-thread loads (index arithmetic per cell, then a barrier) before any
// point can be processed; in 3-D at low density (tens of points per 8^3
// bin, e.g. the uniform half of a clustered set) that load dominates.  Here
// one thread issues the whole tile as one bulk tensor copy per vector
// (cp.async.bulk.tensor, completion on an mbarrier) for the NEXT
// subproblem while the CTA interpolates the current one from the other
// buffer.
//
// Tensor map: the plan's nbatch fine grids as a 4-D array (x, y, z, vector)
// of 8-byte elements (complex64).  A TMA copy must start at a 16-byte
// boundary in x, so each tile box starts at the even cell x0 = o_x rounded
// down and is B2 = T2 + 1 rounded up to even cells wide; the point
// arithmetic adds the offset o_x - x0 (0 or 1).  A grid stored with a
// periodic halo (TileGeom lo / P; the pruned 3-D FFT writes one for type 2)
// holds every tile box; otherwise bins whose tile would wrap around the
// periodic grid are loaded by the CTA's threads with wrap, into the same
// padded layout.
//
// Every mbarrier wait is bounded: after kSpinLimit polls the CTA records
// an error in *err (the plan's host-mapped execute error flag, which the
// next call on the plan reports), waits (bounded again) for both of its
// buffers' copies, and stops.
#include <cuda.h>

#include <algorithm>
#include <cstdlib>
#include <mutex>

#include "spreadinterp.cuh"

namespace nufft {

namespace {

constexpr int kSpinLimit = 1 << 22;

// Threads per CTA of the 3-D TMA-staged interpolation and resident CTAs per
// SM it is compiled for (80 registers): two 384-thread CTAs with two
// 18 x 18 x 20-cell buffers each per SM (3-D type 2, 256^3 modes, 5e7
// clustered points: interp 5.29 ms vs 5.38 with 256 threads).
#ifndef NUFFT_TMA_MINB
#define NUFFT_TMA_MINB 2
#endif
#ifndef NUFFT_TMA_THREADS
#define NUFFT_TMA_THREADS 384
#endif
// Points per thread per round of the 3-D TMA-staged interpolation (their
// global loads are issued together).
#ifndef NUFFT_TMA_U
#define NUFFT_TMA_U 2
#endif

__host__ __device__ __forceinline__ int tma_buffer_cells(const TileGeom& tg, int B2) {
    return ((tg.T[0] * tg.T[1] * B2) + 15) & ~15;
}

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
    return (uint32_t)__cvta_generic_to_shared(p);
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, int count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)),
                 "r"(count)
                 : "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile(
        "mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)),
        "r"(bytes)
        : "memory");
}

// true when the phase with parity `parity` has completed; bounded polling
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity) {
    const uint32_t a = smem_addr(bar);
    for (int it = 0; it < kSpinLimit; ++it) {
        uint32_t done;
        asm volatile(
            "{\n\t.reg .pred p;\n\t"
            "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
            "selp.u32 %0, 1, 0, p;\n\t}"
            : "=r"(done)
            : "r"(a), "r"(parity)
            : "memory");
        if (done) return true;
    }
    return false;
}

__device__ __forceinline__ void tma_load_4d(void* dst, const CUtensorMap* map,
                                            int x, int y, int z, int v,
                                            uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.4d.shared::cluster.global.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%2, %3, %4, %5}], [%6];" ::"r"(smem_addr(dst)),
        "l"(map), "r"(x), "r"(y), "r"(z), "r"(v), "r"(smem_addr(bar))
        : "memory");
}

// Record a failed (timed-out) tile copy in the plan's execute error flag.
// The flag is pinned host memory mapped into the device address space, so
// the host reads it without a device synchronisation; a plain system-scope
// store (no atomic over the host link) is enough for a single flag value.
__device__ __forceinline__ void report_tile_wait(int* err) {
    *(volatile int*)err = kErrTileWait;
    __threadfence_system();
}

// Load a tile that wraps around the periodic grid into the padded tile
// layout (rows of S cells, vector buffers TS cells apart) with `nthr`
// threads (thread `tid`): K independent loads in flight per thread before
// their stores, so the loop is bound by bandwidth, not by one load latency
// per cell.
__device__ __forceinline__ void load_wrapped_tile(float2* tile, const float2* grid,
                                                  const int* o, const TileGeom& tg,
                                                  int S, int TS, int v0, int nvg,
                                                  int tid, int nthr) {
    constexpr int K = 4;
    for (int v = 0; v < nvg; ++v) {
        const float2* gv = grid + (int64_t)(v0 + v) * tg.pcells;
        for (int q0 = tid; q0 < tg.tcells; q0 += K * nthr) {
            float2 val[K];
            int sq[K];
#pragma unroll
            for (int k = 0; k < K; ++k) {
                const int q = q0 + k * nthr;
                sq[k] = -1;
                if (q < tg.tcells) {
                    const int64_t g = tile_to_global<3>(q, o, tg);
                    const int row = (int)__umulhi((unsigned)q, tg.tdiv[2]);
                    sq[k] = row * S + (q - row * tg.T[2]);
                    val[k] = __ldg(gv + g);
                }
            }
#pragma unroll
            for (int k = 0; k < K; ++k)
                if (sq[k] >= 0) tile[v * TS + sq[k]] = val[k];
        }
    }
}

struct TmaBin {
    int o[3];        // tile origin (global cell of tile index 0), per dim
    int x0;          // box start in x (even)
    int c[3];        // box start in the stored grid (o[0], o[1], x0 + halo lo)
    bool interior;   // box inside the stored grid: TMA-loadable
};

__device__ __forceinline__ TmaBin tma_bin(int bin, const TileGeom& tg, int B2,
                                          bool use_tma) {
    TmaBin b;
    bin_origin<3>(bin, tg, b.o);
    b.x0 = b.o[2] - (b.o[2] & 1);
    b.c[0] = b.o[0] + tg.lo[0];
    b.c[1] = b.o[1] + tg.lo[1];
    b.c[2] = b.x0 + tg.lo[2];
    b.interior = use_tma && b.c[0] >= 0 && b.c[0] + tg.T[0] <= tg.P[0] &&
                 b.c[1] >= 0 && b.c[1] + tg.T[1] <= tg.P[1] &&
                 b.c[2] >= 0 && b.c[2] + B2 <= tg.P[2];
    return b;
}

// taps of one point from a padded tile: rows of stride S (cells), planes
// of T1 * S; `base` is the tile index of the point's first tap
template <int W>
__device__ __forceinline__ float2 gather3(const float2* tv, int S, int PS,
                                          int base, float (&wgt)[3][W]) {
    float2 acc = make_float2(0.0f, 0.0f);
#pragma unroll 1
    for (int a = 0; a < W; ++a, base += PS) {
        float2 sa = make_float2(0.0f, 0.0f);
#pragma unroll
        for (int b = 0; b < W; ++b) {
            const float2* row = tv + base + b * S;
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
    return acc;
}

template <int W>
__global__ void __launch_bounds__(NUFFT_TMA_THREADS, NUFFT_TMA_MINB)
k_interp_tma(const __grid_constant__ CUtensorMap tmap, const float2* __restrict__ grid,
             int v0, int nvg, int B2, const uint32_t* __restrict__ perm,
             CellPtrs cells, const float2* __restrict__ phase,
             const int4* __restrict__ subs, int nsub, int* __restrict__ sched,
             float2* __restrict__ out, int64_t ostride, TileGeom tg,
             int* __restrict__ err) {
    extern __shared__ __align__(128) float2 sbuf[];     // [2][nvg][T0][T1][B2]
    __shared__ __align__(8) uint64_t bar[2];
    __shared__ int ring[2];
    __shared__ int s_tma;                                // 0: all tiles by hand
    constexpr int U = NUFFT_TMA_U;
    const int S = B2, PS = tg.T[1] * B2;
    // cells per vector buffer, rounded to 16 cells: every TMA destination
    // is 128-byte aligned
    const int TS = tma_buffer_cells(tg, B2);
    const uint32_t tile_bytes = (uint32_t)(tg.T[0] * PS) * sizeof(float2);
    const uint64_t pol = l2_evict_last_policy();
    if (threadIdx.x == 0) {
        mbar_init(&bar[0], 1);
        mbar_init(&bar[1], 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        s_tma = (smem_addr(sbuf) & 127u) == 0;
    }
    __syncthreads();
    const bool use_tma = s_tma != 0;
    auto issue = [&](const TmaBin& bn, int b) {
        // thread 0: this CTA's generic-proxy reads of buffer b are ordered
        // before the async-proxy writes by the preceding barrier + fence
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        mbar_expect_tx(&bar[b], tile_bytes * (uint32_t)nvg);
        for (int v = 0; v < nvg; ++v)
            tma_load_4d(sbuf + ((size_t)b * nvg + v) * TS, &tmap, bn.c[2], bn.c[1],
                        bn.c[0], v0 + v, &bar[b]);
    };
    // ring[b]: subproblem whose tile occupies buffer b.  Thread 0 claims two
    // ahead, so each subproblem needs one CTA barrier (which also releases
    // the buffer it consumed and agrees on a failed wait).
    if (threadIdx.x == 0) {
        for (int k = 0; k < 2; ++k) {
            ring[k] = atomicAdd(&sched[0], 1);
            if (ring[k] < nsub) {
                const TmaBin nb = tma_bin(subs[ring[k]].z, tg, B2, use_tma);
                if (nb.interior) issue(nb, k);
            }
        }
    }
    __syncthreads();
    int cur = ring[0];
    int b = 0;
    uint32_t parity0 = 0u, parity1 = 0u;
    bool failed = false;
    bool cur_interior = false;
    while (cur < nsub) {
        const int4 sb = subs[cur];
        const TmaBin bn = tma_bin(sb.z, tg, B2, use_tma);
        float2* tile = sbuf + (size_t)b * nvg * TS;
        bool ok = true;
        int xoff;
        cur_interior = bn.interior;
        if (bn.interior) {
            ok = mbar_wait(&bar[b], b ? parity1 : parity0);
            if (b) parity1 ^= 1u; else parity0 ^= 1u;
            xoff = bn.o[2] - bn.x0;
        } else {
            // wrapped tile (uniform across the CTA): per-thread loads into
            // the same padded layout
            load_wrapped_tile(tile, grid, bn.o, tg, S, TS, v0, nvg, threadIdx.x,
                              blockDim.x);
            __syncthreads();
            xoff = 0;
        }
        const int start = sb.x, cnt = sb.y;
        for (int base = 0; ok && base < cnt; base += U * blockDim.x) {
            int2 cl[U][3];
            int64_t dst[U];
            float2 ph[U];
#pragma unroll
            for (int u = 0; u < U; ++u) {
                const int t = base + u * blockDim.x + threadIdx.x;
                const int64_t j = start + min(t, cnt - 1);
#pragma unroll
                for (int d = 0; d < 3; ++d) cl[u][d] = __ldcs(cells.d[d] + j);
                dst[u] = perm ? (int64_t)__ldcs(perm + j) : j;
                ph[u] = phase ? __ldcs(phase + j) : make_float2(1.0f, 0.0f);
            }
#pragma unroll
            for (int u = 0; u < U; ++u) {
                if (base + u * (int)blockDim.x + (int)threadIdx.x >= cnt) break;
                float wgt[3][W];
                int l0[3];
                bool inb = true;
#pragma unroll
                for (int d = 0; d < 3; ++d) {
                    l0[d] = cl[u][d].x - bn.o[d];
                    inb &= (unsigned)l0[d] < (unsigned)tg.m[d];
                    kernel_weights<W>(__int_as_float(cl[u][d].y), tg, wgt[d]);
                }
                const int tb = l0[0] * PS + l0[1] * S + l0[2] + xoff;
                for (int v = 0; v < nvg; ++v) {
                    // gather3 rotates the x-weights W times: back in order
                    float2 acc = make_float2(0.0f, 0.0f);
                    if (inb) {
                        acc = gather3<W>(tile + v * TS, S, PS, tb, wgt);
                        if (phase) acc = cmul(acc, ph[u]);
                    }
                    if (perm)
                        st_keep(out + v * ostride + dst[u], acc, pol);
                    else
                        out[v * ostride + dst[u]] = acc;
                }
            }
        }
        if (__syncthreads_or(!ok)) {           // buffer b consumed by all
            failed = true;
            break;
        }
        if (threadIdx.x == 0) {                // refill buffer b, two ahead
            const int nn = atomicAdd(&sched[0], 1);
            ring[b] = nn;
            if (nn < nsub) {
                const TmaBin nb = tma_bin(subs[nn].z, tg, B2, use_tma);
                if (nb.interior) issue(nb, b);
            }
        }
        cur = ring[b ^ 1];
        b ^= 1;
    }
    if (failed && threadIdx.x == 0) {
        report_tile_wait(err);
        // neither buffer may keep a copy in flight once the CTA's shared
        // memory is released: wait again (bounded) for the copy whose wait
        // timed out (buffer b, the phase before the parity flip) and for
        // the other buffer's
        if (cur_interior) mbar_wait(&bar[b], (b ? parity1 : parity0) ^ 1u);
        const int o = ring[b ^ 1];
        if (o < nsub && tma_bin(subs[o].z, tg, B2, use_tma).interior)
            mbar_wait(&bar[b ^ 1], b ? parity0 : parity1);
    }
    scheduler_done(sched);
}

// ---------------------------------------------------------------------
// 1-D: every subproblem's inputs streamed through shared memory.
//
// A 1-D point has only W taps, so the tiled kernel's time goes to waiting
// on its own global loads (the tile, then the sorted cells and the
// permutation of its points) and to the scattered output stores.  Here
// thread 0 issues, for the NEXT subproblem, 1-D bulk async copies
// (cp.async.bulk, completion on the stage's mbarrier) of the tile (the bin
// plus halo, contiguous in the grid), the subproblem's cells, permutation
// and phases, while the CTA works on the current subproblem from the other
// stage; the warps then read only shared memory and store the results.
// Bulk copies need 16-byte-aligned ranges: each range starts at an aligned
// element at or before its first element and is rounded up (at most 3
// elements past the end of the point arrays, which carry that slack; see
// kPointSlack).  Tiles that wrap around the periodic grid are loaded by
// the CTA's threads.
constexpr int kStreamThreads = 256;

#ifndef NUFFT_STREAM_MINB
#define NUFFT_STREAM_MINB 3
#endif

__host__ __device__ __forceinline__ int align_up(int x, int a) {
    return (x + a - 1) / a * a;
}

// Byte offsets of one stage: [tile x nvg][cells][perm][phase]
struct StreamLayout {
    int tile_cells;     // per vector: T + 1 rounded up to even
    int tile_bytes;     // per vector, 128-byte multiple
    int cells_off, perm_off, phase_off, stage_bytes;
};

__host__ __device__ __forceinline__ StreamLayout stream_layout(int T, int msub,
                                                              int nvg, bool phase) {
    StreamLayout L;
    L.tile_cells = align_up(T + 1, 2);
    L.tile_bytes = align_up(L.tile_cells * 8, 128);
    L.cells_off = nvg * L.tile_bytes;
    L.perm_off = L.cells_off + align_up((msub + 2) * 8, 128);
    L.phase_off = L.perm_off + align_up((msub + 8) * 4, 128);
    L.stage_bytes = L.phase_off + (phase ? align_up((msub + 2) * 8, 128) : 0);
    return L;
}

__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes,
                                          uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes"
        " [%0], [%1], %2, [%3];" ::"r"(smem_addr(dst)),
        "l"(src), "r"(bytes), "r"(smem_addr(bar))
        : "memory");
}

struct StreamSub {
    int start, cnt, o;    // points [start, start + cnt), tile origin o
    int c0, p0;           // aligned first element of the cell / perm ranges
    int c1, p1;           // aligned ends
    bool interior;        // tile copied by the bulk engine
    int g0;               // aligned first grid cell of the tile copy
};

__device__ __forceinline__ StreamSub stream_sub(const int4& sb, const TileGeom& tg,
                                                int tile_cells) {
    StreamSub q;
    q.start = sb.x;
    q.cnt = sb.y;
    q.o = (sb.z % tg.nb[0]) * tg.m[0] - tg.halfw;
    q.g0 = q.o - (q.o & 1);
    q.interior = q.g0 >= 0 && q.g0 + tile_cells <= tg.n[0];
    q.c0 = q.start & ~1;
    q.c1 = align_up(q.start + q.cnt, 2);
    q.p0 = q.start & ~3;
    q.p1 = align_up(q.start + q.cnt, 4);
    return q;
}

template <int W>
__global__ void __launch_bounds__(kStreamThreads, NUFFT_STREAM_MINB)
k_interp1_stream(const float2* __restrict__ grid, int nvg, int msub,
                 const uint32_t* __restrict__ perm, const int2* __restrict__ cells,
                 const float2* __restrict__ phase, const int4* __restrict__ subs,
                 int nsub, int* __restrict__ sched, float2* __restrict__ out,
                 int64_t ostride, TileGeom tg, int* __restrict__ err) {
    extern __shared__ __align__(128) unsigned char sraw[];
    __shared__ __align__(8) uint64_t bar[2];
    __shared__ int ring[2];
    __shared__ int s_ok;
    grid_dep_wait();                  // the FFT that writes `grid` has completed
    const StreamLayout L = stream_layout(tg.tcells, msub, nvg, phase != nullptr);
    const uint64_t pol = l2_evict_last_policy();
    if (threadIdx.x == 0) {
        mbar_init(&bar[0], 1);
        mbar_init(&bar[1], 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        s_ok = (smem_addr(sraw) & 127u) == 0;
    }
    __syncthreads();
    if (!s_ok) {            // misaligned stage buffers: record and stop
        if (threadIdx.x == 0) report_tile_wait(err);
        scheduler_done(sched);
        return;
    }
    auto stage = [&](int b) { return sraw + (size_t)b * L.stage_bytes; };
    // thread 0: all copies of subproblem q into stage b
    auto issue = [&](const StreamSub& q, int b) {
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        unsigned char* st = stage(b);
        uint32_t bytes = (uint32_t)(q.c1 - q.c0) * 8 + (uint32_t)(q.p1 - q.p0) * 4;
        if (phase) bytes += (uint32_t)(q.c1 - q.c0) * 8;
        if (q.interior) bytes += (uint32_t)nvg * L.tile_cells * 8;
        mbar_expect_tx(&bar[b], bytes);
        if (q.interior)
            for (int v = 0; v < nvg; ++v)
                bulk_load(st + v * L.tile_bytes, grid + (int64_t)v * tg.ncells + q.g0,
                          (uint32_t)L.tile_cells * 8, &bar[b]);
        bulk_load(st + L.cells_off, cells + q.c0, (uint32_t)(q.c1 - q.c0) * 8, &bar[b]);
        bulk_load(st + L.perm_off, perm + q.p0, (uint32_t)(q.p1 - q.p0) * 4, &bar[b]);
        if (phase)
            bulk_load(st + L.phase_off, phase + q.c0, (uint32_t)(q.c1 - q.c0) * 8,
                      &bar[b]);
    };
    // ring[b]: subproblem loaded into stage b.  Thread 0 claims two ahead,
    // so each iteration needs a single CTA barrier (which also releases the
    // stage it consumed and agrees on a failed wait).
    if (threadIdx.x == 0) {
        for (int k = 0; k < 2; ++k) {
            ring[k] = atomicAdd(&sched[0], 1);
            if (ring[k] < nsub) issue(stream_sub(subs[ring[k]], tg, L.tile_cells), k);
        }
    }
    __syncthreads();
    int cur = ring[0];
    int b = 0;
    uint32_t parity0 = 0u, parity1 = 0u;
    bool failed = false;
    while (cur < nsub) {
        const StreamSub q = stream_sub(subs[cur], tg, L.tile_cells);
        const bool ok = mbar_wait(&bar[b], b ? parity1 : parity0);
        if (b) parity1 ^= 1u; else parity0 ^= 1u;
        unsigned char* st = stage(b);
        const float2* tile = reinterpret_cast<const float2*>(st);
        int xoff = q.o - q.g0;
        if (!q.interior) {                     // uniform across the CTA
            float2* tw = reinterpret_cast<float2*>(st);
            for (int c = threadIdx.x; c < tg.tcells; c += blockDim.x) {
                const int g = wrap_tile(q.o + c, tg.n[0]);
                for (int v = 0; v < nvg; ++v)
                    tw[v * (L.tile_bytes / 8) + c] = grid[(int64_t)v * tg.ncells + g];
            }
            __syncthreads();
            xoff = 0;
        }
        const int2* sc = reinterpret_cast<const int2*>(st + L.cells_off) + (q.start - q.c0);
        const uint32_t* sp = reinterpret_cast<const uint32_t*>(st + L.perm_off) +
                             (q.start - q.p0);
        const float2* sh = phase ? reinterpret_cast<const float2*>(st + L.phase_off) +
                                       (q.start - q.c0)
                                 : nullptr;
        for (int t = threadIdx.x; ok && t < q.cnt; t += blockDim.x) {
            const int2 cl = sc[t];
            const int l0 = cl.x - q.o;
            float wgt[W];
            kernel_weights<W>(__int_as_float(cl.y), tg, wgt);
            const bool inb = (unsigned)l0 < (unsigned)tg.m[0];
            const int64_t dst = sp[t];
            for (int v = 0; v < nvg; ++v) {
                float2 acc = make_float2(0.0f, 0.0f);
                if (inb) {
                    const float2* tv = tile + v * (L.tile_bytes / 8) + l0 + xoff;
#pragma unroll
                    for (int a = 0; a < W; ++a) {
                        const float2 g = tv[a];
                        acc.x = fmaf(g.x, wgt[a], acc.x);
                        acc.y = fmaf(g.y, wgt[a], acc.y);
                    }
                    if (sh) acc = cmul(acc, sh[t]);
                }
                st_keep(out + v * ostride + dst, acc, pol);
            }
        }
        if (__syncthreads_or(!ok)) {           // stage b consumed by all
            failed = true;
            break;
        }
        if (threadIdx.x == 0) {                // refill stage b, two ahead
            const int nn = atomicAdd(&sched[0], 1);
            ring[b] = nn;
            if (nn < nsub) issue(stream_sub(subs[nn], tg, L.tile_cells), b);
        }
        cur = ring[b ^ 1];
        b ^= 1;
    }
    if (failed && threadIdx.x == 0) {
        report_tile_wait(err);
        // no stage may keep a copy in flight once the CTA's shared memory is
        // released: wait again (bounded) for the stage whose wait timed out
        // (the phase before the parity flip) and for the other stage
        mbar_wait(&bar[b], (b ? parity1 : parity0) ^ 1u);
        if (ring[b ^ 1] < nsub) mbar_wait(&bar[b ^ 1], b ? parity0 : parity1);
    }
    scheduler_done(sched);
}

// cuTensorMapEncodeTiled through the runtime's driver entry point (no
// libcuda link); null when the driver does not provide it.
using EncodeTiled = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t,
                                 void*, const cuuint64_t*, const cuuint64_t*,
                                 const cuuint32_t*, const cuuint32_t*,
                                 CUtensorMapInterleave, CUtensorMapSwizzle,
                                 CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiled encode_tiled() {
    static std::once_flag once;
    static EncodeTiled fn = nullptr;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q{};
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault,
                                    &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = (EncodeTiled)p;
        cudaGetLastError();
    });
    return fn;
}

}  // namespace

int tma_box_x(const TileGeom& tg) {
    return (tg.T[2] + 2) & ~1;          // T2 + 1 rounded up to even
}

bool make_grid_tmap(CUtensorMap* map, const float2* grid, const TileGeom& tg,
                    int nbatch) {
    if (tg.dim != 3) return false;
    EncodeTiled enc = encode_tiled();
    if (!enc) return false;
    const int B2 = tma_box_x(tg);
    if (B2 > 256 || tg.T[1] > 256 || tg.T[0] > 256 || B2 > tg.P[2]) return false;
    // the stored layout: extents P (n plus the periodic halo, if any)
    const cuuint64_t dims[4] = {(cuuint64_t)tg.P[2], (cuuint64_t)tg.P[1],
                                (cuuint64_t)tg.P[0], (cuuint64_t)nbatch};
    const cuuint64_t strides[3] = {(cuuint64_t)tg.P[2] * 8,
                                   (cuuint64_t)tg.P[1] * tg.P[2] * 8,
                                   (cuuint64_t)tg.pcells * 8};
    const cuuint32_t box[4] = {(cuuint32_t)B2, (cuuint32_t)tg.T[1],
                               (cuuint32_t)tg.T[0], 1};
    const cuuint32_t estr[4] = {1, 1, 1, 1};
    const CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_UINT64, 4, (void*)grid, dims,
                           strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                           CU_TENSOR_MAP_SWIZZLE_NONE,
                           CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                           CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS;
}

__global__ void k_mark_planes(const int4* __restrict__ subs, int nsub, TileGeom tg,
                              uint8_t* __restrict__ need) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= nsub) return;
    int o[3];
    bin_origin<3>(subs[i].z, tg, o);
    const int n0 = tg.n[0];
    for (int k = 0; k < tg.T[0]; ++k) {
        need[o[0] + k + tg.lo[0]] = 1;
        need[(((o[0] + k) % n0) + n0) % n0 + tg.lo[0]] = 1;
    }
}

template <int W>
void interp_tma_impl(const PointSet& ps, const TileGeom& tg, const CUtensorMap& map,
                     const float2* grid, int nvec, float2* out, int64_t ostride,
                     int nvg, int* err, cudaStream_t st) {
    auto k = k_interp_tma<W>;
    const int B2 = tma_box_x(tg);
    const size_t per = (size_t)tma_buffer_cells(tg, B2) * sizeof(float2);
    for (int v0 = 0; v0 < nvec; v0 += nvg) {
        const int nv = std::min(nvg, nvec - v0);
        const size_t smem = 2 * nv * per;
        ensure_smem((const void*)k, smem);
        const int blocks = persistent_grid((const void*)k, smem, ps.nsub,
                                           NUFFT_TMA_THREADS);
        k<<<blocks, NUFFT_TMA_THREADS, smem, st>>>(map, grid, v0, nv, B2,
                                     ps.sorted ? ps.perm : nullptr, cell_ptrs(ps),
                                     ps.phase, ps.subs, (int)ps.nsub, ps.sched,
                                     out + v0 * ostride, ostride, tg, err);
        NUFFT_LAUNCH("k_interp_tma");
    }
}

template <int W>
void interp1_stream_impl(const PointSet& ps, const TileGeom& tg, const float2* grid,
                         int nvec, float2* out, int64_t ostride, int nvg, int msub,
                         int* err, cudaStream_t st) {
    auto k = k_interp1_stream<W>;
    const int threads = kStreamThreads, stages = 2;
    for (int v0 = 0; v0 < nvec; v0 += nvg) {
        const int nv = std::min(nvg, nvec - v0);
        const StreamLayout L = stream_layout(tg.tcells, msub, nv, ps.phase != nullptr);
        const size_t smem = stages * (size_t)L.stage_bytes;
        ensure_smem((const void*)k, smem);
        const int blocks = persistent_grid((const void*)k, smem, ps.nsub, threads);
        launch_dependent(k, dim3(blocks), dim3(threads), smem, st,
                         grid + (int64_t)v0 * tg.ncells, nv, msub, ps.perm, ps.cell[0],
                         ps.phase, ps.subs, (int)ps.nsub, ps.sched, out + v0 * ostride,
                         ostride, tg, err);
        NUFFT_LAUNCH("k_interp1_stream");
    }
}

void mark_tile_planes(const PointSet& ps, const TileGeom& tg, uint8_t* need,
                      cudaStream_t st) {
    if (ps.nsub == 0 || tg.dim != 3) return;
    const unsigned blocks = (unsigned)((ps.nsub + 255) / 256);
    k_mark_planes<<<blocks, 256, 0, st>>>(ps.subs, (int)ps.nsub, tg, need);
    NUFFT_LAUNCH("k_mark_planes");
}

bool launch_interp_tma(const PointSet& ps, const TileGeom& tg, int w,
                       const CUtensorMap* map, const float2* grid, int nvec,
                       float2* out, int64_t ostride, int* err, cudaStream_t st) {
    if (ps.tiled && ps.sorted && ps.dim == 1 && ps.msub > 0 && ps.msub <= kStreamMsubMax &&
        w <= 16 && grid) {
        if (ps.nsub == 0) return true;
        // vectors per pass: two stages within ~72 KB
        const size_t one = (size_t)stream_layout(tg.tcells, ps.msub, 1,
                                                  ps.phase != nullptr).stage_bytes;
        const int nvg = (int)std::max<size_t>(1, (36 * 1024) / one);
        NUFFT_WIDTH_SWITCH(w, interp1_stream_impl<W>(ps, tg, grid, nvec, out, ostride,
                                                     nvg, ps.msub, err, st));
        return true;
    }
    if (!map || !ps.tiled || ps.dim != 3 || w > 10) return false;
    if (ps.nsub == 0) return true;
    // two buffers of up to nvg vectors within ~100 KB: two CTAs per SM
    const size_t per = (size_t)tma_buffer_cells(tg, tma_box_x(tg)) * sizeof(float2);
    const int nvg = (int)std::max<size_t>(1, (100 * 1024) / (2 * per));
    if (2 * per > (size_t)tile_smem_limit() - 4096) return false;
    switch (w) {
        case 2: interp_tma_impl<2>(ps, tg, *map, grid, nvec, out, ostride, nvg, err, st); break;
        case 3: interp_tma_impl<3>(ps, tg, *map, grid, nvec, out, ostride, nvg, err, st); break;
        case 4: interp_tma_impl<4>(ps, tg, *map, grid, nvec, out, ostride, nvg, err, st); break;
        case 5: interp_tma_impl<5>(ps, tg, *map, grid, nvec, out, ostride, nvg, err, st); break;
        case 6: interp_tma_impl<6>(ps, tg, *map, grid, nvec, out, ostride, nvg, err, st); break;
        case 7: interp_tma_impl<7>(ps, tg, *map, grid, nvec, out, ostride, nvg, err, st); break;
        case 8: interp_tma_impl<8>(ps, tg, *map, grid, nvec, out, ostride, nvg, err, st); break;
        case 9: interp_tma_impl<9>(ps, tg, *map, grid, nvec, out, ostride, nvg, err, st); break;
        case 10: interp_tma_impl<10>(ps, tg, *map, grid, nvec, out, ostride, nvg, err, st); break;
        default: return false;
    }
    return true;
}

}  // namespace nufft
