// spread.cu -- launchers for the spreading kernels (types 1 and 3).
#include <algorithm>
#include <cstdlib>
#include <map>
#include <mutex>
#include <set>
#include <utility>

#include "spreadinterp.cuh"

namespace nufft {

int tile_smem_limit() {
    static int limit = 0;
    if (!limit) {
        int dev = 0, v = 0;
        NUFFT_CUDA(cudaGetDevice(&dev));
        NUFFT_CUDA(cudaDeviceGetAttribute(
            &v, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev));
        limit = v;
    }
    return limit;
}

int persistent_grid(const void* kernel, size_t smem, int64_t work, int threads) {
    static std::mutex mu;
    static std::map<std::pair<const void*, size_t>, int> cache;
    static int sms = 0;
    int per_sm = 0;
    {
        std::lock_guard<std::mutex> lk(mu);
        if (!sms) {
            int dev = 0;
            NUFFT_CUDA(cudaGetDevice(&dev));
            NUFFT_CUDA(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
        }
        auto key = std::make_pair(kernel, smem * 4096 + (size_t)threads);
        auto it = cache.find(key);
        if (it != cache.end()) {
            per_sm = it->second;
        } else {
            NUFFT_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel,
                                                                     threads, smem));
            per_sm = std::max(per_sm, 1);
            cache[key] = per_sm;
        }
    }
    return (int)std::max<int64_t>(1, std::min<int64_t>(work, (int64_t)per_sm * sms));
}

void ensure_smem(const void* kernel, size_t bytes) {
    static std::mutex mu;
    static std::map<const void*, size_t> statics;  // kernel -> static bytes
    static std::map<const void*, size_t> raised;   // kernel -> limit set
    std::lock_guard<std::mutex> lk(mu);
    auto st = statics.find(kernel);
    if (st == statics.end()) {
        cudaFuncAttributes fa{};
        NUFFT_CUDA(cudaFuncGetAttributes(&fa, kernel));
        st = statics.emplace(kernel, (size_t)fa.sharedSizeBytes).first;
    }
    // without the opt-in, static + dynamic shared memory is limited to 48 KB
    if (bytes + st->second <= 48 * 1024) return;
    auto it = raised.find(kernel);
    if (it != raised.end() && it->second >= bytes) return;
    const size_t cap = (size_t)tile_smem_limit() - st->second;
    if (bytes > cap) fail(-1, "tile does not fit in shared memory");
    NUFFT_CUDA(cudaFuncSetAttribute(
        kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)cap));
    raised[kernel] = cap;
}

namespace {

// Shared memory (tile + staging) of one plane-spread CTA: two CTAs per SM.
constexpr size_t kPlaneSmemBudget = 112 * 1024;

// 3-D plane-owned spreading of NV vectors per launch.
template <int W, int NV, bool PRE>
void launch_planes(const PointSet& ps, const TileGeom& tg, const float2* c,
                   int64_t cstride, const uint32_t* perm, const CellPtrs& cells,
                   float2* grid, cudaStream_t st) {
    auto k = k_spread_planes<W, NV, PRE>;
    const int S = (NUFFT_PLANE_PAIR && NV % 2 == 0) ? tg.S4 : tg.S2;
    const size_t smem = (size_t)NV * tg.T[0] * tg.T[1] * S * sizeof(float2);
    ensure_smem((const void*)k, smem);
    const int blocks = persistent_grid((const void*)k, smem, ps.nsub,
                                       32 * kPlaneWarps);
    k<<<blocks, 32 * kPlaneWarps, smem, st>>>(c, cstride, perm, cells, ps.phase,
                                               ps.subs, (int)ps.nsub, ps.sched,
                                               grid, tg);
    NUFFT_LAUNCH("k_spread_planes");
}

template <int DIM, int W>
void spread_impl(const PointSet& ps, const TileGeom& tg, const float2* c,
                 int64_t cstride, int nvec, float2* grid, int nvg,
                 cudaStream_t st) {
    const uint32_t* perm = ps.sorted ? ps.perm : nullptr;
    const CellPtrs cells = cell_ptrs(ps);
    if (ps.tiled) {
        if (ps.nsub == 0) return;
        if constexpr (DIM == 3 && W <= 10) {
            // groups of 8, 4, 2 or 1 vectors: the most vectors whose tiles
            // and staging fit the budget, with the staged weight products
            // (W <= 8) when they fit too (NUFFT_PLANE_KB overrides the
            // budget, NUFFT_PLANE_PRE=0 turns the products off; tuning)
            static const size_t budget = [] {
                const char* e = std::getenv("NUFFT_PLANE_KB");
                return (e && *e) ? (size_t)std::atoi(e) * 1024 : kPlaneSmemBudget;
            }();
            static const bool pre_on = [] {
                const char* e = std::getenv("NUFFT_PLANE_PRE");
                return !(e && *e && std::atoi(e) == 0);
            }();
            auto fits = [&](int nv, bool pre) {
                const int S = (NUFFT_PLANE_PAIR && nv % 2 == 0) ? tg.S4 : tg.S2;
                const size_t per = (size_t)tg.T[0] * tg.T[1] * S * sizeof(float2);
                return nv * per + plane_static_bytes(W, nv, pre) <= budget;
            };
            for (int v0 = 0; v0 < nvec;) {
                const int left = nvec - v0;
                int nv = 1;
                for (int cand : {8, 4, 2}) {
                    if (left >= cand && fits(cand, false)) {
                        nv = cand;
                        break;
                    }
                }
                const bool pre = pre_on && W <= 8 && fits(nv, true);
                const float2* cv = c + v0 * cstride;
                float2* gv = grid + v0 * tg.ncells;
                if constexpr (W <= 8) {
                    if (pre) {
                        if (nv == 8) launch_planes<W, 8, true>(ps, tg, cv, cstride, perm, cells, gv, st);
                        else if (nv == 4) launch_planes<W, 4, true>(ps, tg, cv, cstride, perm, cells, gv, st);
                        else if (nv == 2) launch_planes<W, 2, true>(ps, tg, cv, cstride, perm, cells, gv, st);
                        else launch_planes<W, 1, true>(ps, tg, cv, cstride, perm, cells, gv, st);
                        v0 += nv;
                        continue;
                    }
                }
                if (nv == 8) launch_planes<W, 8, false>(ps, tg, cv, cstride, perm, cells, gv, st);
                else if (nv == 4) launch_planes<W, 4, false>(ps, tg, cv, cstride, perm, cells, gv, st);
                else if (nv == 2) launch_planes<W, 2, false>(ps, tg, cv, cstride, perm, cells, gv, st);
                else launch_planes<W, 1, false>(ps, tg, cv, cstride, perm, cells, gv, st);
                v0 += nv;
            }
            return;
        }
        auto k = k_spread_tiled<DIM, W>;
        for (int v0 = 0; v0 < nvec; v0 += nvg) {
            const int nv = std::min(nvg, nvec - v0);
            const size_t smem = (size_t)nv * tg.tcells * sizeof(float2);
            ensure_smem((const void*)k, smem);
            const int blocks = persistent_grid((const void*)k, smem, ps.nsub);
            k<<<blocks, 256, smem, st>>>(
                c + v0 * cstride, cstride, nv, perm, cells, ps.phase, ps.subs,
                (int)ps.nsub, ps.sched, grid + v0 * tg.ncells, tg);
            NUFFT_LAUNCH("k_spread_tiled");
        }
    } else {
        const unsigned blocks = (unsigned)((ps.M + 255) / 256);
        k_spread_global<DIM, W><<<blocks, 256, 0, st>>>(
            c, cstride, nvec, perm, cells, ps.phase, ps.M, grid, tg);
        NUFFT_LAUNCH("k_spread_global");
    }
}

// Disjoint-support spread: point j (sorted position) adds into grid
// groups[caller index of j] only.
template <int DIM, int W>
__global__ void __launch_bounds__(256)
k_spread_groups(const float2* __restrict__ c, const int32_t* __restrict__ groups,
                const uint32_t* __restrict__ perm, CellPtrs cells, int64_t M,
                float2* __restrict__ grid, TileGeom tg) {
    const int64_t j = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
    if (j >= M) return;
    const int64_t src = perm ? (int64_t)__ldg(perm + j) : j;
    const int g = __ldg(groups + src);
    if (g < 0) return;
    float wgt[DIM][W];
    int idx[DIM][W];
    global_taps<DIM, W>(cells, j, tg, wgt, idx);
    global_add<DIM, W>(grid + (int64_t)g * tg.ncells, tg, wgt, idx,
                       __ldg(c + src));
}

}  // namespace

void launch_spread(const PointSet& ps, const TileGeom& tg, int w,
                   const float2* c, int64_t cstride, int nvec, float2* grid,
                   int nvg, cudaStream_t st) {
    NUFFT_DIM_SWITCH(ps.dim, NUFFT_WIDTH_SWITCH(w, spread_impl<DIM, W>(
        ps, tg, c, cstride, nvec, grid, nvg, st)));
}

void launch_spread_groups(const PointSet& ps, const TileGeom& tg, int w,
                          const float2* c, const int32_t* groups,
                          float2* grid, cudaStream_t st) {
    const uint32_t* perm = ps.sorted ? ps.perm : nullptr;
    const CellPtrs cells = cell_ptrs(ps);
    const unsigned blocks = (unsigned)((ps.M + 255) / 256);
    NUFFT_DIM_SWITCH(ps.dim, NUFFT_WIDTH_SWITCH(w, {
        k_spread_groups<DIM, W><<<blocks, 256, 0, st>>>(c, groups, perm, cells,
                                                        ps.M, grid, tg);
        NUFFT_LAUNCH("k_spread_groups");
    }));
}

}  // namespace nufft
