// interp.cu -- launchers for the interpolation kernels (types 2 and 3).
// The fine grid is complex64, or complex128 when the plan runs its FFT in
// fp64 (the taps are always evaluated in fp32).
#include <algorithm>

#include "spreadinterp.cuh"

namespace nufft {

namespace {

template <int DIM, int W, typename G>
void interp_impl(const PointSet& ps, const TileGeom& tg, const G* grid,
                 int nvec, float2* out, int64_t ostride, int nvg,
                 cudaStream_t st) {
    const uint32_t* perm = ps.sorted ? ps.perm : nullptr;
    const CellPtrs cells = cell_ptrs(ps);
    if (ps.tiled) {
        if (ps.nsub == 0) return;
        auto k = k_interp_tiled<DIM, W, G>;
        for (int v0 = 0; v0 < nvec; v0 += nvg) {
            const int nv = std::min(nvg, nvec - v0);
            const size_t smem = (size_t)nv * tg.tcells * sizeof(float2);
            ensure_smem((const void*)k, smem);
            const int blocks = persistent_grid((const void*)k, smem, ps.nsub);
            k<<<blocks, 256, smem, st>>>(
                grid + v0 * tg.pcells, nv, perm, cells, ps.phase, ps.subs,
                (int)ps.nsub, ps.sched, out + v0 * ostride, ostride, tg);
            NUFFT_LAUNCH("k_interp_tiled");
        }
    } else {
        const unsigned blocks = (unsigned)((ps.M + 255) / 256);
        k_interp_global<DIM, W, G><<<blocks, 256, 0, st>>>(
            grid, nvec, perm, cells, ps.phase, ps.M, out, ostride, tg);
        NUFFT_LAUNCH("k_interp_global");
    }
}

}  // namespace

void launch_interp(const PointSet& ps, const TileGeom& tg, int w,
                   const void* grid, bool grid64, int nvec, float2* out,
                   int64_t ostride, int nvg, cudaStream_t st) {
    if (grid64) {
        NUFFT_DIM_SWITCH(ps.dim, NUFFT_WIDTH_SWITCH(w, interp_impl<DIM, W>(
            ps, tg, (const double2*)grid, nvec, out, ostride, nvg, st)));
    } else {
        NUFFT_DIM_SWITCH(ps.dim, NUFFT_WIDTH_SWITCH(w, interp_impl<DIM, W>(
            ps, tg, (const float2*)grid, nvec, out, ostride, nvg, st)));
    }
}

}  // namespace nufft
