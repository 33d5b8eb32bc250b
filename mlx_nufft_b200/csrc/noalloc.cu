// noalloc.cu -- nufft_interp_noalloc: the type-2 interpolation stage with
// no device allocation, for callers that must not allocate device memory
// (see include/nufft_b200.h).
//
// The stage needs one piece of scratch: the (cell, fraction) pair of every
// point in every dimension, which a plan keeps in memory it allocates at
// setpts.  Here that scratch is a file-scope device array of fixed size,
// shared by every call on a device and kept by the process until exit.
// Host code never uses the array's name as a pointer: the device address
// is looked up once per device with cudaGetSymbolAddress and passed to the
// kernels.  The interpolation itself is the same kernel a type-2 plan runs
// with the global method on caller-ordered points (k_interp_global).
#include <cmath>
#include <mutex>
#include <string>

#include "../../include/nufft_b200.h"
#include "spreadinterp.cuh"

namespace nufft {
namespace {

static __device__ __align__(256) unsigned char g_noalloc_scratch[NUFFT_NOALLOC_SCRATCH_BYTES];

constexpr int kMaxDevices = 64;
std::mutex g_scratch_mu;
void* g_scratch_addr[kMaxDevices] = {};

// Device address of the scratch array on the current device (looked up on
// the first call per device).
void* scratch_address(int dev) {
    if (dev < 0 || dev >= kMaxDevices) fail(NUFFT_ERR_UNSUPPORTED, "device ordinal too large");
    std::lock_guard<std::mutex> lk(g_scratch_mu);
    if (!g_scratch_addr[dev]) {
        void* p = nullptr;
        const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (e != cudaSuccess || !p) {
            cudaGetLastError();
            fail(NUFFT_ERR_CUDA, std::string("cudaGetSymbolAddress(no-alloc scratch): ") +
                                     cudaGetErrorString(e));
        }
        g_scratch_addr[dev] = p;
    }
    return g_scratch_addr[dev];
}

struct Coords3 {
    const double* p[3];
};

// crit64 fold of types 1/2 (mod 2pi, / h, ceil(xi - w/2)), the cell index
// shifted so that i1 + w/2 lies in [0, n).  A non-finite coordinate gets
// the cell of 0 (so the interpolation reads inside the grid) and a NaN
// fraction, which k_noalloc_mark_nonfinite turns into a NaN output.
__global__ void __launch_bounds__(256)
k_noalloc_cells(int64_t M, int dim, Coords3 X, int64_t n0, int64_t n1,
                int64_t n2, double halfw_d, int halfw, int2* cells) {
    const int64_t j = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
    if (j >= M) return;
    const int64_t n[3] = {n0, n1, n2};
    for (int d = 0; d < dim; ++d) {
        double x = X.p[d][j];
        const bool bad = !isfinite(x);
        if (bad) x = 0.0;
        double r = fmod(x, kTwoPi);
        if (r < 0.0) r += kTwoPi;
        const double xi = r / (2.0 * kPi / (double)n[d]);
        const double i1d = ceil(xi - halfw_d);
        int64_t b = ((int64_t)i1d + halfw) % n[d];
        if (b < 0) b += n[d];
        const float fr = bad ? __int_as_float(0x7fc00000) : (float)(xi - i1d);
        cells[d * M + j] = make_int2((int)(b - halfw), __float_as_int(fr));
    }
}

// Points whose fraction was marked NaN above (a non-finite coordinate)
// get the output NaN + NaN i.
__global__ void __launch_bounds__(256)
k_noalloc_mark_nonfinite(int64_t M, int dim, const int2* cells, float2* out) {
    const int64_t j = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
    if (j >= M) return;
    bool bad = false;
    for (int d = 0; d < dim; ++d) bad |= isnan(__int_as_float(cells[d * M + j].y));
    if (bad) out[j] = make_float2(__int_as_float(0x7fc00000), __int_as_float(0x7fc00000));
}

}  // namespace
}  // namespace nufft

using namespace nufft;

extern "C" int nufft_interp_noalloc(int dim, const int64_t* n_grid, double eps,
                                    double upsampfac, const void* grid,
                                    int64_t M, const double* x, const double* y,
                                    const double* z, void* out, void* stream) {
    try {
        if (dim < 1 || dim > 3) fail(NUFFT_ERR_ARG, "dim must be 1, 2 or 3");
        if (!n_grid) fail(NUFFT_ERR_ARG, "n_grid is NULL");
        if (!(eps > 0.0)) fail(NUFFT_ERR_ARG, "eps must be positive");
        if (!(upsampfac > 1.0)) fail(NUFFT_ERR_ARG, "upsampfac must be > 1");
        if (M < 0) fail(NUFFT_ERR_ARG, "M must be >= 0");
        const int64_t limit = (int64_t)NUFFT_NOALLOC_SCRATCH_BYTES / (int64_t)sizeof(int2);
        if (M * dim > limit)
            fail(NUFFT_ERR_ARG,
                 "nufft_interp_noalloc: M*dim = " + std::to_string(M * dim) +
                     " exceeds the no-allocation scratch limit of " +
                     std::to_string(limit) + " point-dimensions (" +
                     std::to_string(NUFFT_NOALLOC_SCRATCH_BYTES >> 20) +
                     " MiB); use a plan for larger point sets");
        if (M == 0) return NUFFT_OK;
        const double* xs[3] = {x, y, z};
        for (int d = 0; d < dim; ++d)
            if (!xs[d]) fail(NUFFT_ERR_ARG, "missing coordinate array");
        if (!grid || !out) fail(NUFFT_ERR_ARG, "NULL grid or output");
        int w = 0;
        double beta = 0.0;
        kernel_params(eps, upsampfac, &w, &beta);
        TileGeom tg{};
        tg.dim = dim;
        tg.ncells = 1;
        tg.halfw = w / 2;
        tg.c2w = (float)(2.0 / w);
        tg.beta = (float)beta;
        tg.keval = 0;                       // exp/sqrt weights: no fitted table
        for (int d = 0; d < 3; ++d) {
            if (d < dim) {
                if (n_grid[d] < 2 * w || n_grid[d] > 0x7fffffffLL)
                    fail(NUFFT_ERR_ARG, "each grid extent must be in [2w, 2^31)");
                tg.n[d] = (int)n_grid[d];
                tg.ncells *= n_grid[d];
            } else {
                tg.n[d] = 1;
            }
        }
        set_no_halo(tg);
        int dev = 0;
        NUFFT_CUDA(cudaGetDevice(&dev));
        int2* cells = (int2*)scratch_address(dev);
        cudaStream_t st = (cudaStream_t)stream;
        Coords3 X{{x, y, z}};
        const unsigned blocks = (unsigned)((M + 255) / 256);
        k_noalloc_cells<<<blocks, 256, 0, st>>>(
            M, dim, X, n_grid[0], dim > 1 ? n_grid[1] : 1, dim > 2 ? n_grid[2] : 1,
            w / 2.0, w / 2, cells);
        NUFFT_LAUNCH("k_noalloc_cells");
        CellPtrs cp{};
        for (int d = 0; d < 3; ++d) cp.d[d] = d < dim ? cells + d * M : nullptr;
        NUFFT_DIM_SWITCH(dim, NUFFT_WIDTH_SWITCH(w, {
            k_interp_global<DIM, W, float2><<<blocks, 256, 0, st>>>(
                (const float2*)grid, 1, nullptr, cp, nullptr, M, (float2*)out,
                M, tg);
            NUFFT_LAUNCH("k_interp_global (no-alloc)");
        }));
        k_noalloc_mark_nonfinite<<<blocks, 256, 0, st>>>(M, dim, cells, (float2*)out);
        NUFFT_LAUNCH("k_noalloc_mark_nonfinite");
        return NUFFT_OK;
    } catch (const Error& e) {
        set_last_error(e.msg);
        return e.code;
    } catch (const std::exception& e) {
        set_last_error(e.what());
        return NUFFT_ERR_UNSUPPORTED;
    }
}
