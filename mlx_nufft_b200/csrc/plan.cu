// plan.cu -- plan objects and the extern "C" entry points of libnufft_b200.
//
// A plan owns every device buffer the transform needs (sorted point cells,
// permutation, subproblem tables, deconvolution vectors, fine grids, cuFFT
// plans) and runs each execute asynchronously on the caller's stream with
// no host synchronisation.  Stage structure follows the reference:
//   type 1  zero grid -> spread -> FFT -> crop/deconvolve  (nd.py:581-625)
//   type 2  pad/deconvolve -> FFT -> interp                (nd.py:1075-1119)
//   type 3  zero -> prephase+spread (nf grid) -> pad/deconvolve to n_up ->
//           FFT -> interp x post                          (gpu_t3.py:1287-1349)
// cuFFT's inverse transform is unnormalised, so unlike the reference (whose
// MLX ifft divides by n and is undone by folding prod(n_up) into dec[0],
// nd.py:146-147, gpu_t3.py:388-392) no scale is folded into the corrections.
#include <cufft.h>

#include <algorithm>
#include <cmath>
#include <cstdlib>
#include <cstring>
#include <map>
#include <mutex>
#include <new>
#include <string>
#include <vector>

#include "../../include/nufft_b200.h"
#include "internal.h"

namespace nufft {

// ---------------------------------------------------------------------
// errors
thread_local std::string g_last_error;

void set_last_error(const std::string& msg) { g_last_error = msg; }

void fail(int code, const std::string& msg) { throw Error{code, msg}; }

void check_cuda(cudaError_t e, const char* what) {
    if (e == cudaSuccess) return;
    const int code = (e == cudaErrorMemoryAllocation) ? NUFFT_ERR_OOM : NUFFT_ERR_CUDA;
    cudaGetLastError();  // clear a non-sticky error
    fail(code, std::string(what) + ": " + cudaGetErrorString(e));
}

static void check_cufft(cufftResult r, const char* what) {
    if (r == CUFFT_SUCCESS) return;
    const int code = (r == CUFFT_ALLOC_FAILED) ? NUFFT_ERR_OOM : NUFFT_ERR_CUFFT;
    fail(code, std::string(what) + ": cuFFT error " + std::to_string((int)r));
}

void* dmalloc(size_t bytes, const char* what) {
    void* p = nullptr;
    if (bytes == 0) bytes = 16;
    cudaError_t e = cudaMalloc(&p, bytes);
    if (e != cudaSuccess) {
        cudaGetLastError();
        fail(e == cudaErrorMemoryAllocation ? NUFFT_ERR_OOM : NUFFT_ERR_CUDA,
             std::string("device allocation of ") + std::to_string(bytes) +
                 " bytes for " + what + " failed: " + cudaGetErrorString(e));
    }
    return p;
}

void dfree(void* p) {
    if (p) cudaFree(p);
}

namespace {

struct DeviceGuard {
    int prev = -1;
    explicit DeviceGuard(int dev) {
        NUFFT_CUDA(cudaGetDevice(&prev));
        if (prev != dev) NUFFT_CUDA(cudaSetDevice(dev));
    }
    ~DeviceGuard() {
        int cur = -1;
        if (cudaGetDevice(&cur) == cudaSuccess && cur != prev && prev >= 0)
            cudaSetDevice(prev);
    }
};

template <typename F>
int guarded(F&& f) {
    try {
        f();
        return NUFFT_OK;
    } catch (const Error& e) {
        set_last_error(e.msg);
        return e.code;
    } catch (const std::bad_alloc&) {
        set_last_error("host allocation failed");
        return NUFFT_ERR_OOM;
    } catch (const std::exception& e) {
        set_last_error(e.what());
        return NUFFT_ERR_UNSUPPORTED;
    }
}

std::mutex g_plan_mutex;   // serialises plan creation / cuFFT planning

constexpr int kMsubSpread = 1024;   // points per spreading subproblem
constexpr int kMsubInterp = 8192;   // points per interpolation subproblem
constexpr int64_t kTiledMinPoints = 20000;  // below: global kernels (nd.py:304)
constexpr int kTiledMinPerBin = 8;          // points per bin, see want_tiled
constexpr size_t kTileBudget = 96 * 1024;   // smem per CTA for vector groups

}  // namespace
}  // namespace nufft

using namespace nufft;

struct nufft_plan_s {
    int type = 0, dim = 0, device = 0, n_trans = 1, isign = 1;
    double eps = 1e-6;
    nufft_opts opts{};
    double sigma = 2.0, sigma_in = 2.0;
    int w = 0, w2 = 0;
    double beta = 0, beta2 = 0;
    int64_t N[3] = {1, 1, 1};
    int64_t nf[3] = {1, 1, 1};     // spread grid (types 1/2: == nup)
    int64_t nup[3] = {1, 1, 1};    // FFT grid
    int64_t nfcells = 1, nupcells = 1, K = 1;
    int nbatch = 1;
    // type 3
    double C[3] = {0, 0, 0}, D[3] = {0, 0, 0}, gam[3] = {1, 1, 1},
           hf[3] = {0, 0, 0};
    double xlo[3] = {0, 0, 0}, xhi[3] = {0, 0, 0};
    bool sized = false;
    bool points_set = false;
    int64_t Ntgt = 0;
    double* d_ftd = nullptr;   // quadrature nodes for phihat(beta, w)
    double* d_fta = nullptr;
    float* dec[3] = {nullptr, nullptr, nullptr};
    PointSet src, tgt;
    TileGeom tg_src{}, tg_tgt{};
    int nvg_src = 1, nvg_tgt = 1;
    // Fine grids.  gfft holds the FFT grids (complex64, or complex128 when
    // fft64); gspread is the complex64 spreading target of type 3 (nf
    // grids) and of type 1 when fft64 (n_up grids); otherwise type 1
    // spreads straight into gfft.
    bool fft64 = false;
    float2* gspread = nullptr;
    float2* gfft = nullptr;
    // Type 2, 3-D, complex64 with the pruned FFT: gfft is stored with a
    // periodic halo (gh; tg_src carries the layout), so every tile of the
    // TMA interpolation lies inside the stored grid.  gcells: cells per
    // stored FFT grid (nupcells without a halo).
    bool halo = false;
    GridHalo gh{};
    int64_t gcells = 1;
    // Planes of dimension 0 that the point set's tiles read (halo layout;
    // device bytes, gh.P[0] of them), set at setpts: an execute's last FFT
    // pass writes only those when not all are (a plan over one slab of the
    // points); the stage API's grid is always written whole.
    uint8_t* xneed = nullptr;
    bool xneed_all = true;
    // the interior planes among them (fine-grid x, in order) and the map
    // x -> index in that list or -1 (device, n_up[0] ints each): the slab
    // order of the pruned FFT computes only those planes
    int* d_xlist = nullptr;
    int* d_xmap = nullptr;
    int nx_need = 0;
    std::map<int, cufftHandle> ffts;
    Fft1 fft1;                 // two-pass 1-D FFT (fft1.cu), when in use
    Fftn fftn;                 // pruned 3-D FFT with pad / crop (fft1.cu)
    bool profile = false;
    cudaEvent_t ev[4] = {nullptr, nullptr, nullptr, nullptr};
    bool ev_recorded = false;
    int* d_err = nullptr;      // setpts error bits (device memory)
    // execute error flag: pinned host memory mapped into the device address
    // space (h_exec_err on the host, d_exec_err for the kernels); an
    // interpolation kernel whose bounded tile-copy wait ran out stores
    // kErrTileWait there, and the next call on the plan reports it
    int* h_exec_err = nullptr;
    int* d_exec_err = nullptr;
    // Adjoint (nufft_execute_adjoint).  Types 1/2 run the sibling transform
    // (the other type, opposite sign) on this plan's own sorted points,
    // corrections and grids; gadj is the complex64 spreading target of a
    // type-2 plan's adjoint when its FFT grid is complex128.  Type 3 keeps
    // device copies of its sources and targets and builds the sibling plan
    // (targets -> sources, opposite sign) on first use.
    float2* gadj = nullptr;
    double* xcopy[3] = {nullptr, nullptr, nullptr};
    double* scopy[3] = {nullptr, nullptr, nullptr};
    int64_t xcap = 0, scap = 0;
    nufft_plan_s* adj = nullptr;
    int64_t launches = 0;      // own kernels launched by executes
    int64_t fft_execs = 0;     // cuFFT executions issued by executes
    // TMA tensor map over the complex64 FFT grids for the 3-D interpolation,
    // valid for (tmap_grid, tmap_nbatch, tmap_n)
    CUtensorMap tmap{};
    const void* tmap_grid = nullptr;
    int tmap_nbatch = 0;
    int tmap_n[3] = {0, 0, 0};
    bool tmap_ok = false;
};

namespace nufft_impl {

// Integer tuning override from the environment (NUFFT_BIN_1D,
// NUFFT_SORT_CHUNK_LOG2, NUFFT_TILE_KB); the default when unset.
int env_int(const char* name, int dflt) {
    const char* v = std::getenv(name);
    return (v && *v) ? std::atoi(v) : dflt;
}

// Points per interpolation subproblem: 1-D subproblems are streamed
// through a shared-memory stage (interp_tma.cu), at most kStreamMsubMax.
int interp_msub(int dim) {
    static const int m1 = env_int("NUFFT_MSUB_1D", 0);   // tuning overrides
    static const int mn = env_int("NUFFT_MSUB_ND", 0);
    return dim == 1 ? (m1 > 0 ? std::min(m1, kStreamMsubMax) : kStreamMsubMax)
                    : (mn > 0 ? std::min(mn, kMsubInterp) : kMsubInterp);
}

// ----------------------------------------------------------------------
// In-plane tap order of the 3-D plane-owned spread (k_spread_planes).  The
// lanes of a group of G (16: a half-warp of 8-byte accesses; 8: a
// quarter-warp of 16-byte ones) read / write one word each at tile offsets
// y*S + x (in words); the group's accesses are conflict-free when those
// offsets are distinct mod G.  Greedy fill of groups with taps of distinct
// residues, for the smallest row stride S >= T2 (up to T2 + 8) that needs
// only ceil(W^2 / 32) rounds; otherwise the plain order at S = T2
// (correct, with bank conflicts).  Returns S; map[r * 32 + l] = tap
// (y << 4 | x) of lane l in round r, 0xff idle.
int tap_groups(int w, int T2, int G, uint8_t* map, size_t map_bytes) {
    std::memset(map, 0xff, map_bytes);
    const int rounds = (w * w + 31) / 32;
    if (w > kMaxW || rounds > kMaxTapRounds) return T2;
    for (int S = T2; S <= T2 + 8; ++S) {
        std::vector<int> left;
        for (int t = 0; t < w * w; ++t) left.push_back(t);
        std::vector<std::vector<int>> groups;
        while (!left.empty()) {
            std::vector<int> grp, rest;
            bool used[16] = {};
            for (int t : left) {
                const int r = ((t / w) * S + t % w) % G;
                if (!used[r] && (int)grp.size() < G) {
                    used[r] = true;
                    grp.push_back(t);
                } else {
                    rest.push_back(t);
                }
            }
            groups.push_back(grp);
            left.swap(rest);
        }
        const int per_round = 32 / G;
        if ((int)(groups.size() + per_round - 1) / per_round > rounds) continue;
        for (size_t h = 0; h < groups.size(); ++h)
            for (size_t i = 0; i < groups[h].size(); ++i) {
                const int t = groups[h][i];
                map[h * G + i] = (uint8_t)(((t / w) << 4) | (t % w));
            }
        return S;
    }
    for (int t = 0; t < w * w; ++t) map[t] = (uint8_t)(((t / w) << 4) | (t % w));
    return T2;
}

// Both tap orders of a 3-D spread geometry: 8-byte words (one vector per
// tile, tapmap / S2) and 16-byte words (two vectors per tile cell,
// tapmap4 / S4).
void plane_tap_order(TileGeom& tg, int w) {
    tg.S2 = tap_groups(w, tg.T[2], 16, tg.tapmap, sizeof(tg.tapmap));
    tg.S4 = tap_groups(w, tg.T[2], 8, tg.tapmap4, sizeof(tg.tapmap4));
}

// ----------------------------------------------------------------------
// tiling choice per grid: bin extent m per dimension so that the tile
// (m + w - 1)^dim of complex64 fits shared memory with room for several
// vectors: 1024 cells in 1-D for spreading and 512 for interpolation (the
// streamed 1-D interpolation stages a subproblem's tile in shared memory
// next to its points; smaller stages leave room for more CTAs), 32 x 32 in 2-D,
// 8 x 8 x 8 in 3-D for spreading (room for several vectors' tiles) and
// 10 x 10 x 10 for 3-D interpolation (more points per subproblem, less halo:
// measured 21-27 % faster than 8^3 on the 3-D benchmark workloads: 3-D
// type 2 at 5e7 clustered points and 3-D type 3 at 1e6 -> 1e6).  The
// TMA-staged complex64 interpolation at w <= 7 takes 12^3 bins (`m3i`):
// two 18 x 18 x 20-cell buffers per CTA still fit two CTAs per SM, and the
// larger subproblems even out the bank residues of their points (3-D type
// 2, 256^3 modes, 5e7 clustered points: interp 5.37 ms vs 5.67 at 10^3,
// 5.79 at 11^3, 8.44 at 9^3).
bool halo_wanted(const nufft_plan_s* p);

TileGeom make_tile(int dim, const int64_t* n, int w, double beta, int keval,
                   bool interp, int m3i_default = 10) {
    TileGeom tg{};
    tg.dim = dim;
    tg.ncells = 1;
    tg.tcells = 1;
    tg.halfw = w / 2;
    tg.c2w = (float)(2.0 / w);
    tg.beta = (float)beta;
    tg.keval = keval ? 1 : 0;
    tg.poly = make_es_poly(w, beta);
    static const int m1d = env_int("NUFFT_BIN_1D", 0);
    // 1-D interp bins: 1792 cells (cfg 2 interp 0.091 ms; 1024: 0.096,
    // 1536: 0.092, 2048: 0.105 -- its stages leave 3 CTAs per SM, not 4)
    const int m1 = m1d > 0 ? m1d : (interp ? 1792 : 1024);
    static const int m3i = env_int("NUFFT_BIN_3D_INTERP", 0);
    static const int m3s = env_int("NUFFT_BIN_3D_SPREAD", 0);   // tuning
    const int m3 = interp ? (m3i > 0 ? m3i : m3i_default) : (m3s > 0 ? m3s : 8);
    static const int m2d = env_int("NUFFT_BIN_2D", 0);
    const int m2 = m2d > 0 ? m2d : 32;
    int m0 = dim == 1 ? m1 : (dim == 2 ? m2 : m3);
    for (int d = 0; d < 3; ++d) {
        if (d < dim) {
            tg.n[d] = (int)n[d];
            tg.m[d] = (int)std::min<int64_t>(m0, n[d]);
            tg.nb[d] = (int)((n[d] + tg.m[d] - 1) / tg.m[d]);
            tg.T[d] = tg.m[d] + w - 1;
        } else {
            tg.n[d] = tg.m[d] = tg.nb[d] = tg.T[d] = 1;
        }
    }
    for (int d = 0; d < dim; ++d) {
        tg.ncells *= n[d];
        tg.tcells *= tg.T[d];
        tg.tdiv[d] = tg.T[d] > 1
            ? (uint32_t)(((uint64_t)1 << 32) / (uint64_t)tg.T[d] + 1) : 0u;
    }
    tg.S2 = tg.S4 = tg.T[2];
    if (dim == 3) plane_tap_order(tg, w);
    set_no_halo(tg);
    return tg;
}

// Periodic halo that puts every tile box of a 3-D TMA interpolation (tile
// origins o = bin * m - w/2, box [x0, x0 + B2) in the contiguous dimension
// with x0 = o rounded down to even) inside the stored grid; false when a
// halo would exceed a period.  lo[2] and hi[2] are even, so the padded rows
// stay 16-byte multiples and x0 + lo[2] stays even (TMA alignment).
bool grid_halo(const TileGeom& tg, GridHalo* h) {
    if (tg.dim != 3) return false;
    const int B2 = tma_box_x(tg);
    for (int d = 0; d < 3; ++d) {
        const int omax = (tg.nb[d] - 1) * tg.m[d] - tg.halfw;
        int lo, hi;
        if (d < 2) {
            lo = tg.halfw;
            hi = std::max(0, omax + tg.T[d] - tg.n[d]);
        } else {
            lo = tg.halfw + (tg.halfw & 1);
            const int x0max = omax - (omax & 1);
            hi = std::max(0, x0max + B2 - tg.n[d]);
            hi += hi & 1;
        }
        if (lo + hi > tg.n[d]) return false;
        h->lo[d] = lo;
        h->hi[d] = hi;
        h->P[d] = lo + tg.n[d] + hi;
    }
    return true;
}

void apply_halo(TileGeom& tg, const GridHalo& h) {
    tg.pcells = 1;
    for (int d = 0; d < 3; ++d) {
        tg.lo[d] = h.lo[d];
        tg.P[d] = h.P[d];
        tg.pcells *= h.P[d];
    }
}

// Caller-order chunk (points) of the bin sort.  In 1-D / 2-D a point touches
// few cells, so the cost that dominates is the caller-ordered access of
// its strength (spread) or output (interp), which a plain bin sort turns
// into a random 8-byte scatter/gather over the whole array.  Sorting by
// (chunk, bin) bounds the array slice in flight to 8-16 MB (L2-resident);
// the price is one extra tile load per bin per chunk, from L2.  1-D
// interpolation uses 2^20-point chunks (cfg 2 with 1024-cell bins: 0.096 ms
// vs 0.104 for 2^21 with 512-cell bins, which has as many subproblems;
// 2048-cell bins with 2^19 0.123); spreading keeps 2^21.  In 3-D the
// per-point tap work dominates and bins need all their points, so 0.
// NUFFT_SORT_CHUNK_LOG2 overrides the default (tuning; negative disables).
int64_t sort_chunk(int dim, bool interp) {
    static const int lg = env_int("NUFFT_SORT_CHUNK_LOG2", 0);
    const int l = lg > 0 ? lg : (dim == 1 && interp ? 20 : 21);
    return (dim <= 2 && lg >= 0) ? (int64_t)1 << l : 0;
}

// dynamic shared memory available to a tile (kernels keep < 1 KB static)
size_t tile_bytes_max() { return (size_t)tile_smem_limit() - 1024; }

bool tile_fits(const TileGeom& tg) {
    return (size_t)tg.tcells * sizeof(float2) <= tile_bytes_max();
}

int vectors_per_tile(const TileGeom& tg, int nbatch) {
    const size_t per = (size_t)tg.tcells * sizeof(float2);
    static const int kb = env_int("NUFFT_TILE_KB", 0);   // tuning override
    const size_t budget = kb > 0 ? (size_t)kb * 1024 : kTileBudget;
    int nvg = (int)std::max<size_t>(1, budget / per);
    if ((size_t)nvg * per > tile_bytes_max())
        nvg = (int)std::max<size_t>(1, tile_bytes_max() / per);
    return std::max(1, std::min(nvg, nbatch));
}

// Automatic choice: tiled when the tile fits, there are enough points
// (nd.py:304), and the points per bin on average pay for the per-subproblem
// tile traffic (one load, or one zero + flush, of the whole tile).  Below
// that density the global kernels touch only the points' own taps.  A 2-D
// spread (types 1 and 3 sources) also needs kTiled2dSpreadPerCell points
// per fine cell: below it the tiled kernel's zero + flush of 38^2-cell
// tiles costs more than the global atomics (measured on a 512^2 grid:
// 1e5 points 47 vs 39 us, 3e5 134 vs 104 us; 1e6 243 vs 448 us).
constexpr double kTiled2dSpreadPerCell = 2.0;

bool want_tiled(const nufft_plan_s* p, int64_t npts, const TileGeom& tg,
                bool spread) {
    if (p->opts.method == NUFFT_METHOD_GLOBAL) return false;
    const bool fits = tile_fits(tg);
    if (p->opts.method == NUFFT_METHOD_TILED) {
        if (!fits) fail(NUFFT_ERR_ARG, "tiled method not applicable: tile exceeds shared memory");
        return true;
    }
    static const int min_per_bin = env_int("NUFFT_MIN_PER_BIN", kTiledMinPerBin);
    double bins = 1.0;
    for (int d = 0; d < tg.dim; ++d) bins *= tg.nb[d];
    if (spread && tg.dim == 2 &&
        (double)npts < kTiled2dSpreadPerCell * (double)tg.ncells)
        return false;
    return fits && npts >= kTiledMinPoints && (double)npts >= min_per_bin * bins;
}

void upload_dec(nufft_plan_s* p, int d, const std::vector<double>& v) {
    std::vector<float> f(v.size());
    for (size_t i = 0; i < v.size(); ++i) f[i] = (float)v[i];
    dfree(p->dec[d]);
    p->dec[d] = nullptr;
    p->dec[d] = (float*)dmalloc(sizeof(float) * std::max<size_t>(f.size(), 1), "deconvolution");
    NUFFT_CUDA(cudaMemcpy(p->dec[d], f.data(), sizeof(float) * f.size(),
                          cudaMemcpyHostToDevice));
}

double phihat_host(double xi, const std::vector<double>& dq,
                   const std::vector<double>& aq) {
    double s = 0.0;
    for (size_t q = 0; q < dq.size(); ++q) s += aq[q] * std::cos(xi * dq[q]);
    return 2.0 * s;
}

void destroy_ffts(nufft_plan_s* p) {
    for (auto& kv : p->ffts) cufftDestroy(kv.second);
    p->ffts.clear();
}

cufftHandle get_fft(nufft_plan_s* p, int nv) {
    auto it = p->ffts.find(nv);
    if (it != p->ffts.end()) return it->second;
    std::lock_guard<std::mutex> lk(g_plan_mutex);
    cufftHandle h;
    check_cufft(cufftCreate(&h), "cufftCreate");
    long long n[3];
    for (int d = 0; d < p->dim; ++d) n[d] = p->nup[d];
    size_t ws = 0;
    cufftResult r = cufftMakePlanMany64(h, p->dim, n, nullptr, 1, p->nupcells,
                                        nullptr, 1, p->nupcells,
                                        p->fft64 ? CUFFT_Z2Z : CUFFT_C2C, nv,
                                        &ws);
    if (r != CUFFT_SUCCESS) {
        cufftDestroy(h);
        check_cufft(r, "cufftMakePlanMany64");
    }
    p->ffts[nv] = h;
    return h;
}

// In-place FFT of nv fine grids (gfft): the unnormalised inverse when
// `inv` (a transform of sign +1), else the forward transform.
void run_fft(nufft_plan_s* p, int nv, bool inv, cudaStream_t st) {
    cufftHandle h = get_fft(p, nv);
    check_cufft(cufftSetStream(h, st), "cufftSetStream");
    const int dir = inv ? CUFFT_INVERSE : CUFFT_FORWARD;
    ++p->fft_execs;
    if (p->fft64)
        check_cufft(cufftExecZ2Z(h, (cufftDoubleComplex*)p->gfft,
                                 (cufftDoubleComplex*)p->gfft, dir),
                    "cufftExecZ2Z");
    else
        check_cufft(cufftExecC2C(h, (cufftComplex*)p->gfft,
                                 (cufftComplex*)p->gfft, dir),
                    "cufftExecC2C");
}

size_t fft_cell_bytes(const nufft_plan_s* p) {
    return p->fft64 ? sizeof(double2) : sizeof(float2);
}

// Spreading target of type 1 (complex64 n_up grids).
float2* t1_spread_grid(const nufft_plan_s* p) {
    return p->fft64 ? p->gspread : p->gfft;
}

void alloc_grids(nufft_plan_s* p) {
    dfree(p->gadj);             // re-created at the new batch size on use
    p->gadj = nullptr;
    dfree(p->gfft);
    p->gfft = nullptr;
    dfree(p->gspread);
    p->gspread = nullptr;
    p->gfft = (float2*)dmalloc(fft_cell_bytes(p) * p->gcells * p->nbatch,
                               "fine grid");
    if (p->type == 3)
        p->gspread = (float2*)dmalloc(sizeof(float2) * p->nfcells * p->nbatch,
                                      "type-3 spread grid");
    else if (p->type == 1 && p->fft64)
        p->gspread = (float2*)dmalloc(sizeof(float2) * p->nupcells * p->nbatch,
                                      "type-1 spread grid");
}

// fp64 FFT when cuFFT's fp32 rounding would be amplified by the 1/phihat
// corrections: at upsampling < 1.5 the corrections near the band edge reach
// 1e3..1e5, and cuFFT's fp32 error (~1e-7 relative rms, several times that
// of an fp32 FFT with accurate twiddles) then dominates the result.
bool want_fft64(const nufft_plan_s* p, double sigma_inner) {
    if (p->opts.fft_prec == 2) return true;
    if (p->opts.fft_prec == 1) return false;
    return sigma_inner < 1.5 && p->eps < 1e-4;
}

void record(nufft_plan_s* p, int i, cudaStream_t st) {
    if (p->profile) NUFFT_CUDA(cudaEventRecord(p->ev[i], st));
}

// Report (and clear) a tile-copy timeout that an earlier execute recorded in
// the plan's host-mapped flag; reading it needs no device synchronisation
// (a flag raised by an execute still in flight is reported by a later call).
void check_exec_flag(nufft_plan_s* p) {
    if (!p->h_exec_err) return;
    const int h = *(volatile int*)p->h_exec_err;
    if (h) {
        *(volatile int*)p->h_exec_err = 0;
        fail(NUFFT_ERR_CUDA, "an interpolation tile copy of an earlier execute on "
                             "this plan did not complete; that execute's output is "
                             "invalid");
    }
}

void check_err_flag(nufft_plan_s* p, cudaStream_t st) {
    int h = 0;
    NUFFT_CUDA(cudaMemcpyAsync(&h, p->d_err, sizeof(int), cudaMemcpyDeviceToHost, st));
    NUFFT_CUDA(cudaStreamSynchronize(st));
    if (h) {
        NUFFT_CUDA(cudaMemsetAsync(p->d_err, 0, sizeof(int), st));
        NUFFT_CUDA(cudaStreamSynchronize(st));
        fail(NUFFT_ERR_ARG, "non-finite nonuniform coordinate");
    }
}

// ---------------------------------------------------------------------
// types 1 / 2
void create_t12(nufft_plan_s* p) {
    p->sigma = p->opts.upsampfac > 0 ? p->opts.upsampfac : 2.0;
    if (!(p->sigma > 1.0 && p->sigma <= 4.0))
        fail(NUFFT_ERR_ARG, "upsampfac must be in (1, 4]");
    kernel_params(p->eps, p->sigma, &p->w, &p->beta);
    p->w2 = p->w;
    p->beta2 = p->beta;
    p->fft64 = want_fft64(p, p->sigma);
    p->K = 1;
    p->nupcells = 1;
    for (int d = 0; d < p->dim; ++d) {
        if (p->N[d] < 1) fail(NUFFT_ERR_ARG, "mode dims must be >= 1");
        const int64_t up = (int64_t)std::ceil(p->sigma * (double)p->N[d]);
        p->nup[d] = next235even(std::max<int64_t>(2 * p->w, up));
        if (p->nup[d] > 0x7fffffffLL) fail(NUFFT_ERR_ARG, "fine grid too large");
        p->nf[d] = p->nup[d];
        p->K *= p->N[d];
        p->nupcells *= p->nup[d];
    }
    p->nfcells = p->nupcells;
    // corrections 1/phihat(2 pi k / n_up), k in [-N/2, N - N/2)  (nd.py:140-145)
    std::vector<double> dq, aq;
    kernel_ft_nodes(p->beta, p->w, &dq, &aq);
    for (int d = 0; d < p->dim; ++d) {
        std::vector<double> v(p->N[d]);
        for (int64_t i = 0; i < p->N[d]; ++i) {
            const double k = (double)(i - p->N[d] / 2);
            v[i] = 1.0 / phihat_host(2.0 * kPi * k / (double)p->nup[d], dq, aq);
        }
        upload_dec(p, d, v);
    }
    p->tg_src = make_tile(p->dim, p->nup, p->w, p->beta, p->opts.kerevalmeth,
                          p->type == 2, (!p->fft64 && p->w <= 7) ? 12 : 10);
    p->halo = p->type == 2 && halo_wanted(p) && grid_halo(p->tg_src, &p->gh);
    if (p->halo) apply_halo(p->tg_src, p->gh);
    p->gcells = p->halo ? p->tg_src.pcells : p->nupcells;
    p->nvg_src = vectors_per_tile(p->tg_src, p->nbatch);
    alloc_grids(p);
    p->sized = true;
}

// Shared-tile strides of the interpolation kernel that will read an
// interpolation point set (CellParams::rs): the 1-D tile is contiguous;
// the 3-D TMA-staged tile (complex64 grids) has rows of tma_box_x cells,
// the plain tiled kernel's (complex128 grids) rows of T[2] cells; the 2-D
// kernel reads cell-unordered points (rs = 0).
void interp_strides(const nufft_plan_s* p, const TileGeom& tg, CellParams* cp) {
    static const int tma_on = env_int("NUFFT_INTERP_TMA", 1);
    cp->rs[0] = cp->rs[1] = cp->rs[2] = 0;
    if (tg.dim == 1) {
        cp->rs[0] = 1;
    } else if (tg.dim == 3) {
        const int S = (tma_on && !p->fft64) ? tma_box_x(tg) : tg.T[2];
        cp->rs[0] = tg.T[1] * S;
        cp->rs[1] = S;
        cp->rs[2] = 1;
    }
}

void setpts_t12(nufft_plan_s* p, int64_t M, const double* const* xs,
                cudaStream_t st) {
    CellParams cp{};
    cp.kind = CELL_FOLD;
    cp.dim = p->dim;
    cp.fp32 = p->opts.prec == NUFFT_PREC_FP32;
    cp.halfw = p->w / 2;
    cp.halfw_d = p->w / 2.0;
    for (int d = 0; d < p->dim; ++d) {
        cp.n[d] = p->nup[d];
        cp.h[d] = 2.0 * kPi / (double)p->nup[d];
        cp.m[d] = p->tg_src.m[d];
        cp.nb[d] = p->tg_src.nb[d];
    }
    const bool tiled = want_tiled(p, M, p->tg_src, p->type == 1);
    const bool sort = tiled || p->opts.sort_points;
    cp.chunk = tiled ? sort_chunk(p->dim, p->type == 2) : 0;
    if (p->type == 2) interp_strides(p, p->tg_src, &cp);
    PhaseParams pp{};
    build_pointset(&p->src, cp, M, xs, sort, tiled,
                   p->type == 1 ? kMsubSpread : interp_msub(p->dim), p->type == 2,
                   pp, p->d_err, st);
    check_err_flag(p, st);
    p->xneed_all = true;
    if (p->halo && p->src.tiled) {
        const int P0 = p->gh.P[0];
        if (!p->xneed) p->xneed = (uint8_t*)dmalloc(P0, "plane marks");
        NUFFT_CUDA(cudaMemsetAsync(p->xneed, 0, P0, st));
        mark_tile_planes(p->src, p->tg_src, p->xneed, st);
        std::vector<uint8_t> h(P0);
        NUFFT_CUDA(cudaMemcpyAsync(h.data(), p->xneed, P0, cudaMemcpyDeviceToHost, st));
        NUFFT_CUDA(cudaStreamSynchronize(st));
        for (int i = 0; i < P0; ++i) p->xneed_all &= h[i] != 0;
        if (!p->xneed_all) {
            const int n0 = (int)p->nup[0];
            std::vector<int> list, map(n0, -1);
            for (int x = 0; x < n0; ++x)
                if (h[x + p->gh.lo[0]]) {
                    map[x] = (int)list.size();
                    list.push_back(x);
                }
            if (!p->d_xmap) {
                p->d_xmap = (int*)dmalloc(sizeof(int) * n0, "plane map");
                p->d_xlist = (int*)dmalloc(sizeof(int) * n0, "plane list");
            }
            NUFFT_CUDA(cudaMemcpy(p->d_xmap, map.data(), sizeof(int) * n0,
                                  cudaMemcpyHostToDevice));
            NUFFT_CUDA(cudaMemcpy(p->d_xlist, list.data(), sizeof(int) * list.size(),
                                  cudaMemcpyHostToDevice));
            p->nx_need = (int)list.size();
        }
    }
    p->points_set = true;
}

// ---------------------------------------------------------------------
// type 3
void create_t3(nufft_plan_s* p) {
    p->sigma = p->opts.upsampfac > 0 ? p->opts.upsampfac : 1.25;
    if (!(p->sigma > 1.0)) fail(NUFFT_ERR_ARG, "upsampfac must be > 1");
    kernel_params(p->eps, p->sigma, &p->w, &p->beta);
    const double si = p->opts.sigma_inner;
    if (si <= 0.0 || si == p->sigma) {
        p->sigma_in = p->sigma;
        p->w2 = p->w;
        p->beta2 = p->beta;
    } else {
        if (!(si > 1.0)) fail(NUFFT_ERR_ARG, "sigma_inner must be > 1");
        // gpu_t3.py:279-284
        p->sigma_in = si;
        int ns = (int)std::ceil(-std::log(p->eps) / (kPi * std::sqrt(1.0 - 1.0 / si)));
        ns = std::max(2, std::min(ns, 16));
        p->w2 = ns;
        p->beta2 = 0.97 * kPi * (1.0 - 1.0 / (2.0 * si)) * ns;
    }
    p->fft64 = want_fft64(p, p->sigma_in);
    std::vector<double> dq, aq;
    kernel_ft_nodes(p->beta, p->w, &dq, &aq);
    p->d_ftd = (double*)dmalloc(sizeof(double) * dq.size(), "phihat nodes");
    p->d_fta = (double*)dmalloc(sizeof(double) * aq.size(), "phihat weights");
    NUFFT_CUDA(cudaMemcpy(p->d_ftd, dq.data(), sizeof(double) * dq.size(),
                          cudaMemcpyHostToDevice));
    NUFFT_CUDA(cudaMemcpy(p->d_fta, aq.data(), sizeof(double) * aq.size(),
                          cudaMemcpyHostToDevice));
}

// Size grids from source extents [xlo, xhi] and target extents [slo, shi]
// (gpu_t3.py:322-342, 379-383).
void size_t3(nufft_plan_s* p, const double* slo, const double* shi) {
    int64_t nf_new[3], nup_new[3];
    for (int d = 0; d < p->dim; ++d) {
        p->C[d] = 0.5 * (p->xlo[d] + p->xhi[d]);
        p->D[d] = 0.5 * (slo[d] + shi[d]);
        const double X = 0.5 * (p->xhi[d] - p->xlo[d]);
        const double S = 0.5 * (shi[d] - slo[d]);
        double h;
        set_nhg_type3(S, X, p->sigma, p->w, &nf_new[d], &h, &p->gam[d]);
        p->hf[d] = 2.0 * kPi / (double)nf_new[d];
        nup_new[d] = next235even((int64_t)std::ceil(p->sigma_in * (double)nf_new[d]));
        if (nup_new[d] > 0x7fffffffLL) fail(NUFFT_ERR_ARG, "type-3 grid too large");
    }
    bool changed = !p->sized;
    for (int d = 0; d < p->dim; ++d)
        changed |= (nf_new[d] != p->nf[d]) || (nup_new[d] != p->nup[d]);
    p->nfcells = p->nupcells = 1;
    for (int d = 0; d < p->dim; ++d) {
        p->nf[d] = nf_new[d];
        p->nup[d] = nup_new[d];
        p->nfcells *= p->nf[d];
        p->nupcells *= p->nup[d];
    }
    p->gcells = p->nupcells;
    // mode corrections (-1)^q / phihat2(2 pi q / n_up), q in [-nf/2, nf/2)
    std::vector<double> dq, aq;
    kernel_ft_nodes(p->beta2, p->w2, &dq, &aq);
    for (int d = 0; d < p->dim; ++d) {
        std::vector<double> v(p->nf[d]);
        for (int64_t i = 0; i < p->nf[d]; ++i) {
            const int64_t q = i - p->nf[d] / 2;
            const double sgn = (q % 2 == 0) ? 1.0 : -1.0;
            v[i] = sgn / phihat_host(2.0 * kPi * (double)q / (double)p->nup[d], dq, aq);
        }
        upload_dec(p, d, v);
    }
    if (changed) {
        destroy_ffts(p);
        alloc_grids(p);
    }
    p->tg_src = make_tile(p->dim, p->nf, p->w, p->beta, p->opts.kerevalmeth,
                          false);
    p->nvg_src = vectors_per_tile(p->tg_src, p->nbatch);
    p->tg_tgt = make_tile(p->dim, p->nup, p->w2, p->beta2, p->opts.kerevalmeth,
                          true);
    p->nvg_tgt = vectors_per_tile(p->tg_tgt, p->nbatch);
    p->sized = true;
}

void set_sources_t3(nufft_plan_s* p, int64_t M, const double* const* xs,
                    bool check_guard, cudaStream_t st) {
    if (check_guard) {
        double mm[6];
        device_minmax(p->dim, xs, M, mm, st);
        for (int d = 0; d < p->dim; ++d) {
            const double guard = 0.45 * (p->w + 1) * p->gam[d] * (2.0 * kPi / (double)p->nf[d]);
            if (mm[2 * d] < p->xlo[d] - guard || mm[2 * d + 1] > p->xhi[d] + guard) {
                char buf[256];
                snprintf(buf, sizeof buf,
                         "set_sources: dim %d sources exceed the frozen plan extent "
                         "[%.4g, %.4g] (+guard %.3g); rebuild the plan for this geometry",
                         d, p->xlo[d], p->xhi[d], guard);
                fail(NUFFT_ERR_RANGE, buf);
            }
        }
    }
    CellParams cp{};
    cp.kind = CELL_T3SRC;
    cp.dim = p->dim;
    const int prec = p->opts.prec;
    cp.fp32 = !(prec == NUFFT_PREC_CRIT64 || prec == NUFFT_PREC_COORDS64);
    cp.halfw = p->w / 2;
    cp.halfw_d = p->w / 2.0;
    for (int d = 0; d < p->dim; ++d) {
        cp.n[d] = p->nf[d];
        cp.a[d] = p->C[d];
        cp.b[d] = p->gam[d];
        cp.h[d] = p->hf[d];
        cp.c[d] = p->nf[d] / 2.0;
        cp.m[d] = p->tg_src.m[d];
        cp.nb[d] = p->tg_src.nb[d];
    }
    PhaseParams pp{};
    pp.mode = 1;
    pp.isign = p->isign;
    pp.fp32 = !(prec == NUFFT_PREC_CRIT64 || prec == NUFFT_PREC_PHASES64);
    for (int d = 0; d < p->dim; ++d) pp.D[d] = p->D[d];
    const bool tiled = want_tiled(p, M, p->tg_src, true);
    const bool sort = tiled || p->opts.sort_points;
    cp.chunk = tiled ? sort_chunk(p->dim, false) : 0;
    build_pointset(&p->src, cp, M, xs, sort, tiled, kMsubSpread, false, pp,
                   p->d_err, st);
    check_err_flag(p, st);
}

// Device copies of a type-3 plan's coordinates (for its adjoint), grown
// when needed; copies on `st`.
void keep_coords(double** dst, int64_t* cap, int dim, int64_t n,
                 const double* const* src, cudaStream_t st) {
    if (n > *cap) {
        for (int d = 0; d < 3; ++d) {
            dfree(dst[d]);
            dst[d] = nullptr;
        }
        *cap = 0;
        for (int d = 0; d < dim; ++d)
            dst[d] = (double*)dmalloc(sizeof(double) * n, "type-3 coordinates");
        *cap = n;
    }
    for (int d = 0; d < dim; ++d)
        NUFFT_CUDA(cudaMemcpyAsync(dst[d], src[d], sizeof(double) * n,
                                   cudaMemcpyDeviceToDevice, st));
}

void drop_adjoint(nufft_plan_s* p);

void setpts_t3(nufft_plan_s* p, int64_t M, const double* const* xs, int64_t N,
               const double* const* ss, cudaStream_t st) {
    if (N < 1) fail(NUFFT_ERR_ARG, "at least one target is required");
    double smm[6], xmm[6];
    device_minmax(p->dim, ss, N, smm, st);
    if (p->opts.has_source_extent) {
        for (int d = 0; d < p->dim; ++d) {
            p->xlo[d] = p->opts.source_extent[2 * d];
            p->xhi[d] = p->opts.source_extent[2 * d + 1];
        }
    } else {
        device_minmax(p->dim, xs, M, xmm, st);
        for (int d = 0; d < p->dim; ++d) {
            p->xlo[d] = xmm[2 * d];
            p->xhi[d] = xmm[2 * d + 1];
        }
    }
    double slo[3], shi[3];
    for (int d = 0; d < p->dim; ++d) {
        slo[d] = smm[2 * d];
        shi[d] = smm[2 * d + 1];
        if (!std::isfinite(slo[d]) || !std::isfinite(shi[d]) ||
            !std::isfinite(p->xlo[d]) || !std::isfinite(p->xhi[d]))
            fail(NUFFT_ERR_ARG, "non-finite type-3 coordinate");
    }
    size_t3(p, slo, shi);
    // targets (gpu_t3.py:357-377)
    CellParams cp{};
    cp.kind = CELL_T3TGT;
    cp.dim = p->dim;
    const int prec = p->opts.prec;
    cp.fp32 = !(prec == NUFFT_PREC_CRIT64 || prec == NUFFT_PREC_COORDS64);
    cp.halfw = p->w2 / 2;
    cp.halfw_d = p->w2 / 2.0;
    for (int d = 0; d < p->dim; ++d) {
        cp.n[d] = p->nup[d];
        cp.a[d] = p->D[d];
        cp.b[d] = p->hf[d] * p->gam[d];
        cp.c[d] = 2.0 * kPi / (double)p->nup[d];
        cp.e[d] = p->nup[d] / 2.0;
        cp.m[d] = p->tg_tgt.m[d];
        cp.nb[d] = p->tg_tgt.nb[d];
    }
    PhaseParams pp{};
    pp.mode = 2;
    pp.isign = p->isign;
    pp.fp32 = !(prec == NUFFT_PREC_CRIT64 || prec == NUFFT_PREC_PHASES64);
    for (int d = 0; d < p->dim; ++d) {
        pp.C[d] = p->C[d];
        pp.D[d] = p->D[d];
    }
    pp.ftd = p->d_ftd;
    pp.fta = p->d_fta;
    pp.nq = 128;
    const bool tiled = want_tiled(p, N, p->tg_tgt, false);
    const bool sort = tiled || p->opts.sort_points;
    cp.chunk = tiled ? sort_chunk(p->dim, true) : 0;
    interp_strides(p, p->tg_tgt, &cp);
    build_pointset(&p->tgt, cp, N, ss, sort, tiled, interp_msub(p->dim), true, pp,
                   p->d_err, st);
    check_err_flag(p, st);
    p->Ntgt = N;
    // sources: guard against the extent only when it was given explicitly
    set_sources_t3(p, M, xs, p->opts.has_source_extent != 0, st);
    drop_adjoint(p);
    keep_coords(p->scopy, &p->scap, p->dim, N, ss, st);
    keep_coords(p->xcopy, &p->xcap, p->dim, M, xs, st);
    p->points_set = true;
}

// ---------------------------------------------------------------------
// Tensor map for the TMA-staged 3-D interpolation from the FFT grids
// (complex64 only), re-encoded when the grids or the tile geometry change;
// null when not applicable.  NUFFT_INTERP_TMA=0 disables the path (tuning).
const CUtensorMap* interp_tmap(nufft_plan_s* p, const TileGeom& tg) {
    static const int on = env_int("NUFFT_INTERP_TMA", 1);
    if (!on || p->fft64 || tg.dim != 3) return nullptr;
    if (p->tmap_grid != p->gfft || p->tmap_nbatch != p->nbatch ||
        p->tmap_n[0] != tg.P[0] || p->tmap_n[1] != tg.P[1] || p->tmap_n[2] != tg.P[2]) {
        p->tmap_ok = make_grid_tmap(&p->tmap, p->gfft, tg, p->nbatch);
        p->tmap_grid = p->gfft;
        p->tmap_nbatch = p->nbatch;
        for (int d = 0; d < 3; ++d) p->tmap_n[d] = tg.P[d];
    }
    return p->tmap_ok ? &p->tmap : nullptr;
}

// The complex64 FFT grid for the staged interpolation kernels (null: fp64
// FFT grid, or the path disabled with NUFFT_INTERP_STREAM=0 for tuning).
const float2* interp_grid32(const nufft_plan_s* p) {
    static const int on = env_int("NUFFT_INTERP_STREAM", 1);
    return (p->fft64 || !on) ? nullptr : p->gfft;
}

// The two-pass FFT of fft1.cu, with the pad / crop fused into its passes,
// replaces pad + cuFFT (+ crop) for complex64 1-D grids of power-of-two
// size (NUFFT_FFT1=0 keeps cuFFT, for tuning).  Set up on first use, since
// a type-3 plan learns its grid size at setpts.
bool fft1_wanted(const nufft_plan_s* p) {
    static const int on = env_int("NUFFT_FFT1", 1);
    return on && p->dim == 1 && !p->fft64 && fft1_supported(p->nup[0]);
}

bool use_fft1(nufft_plan_s* p) {
    if (!fft1_wanted(p)) return false;
    if (p->fft1.n != p->nup[0]) fft1_init(&p->fft1, p->nup[0]);
    return true;
}

// The pruned 3-D FFT of fft1.cu with the pad / crop fused replaces pad +
// cuFFT (type 2) and cuFFT + crop (type 1) for complex64 3-D grids whose
// sides are powers of two in [64, 2048] (NUFFT_FFTN=0 keeps cuFFT, for
// tuning).
bool fftn_wanted(const nufft_plan_s* p) {
    static const int on = env_int("NUFFT_FFTN", 1);
    return on && p->type != 3 && p->dim == 3 && !p->fft64 && fftn_supported(p->nup);
}

// A type-2 plan stores its FFT grid with a periodic halo when the pruned
// 3-D FFT writes it (complex64) and the TMA interpolation reads it; every
// 3-D interpolation kernel reads the halo layout.  NUFFT_GRID_HALO=0 keeps
// the plain layout (tuning).
bool halo_wanted(const nufft_plan_s* p) {
    static const int on = env_int("NUFFT_GRID_HALO", 1);
    static const int tma = env_int("NUFFT_INTERP_TMA", 1);
    return on && tma && p->type == 2 && fftn_wanted(p);
}

bool use_fftn(nufft_plan_s* p) {
    if (!fftn_wanted(p)) return false;
    if (p->fftn.n[0] != p->nup[0] || p->fftn.n[1] != p->nup[1] ||
        p->fftn.n[2] != p->nup[2])
        fftn_init(&p->fftn, p->nup, p->N);
    return true;
}

void execute_chunk(nufft_plan_s* p, const float2* in, float2* out, int nv,
                   int stage, cudaStream_t st) {
    const bool f1 = use_fft1(p);
    const bool inv = p->isign > 0;
    if (p->type == 1) {
        float2* sg = t1_spread_grid(p);
        if (stage == NUFFT_STAGE_ALL || stage == NUFFT_STAGE_SPREAD) {
            record(p, 0, st);
            NUFFT_CUDA(cudaMemsetAsync(sg, 0, sizeof(float2) * p->nupcells * nv, st));
            launch_spread(p->src, p->tg_src, p->w, in, p->src.M, nv, sg,
                          p->nvg_src, st);
            record(p, 1, st);
        }
        if (stage == NUFFT_STAGE_ALL || stage == NUFFT_STAGE_FINISH) {
            if (stage == NUFFT_STAGE_FINISH) {
                record(p, 0, st);
                record(p, 1, st);
            }
            if (f1) {                  // pass 1, then pass 2 with the crop
                fft1_cols(&p->fft1, sg, 0, nullptr, nv, inv, st);
                record(p, 2, st);
                fft1_rows(&p->fft1, out, p->N[0], p->dec[0], nv, inv, st);
                record(p, 3, st);
            } else if (use_fftn(p)) {  // pruned FFT with the crop fused
                fftn_crop(&p->fftn, sg, p->dec, out, nv, inv, st);
                record(p, 2, st);
                record(p, 3, st);
            } else {
                if (p->fft64)
                    launch_widen(sg, (double2*)p->gfft, p->nupcells * nv, st);
                run_fft(p, nv, inv, st);
                record(p, 2, st);
                launch_crop(p->dim, p->N, p->nup, p->dec, p->gfft, p->fft64, out, nv,
                            st);
                record(p, 3, st);
            }
        }
    } else if (p->type == 2) {
        if (stage == NUFFT_STAGE_ALL || stage == NUFFT_STAGE_SPREAD) {
            record(p, 0, st);
            if (f1) {                  // pass 1 with the pad, then pass 2
                fft1_cols(&p->fft1, in, p->N[0], p->dec[0], nv, inv, st);
                record(p, 1, st);
                fft1_rows(&p->fft1, p->gfft, 0, nullptr, nv, inv, st);
            } else if (use_fftn(p)) {  // pruned FFT with the pad fused
                record(p, 1, st);
                // an execute over a point set that reads only some planes:
                // the slab order computes just those (NUFFT_FFTN_SLAB=0
                // keeps the plain order and only skips their stores)
                static const int slab_on = env_int("NUFFT_FFTN_SLAB", 1);
                const bool pruned = stage == NUFFT_STAGE_ALL && p->halo && !p->xneed_all;
                if (!(pruned && slab_on &&
                      fftn_pad_slab(&p->fftn, in, p->dec, p->gfft, nv, inv, st, p->gh,
                                    p->xneed, p->d_xmap, p->d_xlist, p->nx_need)))
                    fftn_pad(&p->fftn, in, p->dec, p->gfft, nv, inv, st,
                             p->halo ? &p->gh : nullptr, pruned ? p->xneed : nullptr);
            } else {
                launch_pad(p->dim, p->N, p->nup, p->dec, in, p->gfft, p->fft64, nv,
                           st);
                record(p, 1, st);
                run_fft(p, nv, inv, st);
            }
            record(p, 2, st);
        }
        if (stage == NUFFT_STAGE_SPREAD) {
            record(p, 3, st);
            p->ev_recorded = p->profile;
            return;
        }
        if (stage == NUFFT_STAGE_FINISH) {
            record(p, 0, st);
            record(p, 1, st);
            record(p, 2, st);
        }
        if (!launch_interp_tma(p->src, p->tg_src, p->w, interp_tmap(p, p->tg_src),
                               interp_grid32(p), nv, out, p->src.M, p->d_exec_err, st))
            launch_interp(p->src, p->tg_src, p->w, p->gfft, p->fft64, nv, out,
                          p->src.M, p->nvg_src, st);
        record(p, 3, st);
    } else {
        record(p, 0, st);
        NUFFT_CUDA(cudaMemsetAsync(p->gspread, 0, sizeof(float2) * p->nfcells * nv, st));
        launch_spread(p->src, p->tg_src, p->w, in, p->src.M, nv, p->gspread,
                      p->nvg_src, st);
        if (f1) {
            fft1_cols(&p->fft1, p->gspread, p->nf[0], p->dec[0], nv, inv, st);
            record(p, 1, st);
            fft1_rows(&p->fft1, p->gfft, 0, nullptr, nv, inv, st);
        } else {
            launch_pad(p->dim, p->nf, p->nup, p->dec, p->gspread, p->gfft, p->fft64,
                       nv, st);
            record(p, 1, st);
            run_fft(p, nv, inv, st);
        }
        record(p, 2, st);
        if (!launch_interp_tma(p->tgt, p->tg_tgt, p->w2, interp_tmap(p, p->tg_tgt),
                               interp_grid32(p), nv, out, p->Ntgt, p->d_exec_err, st))
            launch_interp(p->tgt, p->tg_tgt, p->w2, p->gfft, p->fft64, nv, out,
                          p->Ntgt, p->nvg_tgt, st);
        record(p, 3, st);
    }
    p->ev_recorded = p->profile;
}

// Adjoint of a type-1 / type-2 plan on nv vectors: the other type with the
// opposite sign, on the plan's own sorted points, corrections and grids
// (the reference builds this sibling as a separate plan over the same
// points, mlx_nufft/api.py:347-388).  A type-1 plan's adjoint maps modes
// in[nv][N...] to points out[nv][M]; a type-2 plan's maps points
// in[nv][M] to modes out[nv][N...].
void adjoint_chunk_t12(nufft_plan_s* p, const float2* in, float2* out, int nv,
                       cudaStream_t st) {
    const bool f1 = use_fft1(p);
    const bool inv = p->isign < 0;             // sign of the adjoint: -isign
    if (p->type == 1) {
        if (f1) {
            fft1_cols(&p->fft1, in, p->N[0], p->dec[0], nv, inv, st);
            fft1_rows(&p->fft1, p->gfft, 0, nullptr, nv, inv, st);
        } else if (use_fftn(p)) {
            fftn_pad(&p->fftn, in, p->dec, p->gfft, nv, inv, st);
        } else {
            launch_pad(p->dim, p->N, p->nup, p->dec, in, p->gfft, p->fft64, nv, st);
            run_fft(p, nv, inv, st);
        }
        if (!launch_interp_tma(p->src, p->tg_src, p->w, interp_tmap(p, p->tg_src),
                               interp_grid32(p), nv, out, p->src.M, p->d_exec_err, st))
            launch_interp(p->src, p->tg_src, p->w, p->gfft, p->fft64, nv, out,
                          p->src.M, p->nvg_src, st);
        return;
    }
    float2* sg = p->gfft;
    if (p->fft64) {
        if (!p->gadj)
            p->gadj = (float2*)dmalloc(sizeof(float2) * p->nupcells * p->nbatch,
                                       "adjoint spread grid");
        sg = p->gadj;
    }
    NUFFT_CUDA(cudaMemsetAsync(sg, 0, sizeof(float2) * p->nupcells * nv, st));
    // the adjoint spreads into plain (halo-free) grids for the crop
    TileGeom tg = p->tg_src;
    set_no_halo(tg);
    launch_spread(p->src, tg, p->w, in, p->src.M, nv, sg, p->nvg_src, st);
    if (f1) {
        fft1_cols(&p->fft1, sg, 0, nullptr, nv, inv, st);
        fft1_rows(&p->fft1, out, p->N[0], p->dec[0], nv, inv, st);
        return;
    }
    if (use_fftn(p)) {
        fftn_crop(&p->fftn, sg, p->dec, out, nv, inv, st);
        return;
    }
    if (p->fft64) launch_widen(sg, (double2*)p->gfft, p->nupcells * nv, st);
    run_fft(p, nv, inv, st);
    launch_crop(p->dim, p->N, p->nup, p->dec, p->gfft, p->fft64, out, nv, st);
}

void drop_adjoint(nufft_plan_s* p) {
    if (p->adj) {
        nufft_plan_destroy(p->adj);
        p->adj = nullptr;
    }
}

// The type-3 sibling plan: the plan's targets as sources and its sources as
// targets, opposite sign, the plan's options (gpu_t3 construction of the
// reference's adjoint, mlx_nufft/api.py:367-372).
nufft_plan_s* t3_adjoint(nufft_plan_s* p, cudaStream_t st) {
    if (p->adj) return p->adj;
    nufft_opts o = p->opts;
    o.has_source_extent = 0;
    o.profile = 0;
    nufft_plan_t q = nullptr;
    int rc = nufft_plan_create(3, p->dim, nullptr, p->n_trans, p->eps, -p->isign, &o,
                               p->device, &q);
    if (rc != NUFFT_OK) fail(rc, "adjoint plan: " + g_last_error);
    rc = nufft_setpts(q, p->Ntgt, p->scopy[0], p->scopy[1], p->scopy[2], p->src.M,
                      p->xcopy[0], p->xcopy[1], p->xcopy[2], st);
    if (rc != NUFFT_OK) {
        const std::string msg = g_last_error;
        nufft_plan_destroy(q);
        fail(rc, "adjoint plan setpts: " + msg);
    }
    p->adj = q;
    return q;
}

// Grow the number of fine grids held by the plan so that nvec vectors run
// in one pass (shared point weights, one batched FFT), bounded by half of
// the free device memory.  Only when opts.max_batch == 0 (automatic).
void ensure_batch(nufft_plan_s* p, int nvec) {
    if (nvec <= p->nbatch || p->opts.max_batch > 0) return;
    size_t free_b = 0, tot = 0;
    NUFFT_CUDA(cudaMemGetInfo(&free_b, &tot));
    size_t per = fft_cell_bytes(p) * (size_t)p->gcells;
    if (p->type == 3) per += sizeof(float2) * (size_t)p->nfcells;
    else if (p->type == 1 && p->fft64) per += sizeof(float2) * (size_t)p->nupcells;
    if (fft1_wanted(p)) per += sizeof(float2) * (size_t)p->nupcells;  // FFT scratch
    if (fftn_wanted(p))
        per += sizeof(float2) * (size_t)(p->N[0] * p->nup[1] * p->nup[2]);
    const size_t have = per * (size_t)p->nbatch;
    const int64_t cap = (int64_t)((free_b / 2 + have) / per);
    const int nb = (int)std::min<int64_t>(nvec, std::max<int64_t>(cap, p->nbatch));
    if (nb <= p->nbatch) return;
    NUFFT_CUDA(cudaDeviceSynchronize());   // grids may still be in use
    p->nbatch = nb;
    alloc_grids(p);
    p->nvg_src = vectors_per_tile(p->tg_src, p->nbatch);
    if (p->type == 3) p->nvg_tgt = vectors_per_tile(p->tg_tgt, p->nbatch);
}

int64_t in_len(const nufft_plan_s* p) {
    return p->type == 2 ? p->K : p->src.M;
}
int64_t out_len(const nufft_plan_s* p) {
    return p->type == 1 ? p->K : (p->type == 2 ? p->src.M : p->Ntgt);
}

__global__ void k_split_cells(const int2* cell, int64_t n, int32_t* i1,
                              float* fr) {
    int64_t j = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
    if (j >= n) return;
    int2 c = cell[j];
    i1[j] = c.x;
    fr[j] = __int_as_float(c.y);
}

__global__ void k_iota(uint32_t* p, int64_t n) {
    int64_t j = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
    if (j < n) p[j] = (uint32_t)j;
}

// label window for execute_disjoint: out = groups - g0 if in [0, ng) else -1
__global__ void k_window_labels(const int32_t* g, int64_t n, int g0, int ng,
                                int32_t* out) {
    int64_t j = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
    if (j >= n) return;
    int v = g[j] - g0;
    out[j] = (v >= 0 && v < ng) ? v : -1;
}

void window_labels(const int32_t* g, int64_t n, int g0, int ng,
                         int32_t* out, cudaStream_t st) {
    k_window_labels<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(g, n, g0, ng, out);
    NUFFT_LAUNCH("k_window_labels");
}

}  // namespace nufft_impl

using namespace nufft_impl;

// =====================================================================
// C ABI
// =====================================================================
extern "C" {

void nufft_default_opts(nufft_opts* o) {
    if (!o) return;
    std::memset(o, 0, sizeof(*o));
    o->prec = NUFFT_PREC_CRIT64;
    o->method = NUFFT_METHOD_AUTO;
    o->sort_points = 1;
    o->kerevalmeth = 1;
}

int nufft_plan_create(int type, int dim, const int64_t* n_modes, int n_trans,
                      double eps, int isign, const nufft_opts* opts, int device,
                      nufft_plan_t* out) {
    return guarded([&] {
        if (!out) fail(NUFFT_ERR_ARG, "plan output pointer is NULL");
        *out = nullptr;
        if (type < 1 || type > 3) fail(NUFFT_ERR_ARG, "nufft_type must be 1, 2 or 3");
        if (dim < 1 || dim > 3) fail(NUFFT_ERR_ARG, "dim must be 1, 2 or 3");
        if (n_trans < 1) fail(NUFFT_ERR_ARG, "n_trans must be >= 1");
        if (!(eps > 0.0)) fail(NUFFT_ERR_ARG, "eps must be positive");
        if (type != 3 && !n_modes) fail(NUFFT_ERR_ARG, "n_modes is NULL");
        int ndev = 0;
        if (cudaGetDeviceCount(&ndev) != cudaSuccess || ndev == 0) {
            cudaGetLastError();
            fail(NUFFT_ERR_CUDA, "no CUDA device available");
        }
        if (device < 0 || device >= ndev) fail(NUFFT_ERR_ARG, "invalid device ordinal");
        DeviceGuard g(device);
        nufft_plan_s* p = new nufft_plan_s();
        try {
            p->type = type;
            p->dim = dim;
            p->device = device;
            p->n_trans = n_trans;
            p->isign = isign >= 0 ? 1 : -1;
            p->eps = eps;
            if (opts) p->opts = *opts;
            else nufft_default_opts(&p->opts);
            if (p->opts.prec < 0 || p->opts.prec > 3) fail(NUFFT_ERR_ARG, "invalid prec");
            if (type != 3 && (p->opts.prec == NUFFT_PREC_COORDS64 ||
                              p->opts.prec == NUFFT_PREC_PHASES64))
                fail(NUFFT_ERR_ARG, "prec must be 'fp32' or 'crit64' for types 1/2");
            p->nbatch = p->opts.max_batch > 0 ? std::min(p->opts.max_batch, n_trans)
                                              : n_trans;
            p->profile = p->opts.profile != 0;
            if (p->profile)
                for (int i = 0; i < 4; ++i) NUFFT_CUDA(cudaEventCreate(&p->ev[i]));
            p->d_err = (int*)dmalloc(sizeof(int), "error flag");
            NUFFT_CUDA(cudaMemset(p->d_err, 0, sizeof(int)));
            NUFFT_CUDA(cudaHostAlloc((void**)&p->h_exec_err, sizeof(int),
                                     cudaHostAllocMapped));
            *p->h_exec_err = 0;
            NUFFT_CUDA(cudaHostGetDevicePointer((void**)&p->d_exec_err, p->h_exec_err, 0));
            if (type != 3) {
                for (int d = 0; d < dim; ++d) p->N[d] = n_modes[d];
                create_t12(p);
            } else {
                create_t3(p);
            }
        } catch (...) {
            nufft_plan_destroy(p);
            throw;
        }
        *out = p;
    });
}

int nufft_setpts(nufft_plan_t p, int64_t M, const double* x, const double* y,
                 const double* z, int64_t N, const double* s, const double* t,
                 const double* u, void* stream) {
    return guarded([&] {
        if (!p) fail(NUFFT_ERR_ARG, "NULL plan");
        DeviceGuard g(p->device);
        check_exec_flag(p);
        cudaStream_t st = (cudaStream_t)stream;
        const double* xs[3] = {x, y, z};
        for (int d = 0; d < p->dim; ++d)
            if (!xs[d]) fail(NUFFT_ERR_ARG, "missing coordinate array");
        if (p->type != 3) {
            setpts_t12(p, M, xs, st);
        } else {
            const double* ss[3] = {s, t, u};
            for (int d = 0; d < p->dim; ++d)
                if (!ss[d]) fail(NUFFT_ERR_ARG, "missing target array");
            setpts_t3(p, M, xs, N, ss, st);
        }
    });
}

int nufft_set_sources(nufft_plan_t p, int64_t M, const double* x,
                      const double* y, const double* z, void* stream) {
    return guarded([&] {
        if (!p) fail(NUFFT_ERR_ARG, "NULL plan");
        DeviceGuard g(p->device);
        cudaStream_t st = (cudaStream_t)stream;
        const double* xs[3] = {x, y, z};
        for (int d = 0; d < p->dim; ++d)
            if (!xs[d]) fail(NUFFT_ERR_ARG, "missing coordinate array");
        if (p->type != 3) {
            setpts_t12(p, M, xs, st);
        } else {
            if (!p->points_set) fail(NUFFT_ERR_STATE, "setpts() must be called first");
            set_sources_t3(p, M, xs, true, st);
            drop_adjoint(p);
            keep_coords(p->xcopy, &p->xcap, p->dim, M, xs, st);
        }
    });
}

int nufft_execute_stage(nufft_plan_t p, int stage, const void* in, void* out,
                        int nvec, void* stream) {
    return guarded([&] {
        if (!p) fail(NUFFT_ERR_ARG, "NULL plan");
        if (!p->points_set) fail(NUFFT_ERR_STATE, "setpts() must be called before execute()");
        if (nvec < 1) fail(NUFFT_ERR_ARG, "nvec must be >= 1");
        if (stage != NUFFT_STAGE_ALL) {
            if (p->type == 3) fail(NUFFT_ERR_ARG, "stages apply to type-1 and type-2 plans");
            if (nvec > p->nbatch) fail(NUFFT_ERR_ARG, "staged execute: nvec exceeds the plan batch");
            if (stage != NUFFT_STAGE_SPREAD && stage != NUFFT_STAGE_FINISH)
                fail(NUFFT_ERR_ARG, "unknown stage");
        }
        if ((stage == NUFFT_STAGE_ALL || stage == NUFFT_STAGE_SPREAD) && !in)
            fail(NUFFT_ERR_ARG, "NULL input pointer");
        if ((stage == NUFFT_STAGE_ALL || stage == NUFFT_STAGE_FINISH) && !out)
            fail(NUFFT_ERR_ARG, "NULL output pointer");
        DeviceGuard g(p->device);
        check_exec_flag(p);
        cudaStream_t st = (cudaStream_t)stream;
        if (stage == NUFFT_STAGE_ALL) ensure_batch(p, nvec);
        const float2* fin = (const float2*)in;
        float2* fout = (float2*)out;
        const int64_t il = in_len(p), ol = out_len(p);
        const int64_t l0 = launch_count;
        struct Count {      // credited on every exit, exceptions included
            nufft_plan_s* p; int64_t l0;
            ~Count() { p->launches += launch_count - l0; }
        } count{p, l0};
        for (int v0 = 0; v0 < nvec; v0 += p->nbatch) {
            const int nv = std::min(p->nbatch, nvec - v0);
            execute_chunk(p, fin ? fin + v0 * il : nullptr,
                          fout ? fout + v0 * ol : nullptr, nv, stage, st);
        }
    });
}

int nufft_execute(nufft_plan_t p, const void* in, void* out, int nvec,
                  void* stream) {
    if (!in || !out) {
        set_last_error("NULL data pointer");
        return NUFFT_ERR_ARG;
    }
    return nufft_execute_stage(p, NUFFT_STAGE_ALL, in, out, nvec, stream);
}

int nufft_execute_adjoint(nufft_plan_t p, const void* in, void* out, int nvec,
                          void* stream) {
    return guarded([&] {
        if (!p) fail(NUFFT_ERR_ARG, "NULL plan");
        if (!p->points_set)
            fail(NUFFT_ERR_STATE, "setpts() must be called before execute_adjoint()");
        if (nvec < 1) fail(NUFFT_ERR_ARG, "nvec must be >= 1");
        if (!in || !out) fail(NUFFT_ERR_ARG, "NULL data pointer");
        DeviceGuard g(p->device);
        check_exec_flag(p);
        cudaStream_t st = (cudaStream_t)stream;
        const int64_t l0 = launch_count;
        struct Count {
            nufft_plan_s* p; int64_t l0;
            ~Count() { p->launches += launch_count - l0; }
        } count{p, l0};
        if (p->type == 3) {
            nufft_plan_s* q = t3_adjoint(p, st);
            const int rc = nufft_execute(q, in, out, nvec, stream);
            if (rc != NUFFT_OK) fail(rc, g_last_error);
            return;
        }
        ensure_batch(p, nvec);
        // adjoint input / output lengths: type 1 modes -> points, type 2
        // points -> modes
        const int64_t il = p->type == 1 ? p->K : p->src.M;
        const int64_t ol = p->type == 1 ? p->src.M : p->K;
        const float2* fin = (const float2*)in;
        float2* fout = (float2*)out;
        for (int v0 = 0; v0 < nvec; v0 += p->nbatch) {
            const int nv = std::min(p->nbatch, nvec - v0);
            adjoint_chunk_t12(p, fin + v0 * il, fout + v0 * ol, nv, st);
        }
    });
}

int nufft_get_grid(nufft_plan_t p, void** grid, int64_t* n_complex) {
    return guarded([&] {
        if (!p) fail(NUFFT_ERR_ARG, "NULL plan");
        // the complex64 spreading target (type 1: what SPREAD leaves for a
        // cross-GPU reduction before FINISH)
        if (grid) *grid = p->type == 1 ? t1_spread_grid(p) : p->gfft;
        if (n_complex) *n_complex = (p->type == 1 ? p->nupcells : p->gcells) * p->nbatch;
    });
}

int nufft_execute_disjoint(nufft_plan_t p, const void* c, const int32_t* groups,
                           int ngroups, void* out, void* stream) {
    return guarded([&] {
        if (!p) fail(NUFFT_ERR_ARG, "NULL plan");
        if (p->type != 1) fail(NUFFT_ERR_ARG, "execute_disjoint applies to type-1 plans");
        if (!p->points_set) fail(NUFFT_ERR_STATE, "setpts() must be called before execute()");
        if (ngroups < 0) fail(NUFFT_ERR_ARG, "ngroups must be >= 0");
        DeviceGuard g(p->device);
        cudaStream_t st = (cudaStream_t)stream;
        const float2* fc = (const float2*)c;
        float2* fo = (float2*)out;
        // groups processed nbatch at a time; a group index outside the
        // current window is skipped by offsetting the labels on the fly.
        int32_t* shifted = (int32_t*)dmalloc(sizeof(int32_t) * p->src.M, "group labels");
        const int64_t l0 = launch_count;
        try {
            for (int g0 = 0; g0 < ngroups; g0 += p->nbatch) {
                const int ng = std::min(p->nbatch, ngroups - g0);
                float2* sg = t1_spread_grid(p);
                NUFFT_CUDA(cudaMemsetAsync(sg, 0, sizeof(float2) * p->nupcells * ng, st));
                // labels relative to this window; out-of-window -> -1
                window_labels(groups, p->src.M, g0, ng, shifted, st);
                launch_spread_groups(p->src, p->tg_src, p->w, fc, shifted, sg, st);
                if (use_fftn(p)) {
                    fftn_crop(&p->fftn, sg, p->dec, fo + (int64_t)g0 * p->K, ng,
                              p->isign > 0, st);
                    continue;
                }
                if (use_fft1(p)) {
                    fft1_cols(&p->fft1, sg, 0, nullptr, ng, p->isign > 0, st);
                    fft1_rows(&p->fft1, fo + (int64_t)g0 * p->K, p->N[0], p->dec[0], ng,
                              p->isign > 0, st);
                    continue;
                }
                if (p->fft64) launch_widen(sg, (double2*)p->gfft, p->nupcells * ng, st);
                run_fft(p, ng, p->isign > 0, st);
                launch_crop(p->dim, p->N, p->nup, p->dec, p->gfft, p->fft64,
                            fo + (int64_t)g0 * p->K, ng, st);
            }
        } catch (...) {
            p->launches += launch_count - l0;
            NUFFT_CUDA(cudaStreamSynchronize(st));
            dfree(shifted);
            throw;
        }
        p->launches += launch_count - l0;
        NUFFT_CUDA(cudaStreamSynchronize(st));
        dfree(shifted);
    });
}

int nufft_plan_destroy(nufft_plan_t p) {
    if (!p) return NUFFT_OK;
    return guarded([&] {
        int cur = 0;
        cudaGetDevice(&cur);
        cudaSetDevice(p->device);
        cudaDeviceSynchronize();
        destroy_ffts(p);
        fft1_free(&p->fft1);
        fftn_free(&p->fftn);
        free_pointset(&p->src);
        free_pointset(&p->tgt);
        for (int d = 0; d < 3; ++d) dfree(p->dec[d]);
        dfree(p->gfft);
        dfree(p->gspread);
        dfree(p->xneed);
        dfree(p->d_xmap);
        dfree(p->d_xlist);
        dfree(p->d_ftd);
        dfree(p->d_fta);
        dfree(p->d_err);
        if (p->h_exec_err) cudaFreeHost(p->h_exec_err);
        dfree(p->gadj);
        for (int d = 0; d < 3; ++d) {
            dfree(p->xcopy[d]);
            dfree(p->scopy[d]);
        }
        drop_adjoint(p);
        for (int i = 0; i < 4; ++i)
            if (p->ev[i]) cudaEventDestroy(p->ev[i]);
        cudaSetDevice(cur);
        delete p;
    });
}

int nufft_plan_check(nufft_plan_t p, void* stream) {
    return guarded([&] {
        if (!p) fail(NUFFT_ERR_ARG, "NULL plan");
        DeviceGuard g(p->device);
        NUFFT_CUDA(cudaStreamSynchronize((cudaStream_t)stream));
        check_exec_flag(p);
    });
}

int nufft_plan_get_info(nufft_plan_t p, nufft_plan_info* info) {
    return guarded([&] {
        if (!p || !info) fail(NUFFT_ERR_ARG, "NULL argument");
        std::memset(info, 0, sizeof(*info));
        info->type = p->type;
        info->dim = p->dim;
        info->n_trans = p->n_trans;
        info->isign = p->isign;
        info->w = p->w;
        info->w2 = p->w2;
        info->beta = p->beta;
        info->beta2 = p->beta2;
        info->eps = p->eps;
        info->upsampfac = p->sigma;
        info->sigma_inner = p->sigma_in;
        for (int d = 0; d < 3; ++d) {
            info->n_modes[d] = p->N[d];
            info->nf[d] = p->nf[d];
            info->n_up[d] = p->nup[d];
            info->C[d] = p->C[d];
            info->D[d] = p->D[d];
            info->gam[d] = p->gam[d];
            info->bin[d] = p->tg_src.m[d];
        }
        info->M = p->src.M;
        info->N_tgt = p->Ntgt;
        info->tiled = p->src.tiled ? 1 : 0;
        info->nsub = p->src.nsub;
        info->nsub_tgt = p->tgt.nsub;
        int64_t b = (int64_t)fft_cell_bytes(p) * (p->nupcells * p->nbatch);
        if (p->type == 1 && p->fft64) b += sizeof(float2) * p->nupcells * p->nbatch;
        if (p->type == 3) b += sizeof(float2) * p->nfcells * p->nbatch;
        b += p->src.cap * (8 * p->dim + 4 + (p->src.phase ? 8 : 0));
        b += p->tgt.cap * (8 * p->dim + 4 + (p->tgt.phase ? 8 : 0));
        info->device_bytes = b;
        info->kernel_launches = p->launches;
        info->fft_execs = p->fft_execs;
        info->fft64 = p->fft64 ? 1 : 0;
        info->fft_own = (fft1_wanted(p) || fftn_wanted(p)) ? 1 : 0;
        info->grid_cells = p->type == 1 ? p->nupcells : p->gcells;
        for (int d = 0; d < 3; ++d) {
            const bool h = p->type == 2 && p->halo && d < p->dim;
            info->grid_ext[d] = h ? p->gh.P[d] : (d < p->dim ? p->nup[d] : 1);
            info->grid_lo[d] = h ? p->gh.lo[d] : 0;
        }
    });
}

int nufft_get_stage_times(nufft_plan_t p, float* ms, int n) {
    int count = 0;
    int rc = guarded([&] {
        if (!p) fail(NUFFT_ERR_ARG, "NULL plan");
        if (!p->profile) fail(NUFFT_ERR_STATE, "plan was not created with opts.profile = 1");
        if (!p->ev_recorded) fail(NUFFT_ERR_STATE, "no execute has been recorded");
        NUFFT_CUDA(cudaEventSynchronize(p->ev[3]));
        float t[4];
        for (int i = 0; i < 3; ++i)
            NUFFT_CUDA(cudaEventElapsedTime(&t[i], p->ev[i], p->ev[i + 1]));
        NUFFT_CUDA(cudaEventElapsedTime(&t[3], p->ev[0], p->ev[3]));
        for (int i = 0; i < 4 && i < n; ++i) ms[i] = t[i];
        count = 4;
    });
    return rc == NUFFT_OK ? count : rc;
}

int nufft_plan_set_profile(nufft_plan_t p, int on) {
    return guarded([&] {
        if (!p) fail(NUFFT_ERR_ARG, "NULL plan");
        DeviceGuard g(p->device);
        if (on && !p->ev[0])
            for (int i = 0; i < 4; ++i) NUFFT_CUDA(cudaEventCreate(&p->ev[i]));
        p->profile = on != 0;
        if (!p->profile) p->ev_recorded = false;
    });
}

int nufft_debug_points(nufft_plan_t p, int which, int32_t* i1, float* fr,
                       uint32_t* perm, void* stream) {
    return guarded([&] {
        if (!p) fail(NUFFT_ERR_ARG, "NULL plan");
        if (!p->points_set) fail(NUFFT_ERR_STATE, "setpts() has not been called");
        const PointSet& ps = which == 0 ? p->src : p->tgt;
        if (which == 1 && p->type != 3) fail(NUFFT_ERR_ARG, "targets exist for type 3 only");
        DeviceGuard g(p->device);
        cudaStream_t st = (cudaStream_t)stream;
        const unsigned blocks = (unsigned)((ps.M + 255) / 256);
        for (int d = 0; d < p->dim; ++d) {
            if (i1 && fr) {
                k_split_cells<<<blocks, 256, 0, st>>>(ps.cell[d], ps.M, i1 + d * ps.M,
                                                      fr + d * ps.M);
                NUFFT_LAUNCH("k_split_cells");
            }
        }
        if (perm) {
            if (ps.sorted)
                NUFFT_CUDA(cudaMemcpyAsync(perm, ps.perm, 4 * ps.M,
                                           cudaMemcpyDeviceToDevice, st));
            else {
                k_iota<<<blocks, 256, 0, st>>>(perm, ps.M);
                NUFFT_LAUNCH("k_iota");
            }
        }
    });
}

int nufft_expi(int ncomp, const double* const* comps, int64_t n, int isign,
               void* out, void* stream) {
    return guarded([&] {
        if (!comps || (!out && n > 0)) fail(NUFFT_ERR_ARG, "NULL argument");
        for (int c = 0; c < ncomp; ++c)
            if (!comps[c] && n > 0) fail(NUFFT_ERR_ARG, "NULL phase component");
        launch_expi(ncomp, comps, n, isign, (float2*)out, (cudaStream_t)stream);
    });
}

int nufft_kernel_params(double eps, double upsampfac, int* w, double* beta) {
    return guarded([&] {
        if (!w || !beta) fail(NUFFT_ERR_ARG, "NULL output");
        if (!(eps > 0.0)) fail(NUFFT_ERR_ARG, "eps must be positive");
        kernel_params(eps, upsampfac, w, beta);
    });
}

int64_t nufft_next235even(int64_t n) { return next235even(n); }

int nufft_kernel_ft(int64_t n, const double* xi, double beta, int w, double* out) {
    return guarded([&] {
        if (n > 0 && (!xi || !out)) fail(NUFFT_ERR_ARG, "NULL argument");
        std::vector<double> dq, aq;
        kernel_ft_nodes(beta, w, &dq, &aq);
        for (int64_t i = 0; i < n; ++i) out[i] = phihat_host(xi[i], dq, aq);
    });
}

int nufft_set_nhg_type3(double S, double X, double upsampfac, int w,
                        int64_t* nf, double* h, double* gam) {
    return guarded([&] {
        if (!nf || !h || !gam) fail(NUFFT_ERR_ARG, "NULL output");
        set_nhg_type3(S, X, upsampfac, w, nf, h, gam);
    });
}

int nufft_last_error(char* buf, int len) {
    const std::string& e = nufft::g_last_error;
    if (buf && len > 0) {
        const int n = std::min<int>(len - 1, (int)e.size());
        std::memcpy(buf, e.data(), n);
        buf[n] = 0;
    }
    return (int)e.size();
}

const char* nufft_version(void) { return "nufft_b200 0.1.0 (sm_100a)"; }

int nufft_device_count(void) {
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess) {
        cudaGetLastError();
        return 0;
    }
    return n;
}

}  // extern "C"

