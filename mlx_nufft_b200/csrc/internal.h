// internal.h -- declarations shared by the translation units of
// libnufft_b200.so.  Not part of the public C ABI (include/nufft_b200.h).
#pragma once

#include <cstdint>
#include <string>
#include <vector>

#include <cuda.h>
#include <cuda_runtime.h>

namespace nufft {

constexpr double kPi = 3.141592653589793238462643383279502884;
// 2*pi as the nearest double (== 2.0 * numpy.pi) and the remainder, used
// for the Cody-Waite reduction mod 2*pi (Cody & Waite, "Software Manual
// for the Elementary Functions", 1980).
constexpr double kTwoPi = 6.283185307179586;
constexpr double kTwoPiLo = 2.4492935982947064e-16;

// ---------------------------------------------------------------------
// errors: every C-ABI entry converts a thrown Error into a status code.
struct Error {
    int code;
    std::string msg;
};
[[noreturn]] void fail(int code, const std::string& msg);
void check_cuda(cudaError_t e, const char* what);
void set_last_error(const std::string& msg);

#define NUFFT_CUDA(call) ::nufft::check_cuda((call), #call)
// Every kernel launch in this library is followed by NUFFT_LAUNCH, which
// checks the launch and counts it on the calling host thread (plans report
// the launches of their executes from the difference of this count).
inline thread_local int64_t launch_count = 0;
#define NUFFT_LAUNCH(what) \
    (++::nufft::launch_count, ::nufft::check_cuda(cudaGetLastError(), what))

// ---------------------------------------------------------------------
// host numerics (sizing.cpp) -- restatements of mlx_nufft/sizing.py
int64_t next235even(int64_t n);
void kernel_params(double eps, double upsampfac, int* w, double* beta);
// 128-node Gauss-Legendre nodes d_q on [0, w/2] and weights a_q =
// wq_q * psi(d_q) such that phihat(xi) = 2 * sum_q a_q cos(xi d_q).
void kernel_ft_nodes(double beta, int w, std::vector<double>* d,
                     std::vector<double>* a);
double kernel_ft(double xi, double beta, int w);
void set_nhg_type3(double S, double X, double upsampfac, int w, int64_t* nf,
                   double* h, double* gam);
// Monomial coefficients coef[k * w + l] (k = 0..deg) of the per-tap
// polynomials psi(l - fr) = sum_k coef[k][l] t^k, t = fr - (w/2 - 1/2).
void es_poly_coeffs(int w, double beta, int deg, float* coef);

// Kernel-width limits and the polynomial degree used for width W.
constexpr int kMaxW = 16;
constexpr int kMaxTapRounds = 4;      // ceil(W^2 / 32) for W <= 10
constexpr int kMaxDeg = kMaxW + 2;
__host__ __device__ constexpr int es_degree(int w) { return w + 2; }

// ES kernel polynomial coefficients, passed to the kernels by value so that
// every coefficient is a constant-bank operand of its FFMA.
struct EsPoly {
    float c[kMaxDeg + 1][kMaxW];
};
EsPoly make_es_poly(int w, double beta);

// ---------------------------------------------------------------------
// geometry handed to the device kernels by value.

// How one nonuniform coordinate becomes (cell index i1, fraction fr).
enum CellKind : int {
    CELL_FOLD = 0,    // types 1/2: xi = mod(x, 2pi) / h           (nd.py:152-165)
    CELL_T3SRC = 1,   // type-3 sources: ((x - C)/gam)/h + nf/2     (gpu_t3.py:486-490)
    CELL_T3TGT = 2,   // type-3 targets: (s - D)*(h*gam)/h2 + n/2   (gpu_t3.py:357-366)
};

struct CellParams {
    int kind;             // CellKind
    int dim;
    int fp32;             // 1: rescale in fp32 (prec "fp32" / "phases64")
    int halfw;            // w / 2 (integer division), bin offset
    double halfw_d;       // w / 2.0
    int64_t n[3];         // grid extent the cells live on
    double h[3];          // CELL_FOLD: 2pi/n ; CELL_T3SRC: 2pi/nf
    double a[3];          // CELL_T3SRC: C ; CELL_T3TGT: D
    double b[3];          // CELL_T3SRC: gam ; CELL_T3TGT: h*gam (python double)
    double c[3];          // CELL_T3SRC: nf/2.0 ; CELL_T3TGT: 2pi/n_up
    double e[3];          // CELL_T3TGT: n_up/2.0
    int m[3];             // bin extent
    int nb[3];            // bins per dimension
    // Caller-order chunking of the sort (0: off).  With chunking the sort
    // key is (j / chunk, bin), so all subproblems of one chunk touch only
    // that chunk's slice of the caller-ordered strengths / outputs, which
    // stays L2-resident while it is being gathered or scattered.
    int64_t chunk;
    // Interpolation point sets ordered inside each subproblem (cell_order):
    // the shared-tile strides (cells) of the interpolation kernel that will
    // read them, per dimension.  Non-zero: points are dealt round-robin over
    // the 16 residues (sum_d l_d rs[d]) mod 16 of their first tap's tile
    // index, so the 16 lanes of a half-warp read 16 distinct 8-byte bank
    // pairs (no shared-memory bank conflicts); zero: plain cell order.
    int rs[3];
};

struct TileGeom {
    int dim;
    int n[3];             // grid extent (unused dims 1)
    int64_t ncells;       // prod n
    int m[3];             // bin extent
    int nb[3];            // bins per dimension
    int T[3];             // tile extent m + w - 1 (unused dims 1)
    uint32_t tdiv[3];     // ceil(2^32 / T[d]) for T[d] > 1 (division by T)
    int tcells;           // prod T
    int halfw;            // w / 2
    float c2w;            // (float)(2.0 / w)
    float beta;           // (float) beta
    int keval;            // 1: polynomial weights, 0: exp/sqrt per tap
    EsPoly poly;          // ES kernel as per-tap polynomials in fr
    // 3-D plane-owned spreading (k_spread_planes): shared row stride S2 >= T[2]
    // and, per round r and lane l, the in-plane tap (y << 4 | x) of lane l
    // (0xff: idle), chosen so each half-warp's 16 accesses hit 16 distinct
    // 8-byte bank pairs; rounds = ceil(W^2 / 32).
    int S2;
    uint8_t tapmap[kMaxTapRounds * 32];
    // the same for tiles of vector pairs (16-byte cells, one float4 = two
    // vectors' complex64): row stride S4, each quarter-warp's 8 accesses
    // on 8 distinct 16-byte bank quads
    int S4;
    uint8_t tapmap4[kMaxTapRounds * 32];
    // Layout of the grid a 3-D interpolation reads (GridHalo): cell i of
    // dimension d at index i + lo[d] of an extent P[d] = lo[d] + n[d] + hi,
    // pcells cells per vector.  No halo: lo = 0, P = n, pcells = ncells.
    int lo[3];
    int P[3];
    int64_t pcells;
};

// The no-halo layout (lo = 0, P = n, pcells = ncells) of a geometry whose
// n and ncells are set.
inline void set_no_halo(TileGeom& tg) {
    for (int d = 0; d < 3; ++d) {
        tg.lo[d] = 0;
        tg.P[d] = tg.n[d];
    }
    tg.pcells = tg.ncells;
}

// Periodic halo of a 3-D fine grid: the cells within lo[d] below and hi[d]
// above the grid in dimension d hold copies of the cells one period away,
// so that every tile of a 3-D interpolation lies inside the stored array
// (no wrap).  P[d] = lo[d] + n[d] + hi[d].
struct GridHalo {
    int lo[3];
    int hi[3];
    int P[3];
};

// Elements allocated past M in every per-point array (cells, permutation,
// phases): 16-byte-aligned bulk copies of a subproblem's range may read up
// to 3 elements beyond its end.
constexpr int64_t kPointSlack = 16;
// Largest subproblem (points) of the 1-D streamed interpolation, whose
// shared-memory stage holds a subproblem's cells and permutation.
constexpr int kStreamMsubMax = 1024;

// One sorted (or caller-ordered) set of nonuniform points on the device.
struct PointSet {
    int dim = 0;
    int64_t M = 0;
    int2* cell[3] = {nullptr, nullptr, nullptr};  // (i1, fr bits) per point
    uint32_t* perm = nullptr;   // sorted position -> caller index (null: identity)
    int4* subs = nullptr;       // (start, count, bin, 0) per subproblem
    int64_t nsub = 0;
    int msub = 0;               // points per subproblem at most
    int64_t cap = 0;            // allocated points
    int64_t subcap = 0;         // allocated subproblems
    float2* phase = nullptr;    // type 3: prephase / postphase, sorted order
    int* sched = nullptr;       // 2 ints: dynamic subproblem scheduler state
    bool sorted = false;
    bool tiled = false;
    // kept across setpts calls (re-pointing allocates nothing once sized):
    // sort scratch, and the second cell / permutation buffers of the
    // per-subproblem cell-order pass
    void* scratch = nullptr;
    size_t scratch_bytes = 0;
    int2* cell_alt[3] = {nullptr, nullptr, nullptr};
    uint32_t* perm_alt = nullptr;
};

// Raise a kernel's dynamic shared-memory limit to `bytes` when it exceeds
// the 48 KB default (host-side attribute call, cached per kernel).
void ensure_smem(const void* kernel, size_t bytes);

// Programmatic dependent launch: a kernel launched this way may be
// scheduled while the previous kernel in its stream drains; its first
// action is griddepcontrol.wait (grid_dep_wait), so it touches no memory
// before that kernel has completed.  NUFFT_PDL=0 launches normally.
bool pdl_on();
template <typename... KArgs, typename... Args>
void launch_dependent(void (*k)(KArgs...), dim3 grid, dim3 block, size_t smem,
                      cudaStream_t st, Args... args) {
    if (!pdl_on()) {
        k<<<grid, block, smem, st>>>(args...);
        return;
    }
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = at;
    cfg.numAttrs = 1;
    check_cuda(cudaLaunchKernelEx(&cfg, k, args...), "cudaLaunchKernelEx");
}

// Two-pass FFT of a power-of-two 1-D fine grid (fft1.cu), n = N1 * N2.
struct Fft1 {
    int n = 0, N1 = 0, N2 = 0;   // n == 0: not in use
    float2* tw = nullptr;        // twiddle tables (device)
    float2* tmp = nullptr;       // pass-1 output, tmp_batch grids
    int tmp_batch = 0;
};
bool fft1_supported(int64_t n);
void fft1_init(Fft1* f, int64_t n);
void fft1_free(Fft1* f);
void fft1_reserve(Fft1* f, int nv);
// pass 1 into f->tmp: with dec, `in` is nv mode vectors of length N that are
// padded (times dec) into the fine grid on the fly; without, nv fine grids
void fft1_cols(Fft1* f, const float2* in, int64_t N, const float* dec, int nv,
               bool inv, cudaStream_t st);
// pass 2 from f->tmp: with dec, the in-band cells times dec into nv mode
// vectors of length N (crop); without, nv fine grids in natural order
void fft1_rows(Fft1* f, float2* out, int64_t N, const float* dec, int nv, bool inv,
               cudaStream_t st);

// Pruned three-pass FFT of a 3-D power-of-two fine grid (each n_d in
// [64, 2048]) with the pad (types 2) or crop (type 1) fused (fft1.cu).
struct Fftn {
    int n[3] = {0, 0, 0};        // fine grid (n[0] == 0: not in use)
    int N[3] = {0, 0, 0};        // mode box
    float2* tw = nullptr;        // W_{n_d} tables, d = 0, 1, 2
    float2* tmp = nullptr;       // scratch B[m0][y][z], tmp_batch grids
    int tmp_batch = 0;
};
bool fftn_supported(const int64_t* n);
void fftn_init(Fftn* f, const int64_t* n, const int64_t* N);
void fftn_free(Fftn* f);
int64_t fftn_scratch_cells(const Fftn& f);
// nv mode boxes (times the corrections dec[d]) -> nv transformed fine grids;
// with a halo (non-null) each grid is stored padded, halo copies included,
// prod P cells apart; with need (halo only) just the stored planes of
// dimension 0 with need[s] != 0 are written
void fftn_pad(Fftn* f, const float2* modes, const float* const* dec, float2* grid,
              int nv, bool inv, cudaStream_t st, const GridHalo* halo = nullptr,
              const uint8_t* need = nullptr);
// The same for a halo grid of which only the nx canonical planes of
// dimension 0 in xlist (xmap: fine plane -> index in xlist, or -1) and the
// stored planes marked in need are wanted: the X pass first, then Y and Z
// over those planes only.  False (nothing launched) when the scratch planes
// do not fit.
bool fftn_pad_slab(Fftn* f, const float2* modes, const float* const* dec, float2* grid,
                   int nv, bool inv, cudaStream_t st, const GridHalo& h,
                   const uint8_t* need, const int* xmap, const int* xlist, int nx);
// nv fine grids -> nv mode boxes of the transform times dec[d]; the grids are
// overwritten (used as scratch)
void fftn_crop(Fftn* f, float2* grid, const float* const* dec, float2* modes, int nv,
               bool inv, cudaStream_t st);

// CTAs for a persistent launch of `kernel` (256 threads, `smem` bytes):
// resident CTAs per SM x SMs, capped at `work` items.
int persistent_grid(const void* kernel, size_t smem, int64_t work,
                    int threads = 256);

// ---------------------------------------------------------------------
// device memory helpers
void* dmalloc(size_t bytes, const char* what);
void dfree(void* p);

// ---------------------------------------------------------------------
// points.cu
// Count + scan + scatter bin sort (or plain caller-order cells when
// sort == false) of M points with coordinates coords[0..dim).
// `phase_mode`: 0 none, 1 type-3 prephase (sources), 2 type-3 post (targets).
struct PhaseParams {
    int mode;            // 0 none, 1 prephase, 2 post
    int isign;
    int fp32;            // phases computed in fp32 (prec fp32 / coords64)
    double D[3];         // prephase: e^{i isign sum D_d x_d}
    double C[3];         // post: e^{i isign sum C_d (s_d - D_d)} / prod phihat
    const double* ftd;   // device: 128 quadrature nodes d_q (post)
    const double* fta;   // device: 128 weights a_q (post)
    int nq;
};
// cell_order: also order the points of each subproblem by cell
// (interpolation point sets in 1-D and 3-D: fewer bank conflicts in the tile
// gathers; measured slower for spreading, whose shared atomics then
// collide, and for the 2-D interpolation).
void build_pointset(PointSet* ps, const CellParams& cp, int64_t M,
                    const double* const* coords, bool sort, bool tiled,
                    int msub, bool cell_order, const PhaseParams& pp,
                    int* d_err, cudaStream_t st);
void free_pointset(PointSet* ps);
// min/max of `n` device arrays of length M each; out: 2*n doubles (min,max)
void device_minmax(int n, const double* const* arrs, int64_t M, double* out,
                   cudaStream_t st);

// spreadinterp.cu
// Spread nvec strength vectors (c, vector stride cstride) onto nvec fine
// grids (grid stride = tg.ncells), accumulating (grid must be zeroed).
void launch_spread(const PointSet& ps, const TileGeom& tg, int w,
                   const float2* c, int64_t cstride, int nvec,
                   float2* grid, int nvg, cudaStream_t st);
// Interpolate nvec grids (complex64, or complex128 when grid64) at the
// points into out (vector stride ostride), multiplying by ps.phase when
// present.
// 3-D interpolation with TMA-staged tiles (interp_tma.cu): the tensor map
// over a plan's nbatch complex64 fine grids, and the launcher (false: not
// applicable, use launch_interp).
bool make_grid_tmap(CUtensorMap* map, const float2* grid, const TileGeom& tg,
                    int nbatch);
// Row stride (cells) of the TMA-staged 3-D tile: T[2] + 1 rounded up to even.
int tma_box_x(const TileGeom& tg);
// need[s] = 1 for every stored plane s (dimension 0, halo layout of tg) that
// a tile of the point set's subproblems covers, and for the interior plane
// each of those copies (one period away); need[] is not cleared first.
void mark_tile_planes(const PointSet& ps, const TileGeom& tg, uint8_t* need,
                      cudaStream_t st);
bool launch_interp_tma(const PointSet& ps, const TileGeom& tg, int w,
                       const CUtensorMap* map, const float2* grid, int nvec,
                       float2* out, int64_t ostride, int* err, cudaStream_t st);
// plan error-flag bits (device int): non-finite coordinate, tile-copy wait
// timed out
constexpr int kErrNonFinite = 1;
constexpr int kErrTileWait = 4;

void launch_interp(const PointSet& ps, const TileGeom& tg, int w,
                   const void* grid, bool grid64, int nvec, float2* out,
                   int64_t ostride, int nvg, cudaStream_t st);
// Largest dynamic shared memory a tile kernel may use (bytes).
int tile_smem_limit();
// Spread one group of a disjoint-support batch: point j goes to grid
// groups[perm[j]] only (global-memory atomics).
void launch_spread_groups(const PointSet& ps, const TileGeom& tg, int w,
                          const float2* c, const int32_t* groups,
                          float2* grid, cudaStream_t st);

// deconv.cu
// Type-1 crop: fk[v][m] = grid[v][r(m)] * prod dec_d[m_d]   (nd.py:416-435)
// (grid complex64, or complex128 when grid64)
void launch_crop(int dim, const int64_t* N, const int64_t* n,
                 const float* const* dec, const void* grid, bool grid64,
                 float2* fk, int nvec, cudaStream_t st);
// Pad: H[v][r] = in-band ? f[v][m(r)] * prod dec_d[m_d] : 0
// (types 2 and 3: nd.py:878-906, gpu_t3.py:629-651); H complex64, or
// complex128 when grid64.
void launch_pad(int dim, const int64_t* N, const int64_t* n,
                const float* const* dec, const float2* f, void* H,
                bool grid64, int nvec, cudaStream_t st);
// complex64 -> complex128 copy of n elements (fp64 FFT input)
void launch_widen(const float2* in, double2* out, int64_t n, cudaStream_t st);
// e^{i isign sum_c comps[c][j]}  (dfmath.py:29-54)
void launch_expi(int ncomp, const double* const* comps, int64_t n, int isign,
                 float2* out, cudaStream_t st);

}  // namespace nufft
