/*
 * nufft_b200.h -- C ABI of libnufft_b200.so, the B200 (sm_100a) NUFFT core.
 *
 * Every entry point is `extern "C"`, takes plain pointers, sizes and an
 * opaque plan handle, and returns an int status (NUFFT_OK == 0, < 0 on
 * error; nufft_last_error() gives the message of the calling thread's last
 * failure).  No torch or CUDA C++ types appear in the signatures: streams
 * are passed as `void*` (a cudaStream_t / CUstream, NULL = legacy default
 * stream), device buffers as `void*` / typed pointers to device memory.
 *
 * The reference (mlx-nufft) is a Python package whose GPU work runs through
 * MLX; its only C ABI is the VkFFT bridge
 * `int vkfft_fft2_inplace(void*, uint64_t, uint64_t, uint64_t, int, int)`
 * (vkfft_bridge/vkfft_bridge.cpp:51-71), whose conventions (caller-owned
 * device pointer, int status 0 / negative) this header follows.  Each entry
 * point below names the reference method it replaces.
 *
 * Conventions (identical to the reference, mlx_nufft/nd.py:1-21,
 * mlx_nufft/api.py:12-21):
 *   type 1:  f[k] = sum_j c[j] exp(i*isign * k . x_j)
 *   type 2:  c[j] = sum_k f[k] exp(i*isign * k . x_j)
 *   type 3:  f[k] = sum_j c[j] exp(i*isign * s_k . x_j)
 *   modes k_d are integers in [-(N_d/2), (N_d-1)/2] (modeord = 0), stored
 *   C-order (last dimension fastest); points x are folded mod 2*pi.
 *   Strengths / modes / outputs are complex64 (interleaved float re, im).
 *   Coordinates are fp64.
 */
#ifndef NUFFT_B200_H
#define NUFFT_B200_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes --------------------------------------------------- */
#define NUFFT_OK               0
#define NUFFT_ERR_ARG         -1  /* bad argument / shape (Python: ValueError) */
#define NUFFT_ERR_OOM         -2  /* device allocation failed                 */
#define NUFFT_ERR_CUDA        -3  /* CUDA runtime error                       */
#define NUFFT_ERR_CUFFT       -4  /* cuFFT error                              */
#define NUFFT_ERR_STATE       -5  /* execute before setpts (RuntimeError)     */
#define NUFFT_ERR_RANGE       -6  /* type-3 re-point outside frozen extent    */
#define NUFFT_ERR_UNSUPPORTED -7  /* valid request this build cannot serve    */

/* ---- precision of the plan-time geometry (mlx_nufft/gpu_t3.py:302) ---- */
#define NUFFT_PREC_CRIT64   0   /* coordinate rescale and phases in fp64 (default) */
#define NUFFT_PREC_FP32     1   /* both in fp32                                    */
#define NUFFT_PREC_COORDS64 2   /* coordinates fp64, phases fp32 (type 3 only)     */
#define NUFFT_PREC_PHASES64 3   /* coordinates fp32, phases fp64 (type 3 only)     */

/* ---- spreading / interpolation method (mlx_nufft/nd.py:389-411) ------ */
#define NUFFT_METHOD_AUTO   0   /* library picks                               */
#define NUFFT_METHOD_TILED  1   /* bin-sorted subproblems, shared-memory tile   */
                                /* (the reference's "od")                       */
#define NUFFT_METHOD_GLOBAL 2   /* one thread per point on the global grid      */
                                /* (the reference's "gm")                       */

/* ---- execute stages (nufft_execute_stage) ---------------------------- */
#define NUFFT_STAGE_ALL     0   /* whole transform == nufft_execute            */
#define NUFFT_STAGE_SPREAD  1   /* type 1: zero the fine grid(s) and spread;   */
                                /* type 2: pad/deconvolve the modes + FFT      */
#define NUFFT_STAGE_FINISH  2   /* type 1: FFT + deconvolve/crop of the grid(s);*/
                                /* type 2: interpolate from the fine grid(s)    */

typedef struct nufft_plan_s* nufft_plan_t;

typedef struct nufft_opts {
    double upsampfac;      /* 0 => type default: 2.0 (types 1/2), 1.25 (type 3)   */
    double sigma_inner;    /* type 3 inner-grid upsampling; 0 => upsampfac        */
    int    prec;           /* NUFFT_PREC_*                                        */
    int    method;         /* NUFFT_METHOD_*                                      */
    int    sort_points;    /* 1 (default): bin-sort points in setpts               */
    int    max_batch;      /* vectors per device pass; 0 => n_trans                */
    int    profile;        /* 1: record CUDA events around every stage             */
    int    has_source_extent;  /* type 3: size from source_extent, not from x     */
    double source_extent[6];   /* type 3: (lo, hi) per dimension                  */
    int    kerevalmeth;    /* ES kernel evaluation (finufft spread_kerevalmeth): */
                           /* 1 per-tap polynomials (default), 0 exp/sqrt      */
    int    fft_prec;       /* fine-grid FFT precision: 0 auto (fp64 when the   */
                           /* upsampling is < 1.5 and eps < 1e-4), 1 fp32,     */
                           /* 2 fp64                                           */
} nufft_opts;

typedef struct nufft_plan_info {
    int     type, dim, n_trans, isign;
    int     w, w2;                 /* ES widths: spread kernel, type-3 inner kernel */
    double  beta, beta2;           /* ES shape parameters                            */
    double  eps, upsampfac, sigma_inner;
    int64_t n_modes[3];            /* types 1/2 mode box                             */
    int64_t nf[3];                 /* type-3 spread grid (== n_up for types 1/2)     */
    int64_t n_up[3];               /* FFT grid                                       */
    int64_t M;                     /* nonuniform points (type 3: sources)            */
    int64_t N_tgt;                 /* type-3 targets                                 */
    double  C[3], D[3], gam[3];    /* type-3 centres and scale factors               */
    int     tiled;                 /* 1 if the tiled (bin-sorted) kernels are used   */
    int     bin[3];                /* bin extent per dimension (tiled path)          */
    int64_t nsub, nsub_tgt;        /* subproblems (sources / type-3 targets)         */
    int64_t device_bytes;          /* device memory held by the plan                 */
    int64_t kernel_launches;       /* this library's kernels launched by executes    */
    int64_t fft_execs;             /* cuFFT executions issued by executes            */
    int     fft64;                 /* 1 if the fine-grid FFT runs in fp64            */
    int     fft_own;               /* 1 if this library's own FFT (two-pass 1-D,
                                      or pruned three-pass 3-D; pad / crop fused)
                                      replaces pad + cuFFT (+ crop)                  */
    int64_t grid_cells;            /* cells per stored fine grid: the n_up product,
                                      plus a periodic halo for 3-D type 2 on the
                                      pruned FFT (nufft_get_grid's layout)           */
    int64_t grid_ext[3];           /* stored extents per dimension (n_up + halo)    */
    int     grid_lo[3];            /* index of fine-grid cell 0 per dimension in the
                                      stored extents (halo cells below it)          */
} nufft_plan_info;

/* Fill `opts` with the defaults above. */
void nufft_default_opts(nufft_opts* opts);

/* Create a plan on CUDA device `device`.
 * Replaces: Type1PlanND.__init__ / Type2PlanND.__init__ (mlx_nufft/nd.py:389,861,
 * mode/grid/deconvolution part of _PointsND.__init__ nd.py:97-150),
 * GpuT3Plan.__init__ (mlx_nufft/gpu_t3.py:288) and
 * Plan.__init__ (mlx_nufft/api.py:270).
 * type: 1, 2 or 3.  dim: 1..3.  n_modes: dim entries (types 1/2; ignored for 3).
 * n_trans: number of vectors a single nufft_execute call handles.          */
int nufft_plan_create(int type, int dim, const int64_t* n_modes, int n_trans,
                      double eps, int isign, const nufft_opts* opts, int device,
                      nufft_plan_t* plan);

/* Set nonuniform points (device fp64 arrays; unused ones may be NULL).
 * Types 1/2: M points x, y, z.  Type 3: M sources x, y, z and N targets
 * s, t, u; this call also sizes the type-3 grids from the extents.
 * Folding, cell/fraction split, bin sort and subproblem tables all run on
 * the device; the call synchronises `stream` once (subproblem count).
 * Replaces: _PointsND._compute_cells / _od_prepare (mlx_nufft/nd.py:152-165,
 * 298-372), Type1PlanND.set_sources (nd.py:627), GpuT3Plan.__init__ sizing
 * and target setup (gpu_t3.py:322-441), Plan.setpts (api.py:299).          */
int nufft_setpts(nufft_plan_t plan, int64_t M, const double* x,
                 const double* y, const double* z, int64_t N,
                 const double* s, const double* t, const double* u,
                 void* stream);

/* Type 3 only: re-point the sources against the frozen grids and targets.
 * Returns NUFFT_ERR_RANGE if a source lies outside the sized extent plus the
 * kernel guard band.  Replaces GpuT3Plan.set_sources (mlx_nufft/gpu_t3.py:444-506). */
int nufft_set_sources(nufft_plan_t plan, int64_t M, const double* x,
                      const double* y, const double* z, void* stream);

/* Run the transform on `nvec` vectors (device complex64, contiguous,
 * vector-major).  nvec may exceed n_trans (processed in chunks).
 * Type 1: in = c[nvec][M], out = f[nvec][N0][N1][N2].
 * Type 2: in = f[nvec][N...], out = c[nvec][M] (caller point order).
 * Type 3: in = c[nvec][M], out = f[nvec][N_tgt] (target order).
 * Asynchronous on `stream`; no host synchronisation.  Device-side failures
 * (an interpolation tile copy whose bounded wait ran out: that execute's
 * output is invalid) are recorded in the plan and returned as
 * NUFFT_ERR_CUDA by the plan's next execute / setpts call, or by
 * nufft_plan_check.
 * Replaces: Type1PlanND.execute / execute_batch (mlx_nufft/nd.py:581,744),
 * Type2PlanND.execute (nd.py:1075), GpuT3Plan.execute / execute_batch
 * (mlx_nufft/gpu_t3.py:1287,941), Plan.execute (mlx_nufft/api.py:331).     */
int nufft_execute(nufft_plan_t plan, const void* in, void* out, int nvec,
                  void* stream);

/* Apply the adjoint of the planned transform to `nvec` vectors (device
 * complex64, vector-major): the sibling transform with the opposite sign.
 * Type-1 plan: in = f[nvec][N...] (modes), out = c[nvec][M] (points, caller
 * order).  Type-2 plan: in = c[nvec][M], out = f[nvec][N...].  Type-3 plan:
 * in = f[nvec][N_tgt] (targets), out = c[nvec][M] (sources).  Types 1/2
 * reuse the plan's own sorted points, corrections and fine grids (no
 * second setpts); a type-3 plan builds its sibling plan (targets as
 * sources, opposite sign) on the first call, from device copies of the
 * coordinates it keeps since setpts, which makes that first call
 * synchronise `stream`.  Asynchronous otherwise.
 * Replaces Plan.execute_adjoint (mlx_nufft/api.py:347-388). */
int nufft_execute_adjoint(nufft_plan_t plan, const void* in, void* out,
                          int nvec, void* stream);

/* Types 1 and 2: one stage of nufft_execute on nvec <= n_trans vectors, so
 * a caller can combine the fine grids across GPUs between the stages: sum
 * type-1 grids of ranks that spread disjoint points, or broadcast one
 * type-2 grid to ranks that interpolate disjoint targets.  SPREAD reads
 * `in`, FINISH writes `out`.  No reference counterpart (the reference is
 * single-GPU); it splits Type1PlanND.execute (nd.py:581-625) and
 * Type2PlanND.execute (nd.py:1075-1119). */
int nufft_execute_stage(nufft_plan_t plan, int stage, const void* in,
                        void* out, int nvec, void* stream);

/* Device address and size (elements, all grids the plan holds) of the
 * plan's fine grid, e.g. for a collective between the stages above: type 1
 * the complex64 spreading grid; type 2 the FFT grid, complex128 when the
 * plan runs its FFT in fp64 (nufft_plan_info.fft64), else complex64.  Grids
 * are grid_cells apart in the stored layout of nufft_plan_info (grid_ext,
 * grid_lo: a periodic halo around a 3-D type-2 grid on the pruned FFT).    */
int nufft_get_grid(nufft_plan_t plan, void** grid, int64_t* n_complex);

/* Type 1 only: transform G disjoint subsets of the plan's points
 * (groups[j] in [0, G)) independently.  out = f[G][N...].
 * Replaces Type1PlanND.execute_disjoint (mlx_nufft/nd.py:796-855).          */
int nufft_execute_disjoint(nufft_plan_t plan, const void* c,
                           const int32_t* groups, int ngroups, void* out,
                           void* stream);

/* Release the plan and every device buffer it owns. */
int nufft_plan_destroy(nufft_plan_t plan);

/* Synchronise `stream` and report a device-side failure recorded by the
 * plan's executes so far (NUFFT_ERR_CUDA; the flag is then cleared), else
 * NUFFT_OK.  No reference counterpart (MLX raises at mx.eval). */
int nufft_plan_check(nufft_plan_t plan, void* stream);

int nufft_plan_get_info(nufft_plan_t plan, nufft_plan_info* info);

/* Per-stage device times (ms) of the last execute on a plan created with
 * opts.profile = 1; synchronises on the last recorded event.
 * ms[0..n): spread/pad, fft, interp/crop, total.  Returns the stage count.
 * Replaces GpuT3Plan.execute_profiled (mlx_nufft/gpu_t3.py:1351-1364).     */
int nufft_get_stage_times(nufft_plan_t plan, float* ms, int n);

/* Turn the per-stage event recording of nufft_get_stage_times on (1) or off
 * (0) for later executes.  Same reference counterpart as above. */
int nufft_plan_set_profile(nufft_plan_t plan, int on);

/* Copy the plan's sorted point geometry into caller-owned DEVICE buffers:
 * which = 0 sources/points, 1 type-3 targets; i1 and fr hold dim*count
 * entries (dimension-major), perm holds count entries (sorted position ->
 * caller index).  Test hook for the setpts parity checks
 * (reference gate: harness/test_type1_setsources_gpu.py:48-69).            */
int nufft_debug_points(nufft_plan_t plan, int which, int32_t* i1, float* fr,
                       uint32_t* perm, void* stream);

/* e^{i*isign*phi} with phi = sum of `ncomp` fp64 component arrays (device),
 * n elements, into complex64 `out` (device).  Replaces mlx_nufft.expi
 * (mlx_nufft/dfmath.py:57-134, kernel dfmath.py:29-54).                    */
int nufft_expi(int ncomp, const double* const* comps, int64_t n, int isign,
               void* out, void* stream);

/* ---- interpolation without device allocation ------------------------- */
/* Size of the device scratch array behind nufft_interp_noalloc: 16 MiB,
 * held by every GPU that loads this library until the process exits. */
#define NUFFT_NOALLOC_SCRATCH_BYTES (16u << 20)

/* Type-2 interpolation stage that allocates no device memory.  No
 * counterpart in the reference.  For callers that must not allocate device
 * memory themselves or through this library -- e.g. code running inside a
 * host framework that owns the GPU's memory budget through its own
 * allocator and treats any other allocation as an error, or a latency-
 * critical loop that cannot afford cudaMalloc / cudaFree, which may
 * synchronise the whole device.  Plans allocate at create / setpts; this
 * entry point does not.
 *
 * Computes, on the current CUDA device and asynchronously on `stream`,
 *   out[j] = sum over the w^dim taps of psi(taps) * grid[(i1 + l) mod n]
 * for the M points (x, y, z) (fp64, folded mod 2*pi onto the grid spacing
 * 2*pi / n_grid[d]), with the ES kernel (w, beta) = nufft_kernel_params(eps,
 * upsampfac) evaluated in its exp/sqrt form.  `grid` must be a complex64
 * (interleaved float) fine grid of n_grid[0] x .. x n_grid[dim-1] cells
 * (C order, FFT order) -- e.g. the grid a type-2 plan with the same eps /
 * upsampfac has just transformed (nufft_get_grid), but only when that plan
 * reports nufft_plan_info.fft64 == 0: a plan that runs its FFT in fp64
 * holds a complex128 grid, which this entry point cannot read (the pointer
 * carries no type; it would be misread).  `out` is complex64[M] in caller
 * order.  Each n_grid[d] must be in [2w, 2^31).
 *
 * Scratch: the points' cell indices and fractions (8 bytes per point per
 * dimension) live in one static device array of NUFFT_NOALLOC_SCRATCH_BYTES,
 * so M * dim may not exceed NUFFT_NOALLOC_SCRATCH_BYTES / 8 (2,097,152);
 * larger requests return NUFFT_ERR_ARG.  Every call on a device shares the
 * array and it keeps the last call's contents (each call rewrites all it
 * reads, nothing needs clearing): calls that overlap on the GPU (different
 * streams, or threads without ordering) race and corrupt each other's
 * results -- order them on one stream.  The first call on each device looks
 * up the array's device address (cudaGetSymbolAddress); make that first call
 * before any stream capture.  A point with a non-finite coordinate gets the
 * output NaN + NaN*i (the call itself is asynchronous and cannot return an
 * error for it; plans reject such points at setpts instead). */
int nufft_interp_noalloc(int dim, const int64_t* n_grid, double eps,
                         double upsampfac, const void* grid, int64_t M,
                         const double* x, const double* y, const double* z,
                         void* out, void* stream);

/* ---- host-side numerics (no GPU needed) ------------------------------ */
/* mlx_nufft/sizing.py:28-50 */
int nufft_kernel_params(double eps, double upsampfac, int* w, double* beta);
/* mlx_nufft/sizing.py:13-25 */
int64_t nufft_next235even(int64_t n);
/* mlx_nufft/sizing.py:74-85: out[i] = phihat(xi[i]) (128-node Gauss-Legendre) */
int nufft_kernel_ft(int64_t n, const double* xi, double beta, int w,
                    double* out);
/* mlx_nufft/sizing.py:88-111 */
int nufft_set_nhg_type3(double S, double X, double upsampfac, int w,
                        int64_t* nf, double* h, double* gam);

/* Message of this thread's last error ("" if none); returns its length. */
int nufft_last_error(char* buf, int len);
/* Library version string. */
const char* nufft_version(void);
/* Number of CUDA devices visible (0 without a GPU; never fails). */
int nufft_device_count(void);

#ifdef __cplusplus
}
#endif

#endif /* NUFFT_B200_H */
