// fft1.cu -- two-pass FFT of power-of-two 1-D fine grids, fused with the
// type-2 / type-3 pad and the type-1 crop.
//
// The reference's 1-D execute is pad (or crop) + one FFT of the n_up-cell
// fine grid (mlx_nufft/nd.py:878-906 and 416-435 around the FFT call).  For
// n = N1 x N2 (powers of two, 2^12 <= n <= 2^22) the FFT here is the
// four-step decomposition
//
//   X[k1 + N1 k2] = sum_{n2} W_N2^{n2 k2} W_n^{n2 k1} sum_{n1} W_N1^{n1 k1} x[n1 N2 + n2]
//
// in two kernels, each a batch of shared-memory FFTs over C adjacent
// columns (C = 8 up to length 1024, else 4: every global access moves
// 32- or 64-byte segments):
//   pass 1: columns n2 of length N1.  Its loads ARE the pad: cell r of the
//           fine grid is mode m = (r >= n - N/2 ? r - n : r) + N/2 times the
//           correction dec[m] when 0 <= m < N, else zero (no zero is read
//           or written); the inter-pass twiddle W_n^{k1 n2} is applied on
//           the store to a scratch grid A[k1][n2].
//   pass 2: rows k1 of A (length N2), stored in natural order X (type 2 /
//           type 3), or -- type 1 -- only the in-band cells, times dec, in
//           mode order (the crop).
// cuFFT's own transform of such a grid is also two passes, plus a separate
// pad kernel that writes (and the FFT then reads) the whole zero-padded grid.
//
// Inside a CTA a length-L FFT is a Stockham sequence of radix-32/16/8
// stages (log2 L split as evenly as possible over ceil(log2 L / 5) stages:
// 1024 = 32 x 32, 2048 = 16 x 16 x 8).  The first stage loads its inputs
// from global memory straight into registers and the last stores its
// outputs straight to global memory; between stages each thread's R-point
// DFTs run in registers and exchange through shared memory, whose
// addresses a are padded to a + a/16 so that the strided stage stores stay
// free of bank conflicts.
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdlib>
#include <mutex>
#include <set>
#include <type_traits>
#include <vector>

#include "internal.h"

namespace nufft {
namespace {

// Threads per CTA and the largest in-register radix.
#ifndef NUFFT_FFT_THREADS
#define NUFFT_FFT_THREADS 256
#endif
#ifndef NUFFT_FFT_RMAX_LOG2
#define NUFFT_FFT_RMAX_LOG2 5
#endif
constexpr int kFftThreads = NUFFT_FFT_THREADS;

// Columns per CTA at length 2048, and resident CTAs per SM the kernels are
// compiled for (caps their registers at 128; measured on 2^21 cells: pass 1
// 18.4 us vs 21.1 uncapped, 2 rows per CTA at length 2048 slower).
#ifndef NUFFT_FFT_COLS_2048
#define NUFFT_FFT_COLS_2048 4
#endif
#ifndef NUFFT_FFT_MINB_COLS
#define NUFFT_FFT_MINB_COLS 2
#endif
#ifndef NUFFT_FFT_MINB_ROWS
#define NUFFT_FFT_MINB_ROWS 2
#endif

__host__ __device__ constexpr int ilog2(int x) {
    int k = 0;
    while ((1 << k) < x) ++k;
    return k;
}

// Columns (pass 1) / rows (pass 2) per CTA.
__host__ __device__ constexpr int fft_cols(int L) {
    return L <= 1024 ? 8 : NUFFT_FFT_COLS_2048;
}

// Radix of the stage that starts at span NS (see the file comment).
__host__ __device__ constexpr int stage_radix(int L, int NS) {
    constexpr int rb = NUFFT_FFT_RMAX_LOG2;
    const int k = ilog2(L), st = (k + rb - 1) / rb;
    const int done = ilog2(NS);
    int t = 0, acc = 0;
    while (acc < done) {
        acc += k / st + (t < k % st ? 1 : 0);
        ++t;
    }
    return 1 << (k / st + (t < k % st ? 1 : 0));
}

__device__ __forceinline__ int fpad(int a) { return a + (a >> 4); }

__host__ __device__ constexpr int fft_data_cells(int L) {
    return (L * fft_cols(L)) + ((L * fft_cols(L)) >> 4);
}

// Wait for the kernel this one was launched after (programmatic dependent
// launch; a no-op for a normal launch).
__device__ __forceinline__ void grid_dep_sync() {
    asm volatile("griddepcontrol.wait;" ::: "memory");
}

__device__ __forceinline__ float2 cmulf(float2 a, float2 b) {
    return make_float2(a.x * b.x - a.y * b.y, a.x * b.y + a.y * b.x);
}

// x * W_32^m, W_32 = exp(-2 pi i / 32) (INV: its conjugate); m in 0..15,
// a compile-time constant once the register DFT is unrolled.
template <bool INV>
__device__ __forceinline__ float2 rot32(float2 x, int m) {
    constexpr float a1 = 0.98078528040323044f;   // cos(pi / 16)
    constexpr float b1 = 0.19509032201612827f;   // sin(pi / 16)
    constexpr float a2 = 0.92387953251128674f;   // cos(pi / 8)
    constexpr float b2 = 0.38268343236508977f;   // sin(pi / 8)
    constexpr float a3 = 0.83146961230254524f;   // cos(3 pi / 16)
    constexpr float b3 = 0.55557023301960218f;   // sin(3 pi / 16)
    constexpr float h = 0.70710678118654752f;    // cos(pi / 4)
    float c, s;                                  // W_32^m = c - i s
    switch (m) {
        case 0: return x;
        case 8: return INV ? make_float2(-x.y, x.x) : make_float2(x.y, -x.x);
        case 1: c = a1; s = b1; break;
        case 2: c = a2; s = b2; break;
        case 3: c = a3; s = b3; break;
        case 4: c = h; s = h; break;
        case 5: c = b3; s = a3; break;
        case 6: c = b2; s = a2; break;
        case 7: c = b1; s = a1; break;
        case 9: c = -b1; s = a1; break;
        case 10: c = -b2; s = a2; break;
        case 11: c = -b3; s = a3; break;
        case 12: c = -h; s = h; break;
        case 13: c = -a3; s = b3; break;
        case 14: c = -a2; s = b2; break;
        default: c = -a1; s = b1; break;         // 15
    }
    return INV ? make_float2(x.x * c - x.y * s, x.y * c + x.x * s)
               : make_float2(x.x * c + x.y * s, x.y * c - x.x * s);
}

template <int R>
__host__ __device__ constexpr int bit_reverse(int i) {
    int r = 0;
    for (int b = 1; b < R; b <<= 1) {
        r = (r << 1) | (i & 1);
        i >>= 1;
    }
    return r;
}

// In-register R-point DFT (R = 2 .. 32), radix-2 decimation in time.
template <int R, bool INV>
__device__ __forceinline__ void dft_reg(float2 (&v)[R]) {
#pragma unroll
    for (int i = 0; i < R; ++i) {
        const int j = bit_reverse<R>(i);
        if (j > i) {
            const float2 t = v[i];
            v[i] = v[j];
            v[j] = t;
        }
    }
#pragma unroll
    for (int h = 1; h < R; h <<= 1) {
#pragma unroll
        for (int s = 0; s < R; s += 2 * h) {
#pragma unroll
            for (int k = 0; k < h; ++k) {
                const float2 a = v[s + k];
                const float2 b = rot32<INV>(v[s + k + h], k * (16 / h));  // W_2h^k
                v[s + k] = make_float2(a.x + b.x, a.y + b.y);
                v[s + k + h] = make_float2(a.x - b.x, a.y - b.y);
            }
        }
    }
}

// Stockham stages NS, NS*R, ... of a length-L FFT over the CTA's C columns
// (fft_stages: C = fft_cols(L)).  SMEM_IO: the input is already in s (the
// inter-stage layout) and the output is left there in natural order (the
// caller loads and stores coalesced rows around the call).  The first stage takes its inputs from load(c, i)
// (row i of column c); the last hands each butterfly's outputs to
// store(c, base, stride, v): v[r] is row base + r * stride of column c.
// In between, element (i, c) lives at s[fpad(i * C + c)].  twL[m] = W_L^m
// (global, read through L1).
template <int L, int NS, bool INV, int C, bool SMEM_IO = false, class Load, class Store>
__device__ __forceinline__ void fft_stages_c(float2* s, const float2* __restrict__ twL,
                                             const Load& load, const Store& store) {
    if constexpr (NS < L) {
        constexpr int R = stage_radix(L, NS);
        constexpr bool LAST = NS * R == L;
        constexpr int NB = (L / R) * C;                 // butterflies
        constexpr int PER = (NB + kFftThreads - 1) / kFftThreads;
        float2 v[PER][R];
#pragma unroll
        for (int t = 0; t < PER; ++t) {
            const int bid = threadIdx.x + t * kFftThreads;
            if (NB % kFftThreads == 0 || bid < NB) {
                const int c = bid % C, j = bid / C;
#pragma unroll
                for (int r = 0; r < R; ++r)
                    v[t][r] = (NS == 1 && !SMEM_IO) ? load(c, j + r * (L / R))
                                                    : s[fpad((j + r * (L / R)) * C + c)];
                if (NS > 1) {
                    const int k = j % NS;
#pragma unroll
                    for (int r = 1; r < R; ++r) {
                        float2 w = __ldg(twL + r * k * (L / (NS * R)));
                        if (INV) w.y = -w.y;
                        v[t][r] = cmulf(v[t][r], w);
                    }
                }
                dft_reg<R, INV>(v[t]);
            }
        }
        if constexpr (LAST) {
            if (SMEM_IO) __syncthreads();              // all reads of s done
#pragma unroll
            for (int t = 0; t < PER; ++t) {
                const int bid = threadIdx.x + t * kFftThreads;
                if (NB % kFftThreads == 0 || bid < NB) {
                    const int c = bid % C, j = bid / C;
                    const int base = (j / NS) * NS * R + (j % NS);
                    if constexpr (SMEM_IO) {
#pragma unroll
                        for (int r = 0; r < R; ++r)
                            s[fpad((base + r * NS) * C + c)] = v[t][r];
                    } else {
                        store(c, base, NS, v[t]);
                    }
                }
            }
        } else {
            if (NS > 1 || SMEM_IO) __syncthreads();    // all reads of s done
#pragma unroll
            for (int t = 0; t < PER; ++t) {
                const int bid = threadIdx.x + t * kFftThreads;
                if (NB % kFftThreads == 0 || bid < NB) {
                    const int c = bid % C, j = bid / C;
                    const int base = (j / NS) * NS * R + (j % NS);
#pragma unroll
                    for (int r = 0; r < R; ++r)
                        s[fpad((base + r * NS) * C + c)] = v[t][r];
                }
            }
            __syncthreads();
            fft_stages_c<L, NS * R, INV, C, SMEM_IO>(s, twL, load, store);
        }
    }
}

template <int L, int NS, bool INV, class Load, class Store>
__device__ __forceinline__ void fft_stages(float2* s, const float2* __restrict__ twL,
                                           const Load& load, const Store& store) {
    fft_stages_c<L, NS, INV, fft_cols(L)>(s, twL, load, store);
}

// Inter-pass twiddles are taken exactly from the tables every kTwExact
// rows and by complex multiplication by the row step in between (at most
// kTwExact - 1 products, a few fp32 ulps).
constexpr int kTwExact = 4;

// Pass 1: columns c0 .. c0 + C - 1 of the fine grid (length L = N1), read
// either as padded modes (PAD: in = modes of box N with correction dec)
// or as a plain grid; A[k1 * N2 + n2] = W_n^{k1 n2} * column FFT.
// twL = W_N1 table, twn[e] = W_n^e for e < N2; N2 = 1 << lg2.
template <int L, bool INV, bool PAD>
__global__ void __launch_bounds__(kFftThreads, NUFFT_FFT_MINB_COLS)
k_fft1_cols(const float2* __restrict__ in, int64_t in_stride, int64_t N,
            const float* __restrict__ dec, int n, int lg2,
            const float2* __restrict__ twL, const float2* __restrict__ twn,
            float2* __restrict__ A) {
    constexpr int C = fft_cols(L);
    extern __shared__ float2 s[];
    const int v = blockIdx.y;
    const int c0 = blockIdx.x * C;
    in += v * in_stride;
    A += (int64_t)v * n;
    const int64_t lo = n - N / 2;                 // first negative-mode cell
    const int64_t half = N / 2;
    const uint32_t emask = (uint32_t)(n - 1), lmask = (1u << lg2) - 1u;
    auto load = [&](int c, int i) {
        const int64_t cell = ((int64_t)i << lg2) + c0 + c;
        float2 x = make_float2(0.0f, 0.0f);
        if (PAD) {
            const int64_t m = (cell >= lo ? cell - n : cell) + half;
            if (m >= 0 && m < N) {
                const float d = __ldg(dec + m);
                const float2 g = __ldg(in + m);
                x = make_float2(g.x * d, g.y * d);
            }
        } else {
            x = __ldg(in + cell);
        }
        return x;
    };
    // W_n^e from the tables: e = eh * N2 + el, W_n^{eh N2} = W_L^{eh}
    auto wn = [&](uint32_t e) {
        e &= emask;
        float2 w = cmulf(__ldg(twL + (e >> lg2)), __ldg(twn + (e & lmask)));
        if (INV) w.y = -w.y;
        return w;
    };
    auto store = [&](int c, int base, int stride, auto& vals) {
        constexpr int R = std::extent<std::remove_reference_t<decltype(vals)>>::value;
        const uint32_t n2 = (uint32_t)(c0 + c);
        const float2 step = wn((uint32_t)stride * n2);
        float2 w = make_float2(1.0f, 0.0f);
#pragma unroll
        for (int r = 0; r < R; ++r) {
            const int k1 = base + r * stride;
            w = (r % kTwExact == 0) ? wn((uint32_t)k1 * n2) : cmulf(w, step);
            A[((int64_t)k1 << lg2) + n2] = cmulf(vals[r], w);
        }
    };
    fft_stages<L, 1, INV>(s, twL, load, store);
}

// Pass 2: rows r0 .. r0 + C - 1 of A (length L = N2).  CROP: fk[m] =
// X[k] * dec[m] for the in-band cells k (mode m as in pass 1), else X[k]
// (natural order).
template <int L, bool INV, bool CROP>
__global__ void __launch_bounds__(kFftThreads, NUFFT_FFT_MINB_ROWS)
k_fft1_rows(const float2* __restrict__ A, int N1, int n,
            const float2* __restrict__ twL, float2* __restrict__ out,
            int64_t out_stride, int64_t N, const float* __restrict__ dec) {
    constexpr int C = fft_cols(L);
    extern __shared__ float2 s[];
    asm volatile("griddepcontrol.wait;" ::: "memory");   // pass 1 has completed
    const int v = blockIdx.y;
    const int r0 = blockIdx.x * C;
    A += (int64_t)v * n;
    out += v * out_stride;
    const int64_t lo = n - N / 2;
    const int64_t half = N / 2;
    auto load = [&](int c, int j) {
        return __ldg(A + (int64_t)(r0 + c) * L + j);
    };
    auto store = [&](int c, int base, int stride, auto& vals) {
        constexpr int R = std::extent<std::remove_reference_t<decltype(vals)>>::value;
#pragma unroll
        for (int r = 0; r < R; ++r) {
            const int64_t k = (int64_t)(r0 + c) + (int64_t)N1 * (base + r * stride);
            const float2 x = vals[r];
            if (CROP) {
                const int64_t m = (k >= lo ? k - n : k) + half;
                if (m >= 0 && m < N) {
                    const float d = __ldg(dec + m);
                    out[m] = make_float2(x.x * d, x.y * d);
                }
            } else {
                out[k] = x;
            }
        }
    };
    fft_stages<L, 1, INV>(s, twL, load, store);
}

template <int L>
size_t fft_smem() {
    return sizeof(float2) * (size_t)fft_data_cells(L);
}

// Compile-time dispatch over the supported lengths 64..2048.
#define NUFFT_FFT_LEN_SWITCH(len, ...)                                 \
    switch (len) {                                                     \
        case 64: { constexpr int L = 64; __VA_ARGS__; } break;         \
        case 128: { constexpr int L = 128; __VA_ARGS__; } break;       \
        case 256: { constexpr int L = 256; __VA_ARGS__; } break;       \
        case 512: { constexpr int L = 512; __VA_ARGS__; } break;       \
        case 1024: { constexpr int L = 1024; __VA_ARGS__; } break;     \
        case 2048: { constexpr int L = 2048; __VA_ARGS__; } break;     \
        default: fail(-1, "fft1: unsupported length");                  \
    }

// Dynamic shared memory opt-in, and the largest shared-memory carveout so
// that as many CTAs as the registers allow stay resident (once per kernel).
void prepare(const void* kernel, size_t smem) {
    ensure_smem(kernel, smem);
    static std::mutex mu;
    static std::set<const void*> done;
    std::lock_guard<std::mutex> lk(mu);
    if (done.insert(kernel).second)
        NUFFT_CUDA(cudaFuncSetAttribute(
            kernel, cudaFuncAttributePreferredSharedMemoryCarveout,
            (int)cudaSharedmemCarveoutMaxShared));
}

// pass 1 for nv vectors
void run_cols(const Fft1& f, const float2* in, int64_t in_stride, int64_t N,
              const float* dec, bool pad, bool inv, float2* A, int nv,
              cudaStream_t st) {
    NUFFT_FFT_LEN_SWITCH(f.N1, {
        const size_t smem = fft_smem<L>();
        dim3 g((unsigned)(f.N2 / fft_cols(L)), (unsigned)nv);
        auto launch = [&](auto k) {
            prepare((const void*)k, smem);
            k<<<g, kFftThreads, smem, st>>>(in, in_stride, N, dec, f.n, ilog2(f.N2),
                                            f.tw, f.tw + f.N1 + f.N2, A);
        };
        if (pad)
            inv ? launch(k_fft1_cols<L, true, true>) : launch(k_fft1_cols<L, false, true>);
        else
            inv ? launch(k_fft1_cols<L, true, false>) : launch(k_fft1_cols<L, false, false>);
    });
    NUFFT_LAUNCH("k_fft1_cols");
}

// pass 2 for nv vectors
void run_rows(const Fft1& f, const float2* A, bool crop, bool inv, float2* out,
              int64_t out_stride, int64_t N, const float* dec, int nv,
              cudaStream_t st) {
    NUFFT_FFT_LEN_SWITCH(f.N2, {
        const size_t smem = fft_smem<L>();
        dim3 g((unsigned)(f.N1 / fft_cols(L)), (unsigned)nv);
        auto launch = [&](auto k) {
            prepare((const void*)k, smem);
            launch_dependent(k, g, dim3(kFftThreads), smem, st, A, f.N1, f.n,
                             (const float2*)(f.tw + f.N1), out, out_stride, N, dec);
        };
        if (crop)
            inv ? launch(k_fft1_rows<L, true, true>) : launch(k_fft1_rows<L, false, true>);
        else
            inv ? launch(k_fft1_rows<L, true, false>) : launch(k_fft1_rows<L, false, false>);
    });
    NUFFT_LAUNCH("k_fft1_rows");
}

// ---------------------------------------------------------------------
// 3-D power-of-two fine grids: the FFT pruned to the mode box, with the
// pad (types 2) or the crop (type 1) fused.
//
// A type-2 grid is the FFT of the padded modes, nonzero on an N0 x N1 x N2
// box of the n0 x n1 x n2 cells.  Transforming axis by axis from the
// innermost one, the first pass needs only the N0 N1 rows that hold modes
// and the second only the N0 planes: three batches of column FFTs
//   Z: f[m0][m1][.] (x dec) -> A[m0][m1][z]     N0 N1 rows of length n2
//   Y: A[m0][.][z]          -> B[m0][y][z]      N0 n2 columns of length n1
//   X: B[.][y][z]           -> G[x][y][z]       n1 n2 columns of length n0
// whose loads read only in-band entries (the zeros of the padded grid are
// never read or written) and whose stores write the next pass's layout.
// Pass by pass the DRAM traffic is 8 (N0 N1 N2 + N0 N1 n2 | N0 N1 n2 +
// N0 n1 n2 | N0 n1 n2 + n0 n1 n2) bytes, 2.8 GB for 256^3 modes on 512^3
// cells against ~9.7 GB for a pad kernel plus a full three-pass FFT.  A
// type-1 grid runs the mirror image (X, Y, Z passes keeping only in-band
// outputs, the deconvolution applied by the last store).  A lives in the
// fine grid's own memory (type 2: free until pass X writes it; type 1:
// dead once pass X has read it) and B in a plan-owned scratch grid.
// Columns of the Y and X passes are C adjacent z-cells, so every access is
// a contiguous C x 8-byte segment.

// Columns per CTA of the 3-D passes: 16 up to length 512 (every load and
// store of the Y / X passes a 128-byte row segment, and every thread busy
// in the first stage), as the 1-D passes above that.
__host__ __device__ constexpr int fftn_cols(int L) {
    return L <= 512 ? 16 : fft_cols(L);
}

template <int L>
size_t fftn_smem() {
    constexpr int cells = L * fftn_cols(L) + ((L * fftn_cols(L)) >> 4);
    return sizeof(float2) * (size_t)cells;
}

// Resident CTAs per SM the 3-D passes are compiled for (caps registers at
// 85; measured 0.85 vs 1.00 ms for the pad passes of a 512^3 grid at 2).
#ifndef NUFFT_FFTN_MINB
#define NUFFT_FFTN_MINB 3
#endif

__device__ __forceinline__ int band_mode(int i, int n, int N) {
    // mode index m (0..N-1) of fine cell i, or -1 outside the mode box
    const int m = (i >= n - N / 2 ? i - n : i) + N / 2;
    return (m >= 0 && m < N) ? m : -1;
}

template <class V>
__device__ __forceinline__ constexpr int vals_len() {
    return std::extent<std::remove_reference_t<V>>::value;
}

// pass Z of the pad: rows r = m0 * N1 + m1 of the mode box.  The CTA's C
// rows are contiguous in both the modes and A, so they move through shared
// memory: coalesced loads of the in-band modes (times the corrections)
// into the transform's layout, the FFT in place, coalesced stores of whole
// rows.
template <int L, bool INV>
__global__ void __launch_bounds__(kFftThreads, NUFFT_FFTN_MINB)
k_fftn_pad_z(const float2* __restrict__ f, int64_t f_vs, const float* __restrict__ d0,
             const float* __restrict__ d1, const float* __restrict__ d2, int N1,
             int N2, int nrows, const float2* __restrict__ twL,
             float2* __restrict__ A, int64_t A_vs) {
    constexpr int C = fftn_cols(L);
    extern __shared__ float2 s[];
    __shared__ float s_d01[C];                   // row corrections d0 * d1
    const int r0 = blockIdx.x * C;
    const int rows = min(C, nrows - r0);
    f += blockIdx.y * f_vs + (int64_t)r0 * N2;
    A += blockIdx.y * A_vs + (int64_t)r0 * L;
    if (threadIdx.x < rows) {
        const int r = r0 + threadIdx.x;
        s_d01[threadIdx.x] = __ldg(d0 + r / N1) * __ldg(d1 + r % N1);
    }
    __syncthreads();
    // thread t loads mode m = t (+ multiples of the block) of every row, K
    // rows in flight before their shared stores; mode m = k + N2/2 sits at
    // fine cell k mod L
    constexpr int K = 8;
    for (int m = threadIdx.x; m < N2; m += kFftThreads) {
        const float dm = __ldg(d2 + m);
        const int cell = ((m - N2 / 2 + L) % L) * C;
        for (int c0 = 0; c0 < C; c0 += K) {
            float2 x[K];
#pragma unroll
            for (int k = 0; k < K; ++k) {
                const int c = c0 + k;
                x[k] = make_float2(0.0f, 0.0f);
                if (c < rows) {
                    const float d = s_d01[c] * dm;
                    const float2 g = __ldg(f + (int64_t)c * N2 + m);
                    x[k] = make_float2(g.x * d, g.y * d);
                }
            }
#pragma unroll
            for (int k = 0; k < K; ++k) s[fpad(cell + c0 + k)] = x[k];
        }
    }
    for (int q = threadIdx.x; q < C * (L - N2); q += kFftThreads) {
        const int c = q % C, i = N2 - N2 / 2 + q / C;     // out-of-band fine cells
        s[fpad(i * C + c)] = make_float2(0.0f, 0.0f);
    }
    __syncthreads();
    auto none = [](int, int) { return make_float2(0.0f, 0.0f); };
    auto nost = [](int, int, int, auto&) {};
    fft_stages_c<L, 1, INV, C, true>(s, twL, none, nost);
    __syncthreads();
    for (int q = threadIdx.x; q < rows * L; q += kFftThreads) {
        const int c = q / L, i = q - c * L;
        A[q] = s[fpad(i * C + c)];
    }
}

// pass Y of the pad: columns (m0, z0 + c); blockIdx.y = m0
template <int L, bool INV>
__global__ void __launch_bounds__(kFftThreads, NUFFT_FFTN_MINB)
k_fftn_pad_y(const float2* __restrict__ A, int64_t A_vs, int N1, int n2,
             const float2* __restrict__ twL, float2* __restrict__ B, int64_t B_vs) {
    constexpr int C = fftn_cols(L);
    extern __shared__ float2 s[];
    grid_dep_sync();
    const int z0 = blockIdx.x * C;
    const int64_t m0 = blockIdx.y;
    A += blockIdx.z * A_vs;
    B += blockIdx.z * B_vs;
    auto load = [&](int c, int i) {
        const int m = band_mode(i, L, N1);
        return m >= 0 ? __ldg(A + (m0 * N1 + m) * n2 + z0 + c) : make_float2(0.0f, 0.0f);
    };
    auto store = [&](int c, int base, int stride, auto& vals) {
#pragma unroll
        for (int k = 0; k < vals_len<decltype(vals)>(); ++k)
            B[(m0 * L + base + k * stride) * n2 + z0 + c] = vals[k];
    };
    fft_stages_c<L, 1, INV, C>(s, twL, load, store);
}

// pass X of the pad: columns (y, z0 + c); blockIdx.y = y.  HALO: the grid
// is stored with the periodic halo h (GridHalo); this pass writes the
// interior, k_halo_fill the halo copies.
template <int L, bool INV, bool HALO, bool PRUNE>
__global__ void __launch_bounds__(kFftThreads, NUFFT_FFTN_MINB)
k_fftn_pad_x(const float2* __restrict__ B, int64_t B_vs, int N0, int n1, int n2,
             const float2* __restrict__ twL, float2* __restrict__ G, int64_t G_vs,
             GridHalo h, const uint8_t* __restrict__ need) {
    constexpr int C = fftn_cols(L);
    extern __shared__ float2 s[];
    grid_dep_sync();
    const int z0 = blockIdx.x * C;
    const int64_t y = blockIdx.y;
    B += blockIdx.z * B_vs;
    G += blockIdx.z * G_vs;
    auto load = [&](int c, int i) {
        const int m = band_mode(i, L, N0);
        return m >= 0 ? __ldg(B + ((int64_t)m * n1 + y) * n2 + z0 + c)
                      : make_float2(0.0f, 0.0f);
    };
    auto store = [&](int c, int base, int stride, auto& vals) {
        if constexpr (!HALO) {
#pragma unroll
            for (int k = 0; k < vals_len<decltype(vals)>(); ++k)
                G[((int64_t)(base + k * stride) * n1 + y) * n2 + z0 + c] = vals[k];
        } else {
            const int64_t PP = (int64_t)h.P[1] * h.P[2];
            const int64_t yz = (y + h.lo[1]) * h.P[2] + h.lo[2] + z0 + c;
#pragma unroll
            for (int k = 0; k < vals_len<decltype(vals)>(); ++k) {
                const int xs = base + k * stride + h.lo[0];
                if (!PRUNE || __ldg(need + xs)) G[(int64_t)xs * PP + yz] = vals[k];
            }
        }
    };
    fft_stages_c<L, 1, INV, C>(s, twL, load, store);
}

// Periodic halo of nv stored grids (GridHalo h) copied from their
// interior, one dimension per launch: pass 2 (contiguous dimension) over the
// interior rows, pass 1 whole rows (their pass-2 halo included) over the
// interior planes, pass 0 whole planes.  Each halo cell at stored index i'
// takes the cell one period away (i' + n below the grid, i' - n above it),
// which lies in the interior since lo, hi <= n.  need (optional): only the
// stored planes of dimension 0 with need[s] != 0 (whose interior
// counterparts are marked too).
__global__ void __launch_bounds__(256)
k_halo_fill(float2* __restrict__ G, int64_t G_vs, GridHalo h, int n0, int n1, int n2,
            int pass, const uint8_t* __restrict__ need) {
    const int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
    G += blockIdx.y * G_vs;
    const int64_t P2 = h.P[2], PP = (int64_t)h.P[1] * h.P[2];
    auto src = [](int k, int lo, int n, int& dst) {
        dst = k < lo ? k : n + k;            // k: index among the halo cells
        return k < lo ? dst + n : dst - n;
    };
    if (pass == 2) {
        const int hz = h.lo[2] + h.hi[2];
        if (i >= (int64_t)n0 * n1 * hz) return;
        const int64_t r = i / hz;
        const int k = (int)(i - r * hz);
        const int x = (int)(r / n1), y = (int)(r - (int64_t)x * n1);
        if (need && !need[x + h.lo[0]]) return;
        int zd;
        const int zs = src(k, h.lo[2], n2, zd);
        float2* row = G + (int64_t)(x + h.lo[0]) * PP + (int64_t)(y + h.lo[1]) * P2;
        row[zd] = row[zs];
    } else if (pass == 1) {
        const int hy = h.lo[1] + h.hi[1];
        if (i >= (int64_t)n0 * hy * P2) return;
        const int64_t r = i / P2;
        const int64_t z = i - r * P2;
        const int x = (int)(r / hy), k = (int)(r - (int64_t)x * hy);
        if (need && !need[x + h.lo[0]]) return;
        int yd;
        const int ys = src(k, h.lo[1], n1, yd);
        float2* pl = G + (int64_t)(x + h.lo[0]) * PP;
        pl[yd * P2 + z] = pl[ys * P2 + z];
    } else {
        const int hx = h.lo[0] + h.hi[0];
        if (i >= (int64_t)hx * PP) return;
        const int k = (int)(i / PP);
        const int64_t q = i - (int64_t)k * PP;
        int xd;
        const int xs = src(k, h.lo[0], n0, xd);
        if (need && !need[xd]) return;
        G[xd * PP + q] = G[xs * PP + q];
    }
}

// ---------------------------------------------------------------------
// Slab order of the pad, for a plan whose points read only some planes of
// dimension 0 (one x-slab of the points per GPU): the X pass first, over
// the N1 x N2 mode columns, keeping only the nx needed planes (xmap[x]:
// compact index of fine plane x, or -1); then Y and Z over those planes
// only.  The Z pass writes the interior of the halo-padded grid (plane
// xlist[xi] at stored index xlist[xi] + lo[0]); k_halo_fill adds the
// copies.  T1 [nx][N1][N2] and T2 [nx][n1][N2] are the scratch planes.

// pass X: columns (m1, z0 + c) of the mode box; blockIdx.y = m1
template <int L, bool INV>
__global__ void __launch_bounds__(kFftThreads, NUFFT_FFTN_MINB)
k_fftn_slab_x(const float2* __restrict__ f, int64_t f_vs, const float* __restrict__ d0,
              const float* __restrict__ d1, const float* __restrict__ d2, int N0, int N1,
              int N2, const int* __restrict__ xmap, const float2* __restrict__ twL,
              float2* __restrict__ T1, int64_t T1_vs) {
    constexpr int C = fftn_cols(L);
    extern __shared__ float2 s[];
    const int z0 = blockIdx.x * C;
    const int m1 = blockIdx.y;
    f += blockIdx.z * f_vs;
    T1 += blockIdx.z * T1_vs;
    const float dm1 = __ldg(d1 + m1);
    auto load = [&](int c, int i) {
        const int m = band_mode(i, L, N0), m2 = z0 + c;
        if (m < 0 || m2 >= N2) return make_float2(0.0f, 0.0f);
        const float d = __ldg(d0 + m) * dm1 * __ldg(d2 + m2);
        const float2 g = __ldg(f + ((int64_t)m * N1 + m1) * N2 + m2);
        return make_float2(g.x * d, g.y * d);
    };
    auto store = [&](int c, int base, int stride, auto& vals) {
        const int m2 = z0 + c;
        if (m2 >= N2) return;
#pragma unroll
        for (int k = 0; k < vals_len<decltype(vals)>(); ++k) {
            const int xi = __ldg(xmap + base + k * stride);
            if (xi >= 0) T1[((int64_t)xi * N1 + m1) * N2 + m2] = vals[k];
        }
    };
    fft_stages_c<L, 1, INV, C>(s, twL, load, store);
}

// pass Y: columns (xi, z0 + c); blockIdx.y = xi
template <int L, bool INV>
__global__ void __launch_bounds__(kFftThreads, NUFFT_FFTN_MINB)
k_fftn_slab_y(const float2* __restrict__ T1, int64_t T1_vs, int N1, int N2,
              const float2* __restrict__ twL, float2* __restrict__ T2, int64_t T2_vs) {
    constexpr int C = fftn_cols(L);
    extern __shared__ float2 s[];
    grid_dep_sync();
    const int z0 = blockIdx.x * C;
    const int64_t xi = blockIdx.y;
    T1 += blockIdx.z * T1_vs;
    T2 += blockIdx.z * T2_vs;
    auto load = [&](int c, int i) {
        const int m = band_mode(i, L, N1), m2 = z0 + c;
        return (m >= 0 && m2 < N2) ? __ldg(T1 + (xi * N1 + m) * N2 + m2)
                                   : make_float2(0.0f, 0.0f);
    };
    auto store = [&](int c, int base, int stride, auto& vals) {
        const int m2 = z0 + c;
        if (m2 >= N2) return;
#pragma unroll
        for (int k = 0; k < vals_len<decltype(vals)>(); ++k)
            T2[(xi * L + base + k * stride) * N2 + m2] = vals[k];
    };
    fft_stages_c<L, 1, INV, C>(s, twL, load, store);
}

// pass Z: rows r = xi * n1 + y of T2 (N2 modes each, contiguous), padded to
// L = n2, written as whole rows of the stored grid
template <int L, bool INV>
__global__ void __launch_bounds__(kFftThreads, NUFFT_FFTN_MINB)
k_fftn_slab_z(const float2* __restrict__ T2, int64_t T2_vs, int N2, int nrows, int n1,
              const int* __restrict__ xlist, GridHalo h, const float2* __restrict__ twL,
              float2* __restrict__ G, int64_t G_vs) {
    constexpr int C = fftn_cols(L);
    extern __shared__ float2 s[];
    __shared__ int64_t s_row[C];                 // stored-grid offset of each row
    grid_dep_sync();
    const int r0 = blockIdx.x * C;
    const int rows = min(C, nrows - r0);
    T2 += blockIdx.z * T2_vs + (int64_t)r0 * N2;
    G += blockIdx.z * G_vs;
    if (threadIdx.x < rows) {
        const int r = r0 + threadIdx.x;
        const int xi = r / n1, y = r - xi * n1;
        s_row[threadIdx.x] = ((int64_t)(__ldg(xlist + xi) + h.lo[0]) * h.P[1] + y + h.lo[1]) *
                                 h.P[2] + h.lo[2];
    }
    constexpr int K = 8;
    for (int m = threadIdx.x; m < N2; m += kFftThreads) {
        const int cell = ((m - N2 / 2 + L) % L) * C;
        for (int c0 = 0; c0 < C; c0 += K) {
            float2 x[K];
#pragma unroll
            for (int k = 0; k < K; ++k)
                x[k] = c0 + k < rows ? __ldg(T2 + (int64_t)(c0 + k) * N2 + m)
                                     : make_float2(0.0f, 0.0f);
#pragma unroll
            for (int k = 0; k < K; ++k) s[fpad(cell + c0 + k)] = x[k];
        }
    }
    for (int q = threadIdx.x; q < C * (L - N2); q += kFftThreads) {
        const int c = q % C, i = N2 - N2 / 2 + q / C;     // out-of-band fine cells
        s[fpad(i * C + c)] = make_float2(0.0f, 0.0f);
    }
    __syncthreads();
    auto none = [](int, int) { return make_float2(0.0f, 0.0f); };
    auto nost = [](int, int, int, auto&) {};
    fft_stages_c<L, 1, INV, C, true>(s, twL, none, nost);
    __syncthreads();
    for (int q = threadIdx.x; q < rows * L; q += kFftThreads) {
        const int c = q / L, i = q - c * L;
        G[s_row[c] + i] = s[fpad(i * C + c)];
    }
}

// pass X of the crop: columns (y, z0 + c) of the full grid, in-band x only
template <int L, bool INV>
__global__ void __launch_bounds__(kFftThreads, NUFFT_FFTN_MINB)
k_fftn_crop_x(const float2* __restrict__ G, int64_t G_vs, int N0, int n1, int n2,
              const float2* __restrict__ twL, float2* __restrict__ B, int64_t B_vs) {
    constexpr int C = fftn_cols(L);
    extern __shared__ float2 s[];
    const int z0 = blockIdx.x * C;
    const int64_t y = blockIdx.y;
    G += blockIdx.z * G_vs;
    B += blockIdx.z * B_vs;
    auto load = [&](int c, int i) {
        return __ldg(G + ((int64_t)i * n1 + y) * n2 + z0 + c);
    };
    auto store = [&](int c, int base, int stride, auto& vals) {
#pragma unroll
        for (int k = 0; k < vals_len<decltype(vals)>(); ++k) {
            const int m = band_mode(base + k * stride, L, N0);
            if (m >= 0) B[((int64_t)m * n1 + y) * n2 + z0 + c] = vals[k];
        }
    };
    fft_stages_c<L, 1, INV, C>(s, twL, load, store);
}

// pass Y of the crop: columns (m0, z0 + c), in-band y only
template <int L, bool INV>
__global__ void __launch_bounds__(kFftThreads, NUFFT_FFTN_MINB)
k_fftn_crop_y(const float2* __restrict__ B, int64_t B_vs, int N1, int n2,
              const float2* __restrict__ twL, float2* __restrict__ A, int64_t A_vs) {
    constexpr int C = fftn_cols(L);
    extern __shared__ float2 s[];
    grid_dep_sync();
    const int z0 = blockIdx.x * C;
    const int64_t m0 = blockIdx.y;
    B += blockIdx.z * B_vs;
    A += blockIdx.z * A_vs;
    auto load = [&](int c, int i) {
        return __ldg(B + (m0 * L + i) * n2 + z0 + c);
    };
    auto store = [&](int c, int base, int stride, auto& vals) {
#pragma unroll
        for (int k = 0; k < vals_len<decltype(vals)>(); ++k) {
            const int m = band_mode(base + k * stride, L, N1);
            if (m >= 0) A[(m0 * N1 + m) * n2 + z0 + c] = vals[k];
        }
    };
    fft_stages_c<L, 1, INV, C>(s, twL, load, store);
}

// pass Z of the crop: rows r = m0 * N1 + m1, in-band z only, times the
// deconvolution.  Rows are contiguous in A and in the modes: coalesced
// loads into shared memory, the FFT in place, coalesced stores of the
// in-band cells.
template <int L, bool INV>
__global__ void __launch_bounds__(kFftThreads, NUFFT_FFTN_MINB)
k_fftn_crop_z(const float2* __restrict__ A, int64_t A_vs, const float* __restrict__ d0,
              const float* __restrict__ d1, const float* __restrict__ d2, int N1,
              int N2, int nrows, const float2* __restrict__ twL,
              float2* __restrict__ f, int64_t f_vs) {
    constexpr int C = fftn_cols(L);
    extern __shared__ float2 s[];
    __shared__ float s_d01[C];                   // row corrections d0 * d1
    grid_dep_sync();
    const int r0 = blockIdx.x * C;
    const int rows = min(C, nrows - r0);
    A += blockIdx.y * A_vs + (int64_t)r0 * L;
    f += blockIdx.y * f_vs + (int64_t)r0 * N2;
    constexpr int K = 8;             // loads in flight per thread
    for (int q0 = threadIdx.x; q0 < C * L; q0 += K * kFftThreads) {
        float2 x[K];
#pragma unroll
        for (int k = 0; k < K; ++k) {
            const int q = q0 + k * kFftThreads;
            x[k] = (q < C * L && q / L < rows) ? __ldg(A + q) : make_float2(0.0f, 0.0f);
        }
#pragma unroll
        for (int k = 0; k < K; ++k) {
            const int q = q0 + k * kFftThreads;
            if (q < C * L) s[fpad((q % L) * C + q / L)] = x[k];
        }
    }
    __syncthreads();
    auto none = [](int, int) { return make_float2(0.0f, 0.0f); };
    auto nost = [](int, int, int, auto&) {};
    if (threadIdx.x < rows) {
        const int r = r0 + threadIdx.x;
        s_d01[threadIdx.x] = __ldg(d0 + r / N1) * __ldg(d1 + r % N1);
    }
    fft_stages_c<L, 1, INV, C, true>(s, twL, none, nost);
    __syncthreads();
    // thread t stores mode m = t (+ multiples of the block) of every row
    for (int m = threadIdx.x; m < N2; m += kFftThreads) {
        const float dm = __ldg(d2 + m);
        const int cell = ((m - N2 / 2 + L) % L) * C;
        for (int c = 0; c < rows; ++c) {
            const float d = s_d01[c] * dm;
            const float2 x = s[fpad(cell + c)];
            f[(int64_t)c * N2 + m] = make_float2(x.x * d, x.y * d);
        }
    }
}

// W_L^m tables (fp64 rounded once to fp32, forward sign) for L = n_d
void fftn_tables(Fftn* f) {
    const double two_pi = 6.283185307179586476925286766559;
    size_t tot = 0;
    for (int d = 0; d < 3; ++d) tot += (size_t)f->n[d];
    std::vector<float2> h(tot);
    size_t o = 0;
    for (int d = 0; d < 3; ++d) {
        for (int m = 0; m < f->n[d]; ++m) {
            const double a = two_pi * (double)m / (double)f->n[d];
            h[o + m] = make_float2((float)std::cos(a), (float)-std::sin(a));
        }
        o += (size_t)f->n[d];
    }
    NUFFT_CUDA(cudaMalloc(&f->tw, sizeof(float2) * tot));
    NUFFT_CUDA(cudaMemcpy(f->tw, h.data(), sizeof(float2) * tot, cudaMemcpyHostToDevice));
}

const float2* fftn_tw(const Fftn& f, int d) {
    size_t o = 0;
    for (int e = 0; e < d; ++e) o += (size_t)f.n[e];
    return f.tw + o;
}

template <class K, class... Args>
void fftn_launch(K k, dim3 g, size_t smem, cudaStream_t st, bool dependent,
                 Args... args) {
    prepare((const void*)k, smem);
    if (dependent)
        launch_dependent(k, g, dim3(kFftThreads), smem, st, args...);
    else
        k<<<g, kFftThreads, smem, st>>>(args...);
}

}  // namespace

bool fftn_supported(const int64_t* n) {
    for (int d = 0; d < 3; ++d)
        if (n[d] < 64 || n[d] > 2048 || (n[d] & (n[d] - 1)) != 0) return false;
    return true;
}

void fftn_init(Fftn* f, const int64_t* n, const int64_t* N) {
    fftn_free(f);
    if (!fftn_supported(n)) fail(-1, "fftn: unsupported grid");
    for (int d = 0; d < 3; ++d) {
        f->n[d] = (int)n[d];
        f->N[d] = (int)N[d];
    }
    fftn_tables(f);
}

void fftn_free(Fftn* f) {
    if (f->tw) cudaFree(f->tw);
    if (f->tmp) cudaFree(f->tmp);
    *f = Fftn{};
}

int64_t fftn_scratch_cells(const Fftn& f) {
    return (int64_t)f.N[0] * f.n[1] * f.n[2];
}

void fftn_reserve(Fftn* f, int nv) {
    if (nv <= f->tmp_batch) return;
    if (f->tmp) {
        NUFFT_CUDA(cudaDeviceSynchronize());     // scratch may still be in use
        cudaFree(f->tmp);
        f->tmp = nullptr;
        f->tmp_batch = 0;
    }
    NUFFT_CUDA(cudaMalloc(&f->tmp, sizeof(float2) * (size_t)fftn_scratch_cells(*f) * nv));
    f->tmp_batch = nv;
}

// The periodic copies of k grids (stored layout h, G cells apart) from
// their interior: three k_halo_fill passes (need: marked planes only).
void halo_fill(float2* Gv, int64_t G, const GridHalo& h, int n0, int n1, int n2, int k,
               const uint8_t* need, cudaStream_t st) {
    const int64_t work[3] = {(int64_t)(h.lo[0] + h.hi[0]) * h.P[1] * h.P[2],
                             (int64_t)n0 * (h.lo[1] + h.hi[1]) * h.P[2],
                             (int64_t)n0 * n1 * (h.lo[2] + h.hi[2])};
    for (int pass = 2; pass >= 0; --pass) {
        if (work[pass] == 0) continue;
        const dim3 g((unsigned)((work[pass] + 255) / 256), (unsigned)k);
        k_halo_fill<<<g, 256, 0, st>>>(Gv, G, h, n0, n1, n2, pass, need);
        NUFFT_LAUNCH("k_halo_fill");
    }
}

void fftn_pad(Fftn* f, const float2* modes, const float* const* dec, float2* grid,
              int nv, bool inv, cudaStream_t st, const GridHalo* halo,
              const uint8_t* need) {
    if (!halo) need = nullptr;
    fftn_reserve(f, nv);
    const int n0 = f->n[0], n1 = f->n[1], n2 = f->n[2];
    const int N0 = f->N[0], N1 = f->N[1], N2 = f->N[2];
    // cells per stored grid (with the halo, if any); the first pass's
    // output A also lives in each grid's memory
    const int64_t K = (int64_t)N0 * N1 * N2,
                  G = halo ? (int64_t)halo->P[0] * halo->P[1] * halo->P[2]
                           : (int64_t)n0 * n1 * n2;
    const GridHalo h = halo ? *halo : GridHalo{};
    const int64_t Bs = fftn_scratch_cells(*f);
    float2* A = grid;            // A[m0][m1][z] in the grid's own memory
    float2* B = f->tmp;
    for (int v0 = 0; v0 < nv; v0 += 65535) {
        const int k = std::min(65535, nv - v0);
        const float2* fv = modes + v0 * K;
        float2* Av = A + v0 * G;
        float2* Bv = B + v0 * Bs;
        float2* Gv = grid + v0 * G;
        NUFFT_FFT_LEN_SWITCH(n2, {
            const int nrows = N0 * N1;
            dim3 g((unsigned)((nrows + fftn_cols(L) - 1) / fftn_cols(L)), (unsigned)k);
            if (inv) fftn_launch(k_fftn_pad_z<L, true>, g, fftn_smem<L>(), st, false, fv, K,
                                 dec[0], dec[1], dec[2], N1, N2, nrows, fftn_tw(*f, 2), Av, G);
            else fftn_launch(k_fftn_pad_z<L, false>, g, fftn_smem<L>(), st, false, fv, K,
                             dec[0], dec[1], dec[2], N1, N2, nrows, fftn_tw(*f, 2), Av, G);
        });
        NUFFT_LAUNCH("k_fftn_pad_z");
        NUFFT_FFT_LEN_SWITCH(n1, {
            dim3 g((unsigned)(n2 / fftn_cols(L)), (unsigned)N0, (unsigned)k);
            if (inv) fftn_launch(k_fftn_pad_y<L, true>, g, fftn_smem<L>(), st, true,
                                 (const float2*)Av, G, N1, n2, fftn_tw(*f, 1), Bv, Bs);
            else fftn_launch(k_fftn_pad_y<L, false>, g, fftn_smem<L>(), st, true,
                             (const float2*)Av, G, N1, n2, fftn_tw(*f, 1), Bv, Bs);
        });
        NUFFT_LAUNCH("k_fftn_pad_y");
        NUFFT_FFT_LEN_SWITCH(n0, {
            dim3 g((unsigned)(n2 / fftn_cols(L)), (unsigned)n1, (unsigned)k);
            const float2* Bc = Bv;
            const float2* tw = fftn_tw(*f, 0);
            const size_t sm = fftn_smem<L>();
            if (need) {
                if (inv) fftn_launch(k_fftn_pad_x<L, true, true, true>, g, sm, st, true,
                                     Bc, Bs, N0, n1, n2, tw, Gv, G, h, need);
                else fftn_launch(k_fftn_pad_x<L, false, true, true>, g, sm, st, true,
                                 Bc, Bs, N0, n1, n2, tw, Gv, G, h, need);
            } else if (halo) {
                if (inv) fftn_launch(k_fftn_pad_x<L, true, true, false>, g, sm, st, true,
                                     Bc, Bs, N0, n1, n2, tw, Gv, G, h, need);
                else fftn_launch(k_fftn_pad_x<L, false, true, false>, g, sm, st, true,
                                 Bc, Bs, N0, n1, n2, tw, Gv, G, h, need);
            } else {
                if (inv) fftn_launch(k_fftn_pad_x<L, true, false, false>, g, sm, st, true,
                                     Bc, Bs, N0, n1, n2, tw, Gv, G, h, need);
                else fftn_launch(k_fftn_pad_x<L, false, false, false>, g, sm, st, true,
                                 Bc, Bs, N0, n1, n2, tw, Gv, G, h, need);
            }
        });
        NUFFT_LAUNCH("k_fftn_pad_x");
        if (halo) halo_fill(Gv, G, h, n0, n1, n2, k, need, st);
    }
}

bool fftn_pad_slab(Fftn* f, const float2* modes, const float* const* dec, float2* grid,
                   int nv, bool inv, cudaStream_t st, const GridHalo& h,
                   const uint8_t* need, const int* xmap, const int* xlist, int nx) {
    const int n0 = f->n[0], n1 = f->n[1], n2 = f->n[2];
    const int N0 = f->N[0], N1 = f->N[1], N2 = f->N[2];
    const int64_t K = (int64_t)N0 * N1 * N2;
    const int64_t G = (int64_t)h.P[0] * h.P[1] * h.P[2];
    const int64_t Bs = fftn_scratch_cells(*f);
    const int64_t t1 = (int64_t)nx * N1 * N2, t2 = (int64_t)nx * n1 * N2;
    if (nx < 1 || t1 > G || t2 > Bs) return false;   // scratch planes do not fit
    fftn_reserve(f, nv);
    for (int v0 = 0; v0 < nv; v0 += 65535) {
        const int k = std::min(65535, nv - v0);
        const float2* fv = modes + v0 * K;
        float2* T1 = grid + v0 * G;       // dead before the Z pass writes the grid
        float2* T2 = f->tmp + v0 * Bs;
        float2* Gv = grid + v0 * G;
        NUFFT_FFT_LEN_SWITCH(n0, {
            dim3 g((unsigned)((N2 + fftn_cols(L) - 1) / fftn_cols(L)), (unsigned)N1, (unsigned)k);
            if (inv) fftn_launch(k_fftn_slab_x<L, true>, g, fftn_smem<L>(), st, false, fv, K,
                                 dec[0], dec[1], dec[2], N0, N1, N2, xmap, fftn_tw(*f, 0), T1, G);
            else fftn_launch(k_fftn_slab_x<L, false>, g, fftn_smem<L>(), st, false, fv, K,
                             dec[0], dec[1], dec[2], N0, N1, N2, xmap, fftn_tw(*f, 0), T1, G);
        });
        NUFFT_LAUNCH("k_fftn_slab_x");
        NUFFT_FFT_LEN_SWITCH(n1, {
            dim3 g((unsigned)((N2 + fftn_cols(L) - 1) / fftn_cols(L)), (unsigned)nx, (unsigned)k);
            if (inv) fftn_launch(k_fftn_slab_y<L, true>, g, fftn_smem<L>(), st, true,
                                 (const float2*)T1, G, N1, N2, fftn_tw(*f, 1), T2, Bs);
            else fftn_launch(k_fftn_slab_y<L, false>, g, fftn_smem<L>(), st, true,
                             (const float2*)T1, G, N1, N2, fftn_tw(*f, 1), T2, Bs);
        });
        NUFFT_LAUNCH("k_fftn_slab_y");
        NUFFT_FFT_LEN_SWITCH(n2, {
            const int nrows = nx * n1;
            dim3 g((unsigned)((nrows + fftn_cols(L) - 1) / fftn_cols(L)), 1u, (unsigned)k);
            if (inv) fftn_launch(k_fftn_slab_z<L, true>, g, fftn_smem<L>(), st, true,
                                 (const float2*)T2, Bs, N2, nrows, n1, xlist, h,
                                 fftn_tw(*f, 2), Gv, G);
            else fftn_launch(k_fftn_slab_z<L, false>, g, fftn_smem<L>(), st, true,
                             (const float2*)T2, Bs, N2, nrows, n1, xlist, h,
                             fftn_tw(*f, 2), Gv, G);
        });
        NUFFT_LAUNCH("k_fftn_slab_z");
        halo_fill(Gv, G, h, n0, n1, n2, k, need, st);
    }
    return true;
}

void fftn_crop(Fftn* f, float2* grid, const float* const* dec, float2* modes, int nv,
               bool inv, cudaStream_t st) {
    fftn_reserve(f, nv);
    const int n0 = f->n[0], n1 = f->n[1], n2 = f->n[2];
    const int N0 = f->N[0], N1 = f->N[1], N2 = f->N[2];
    const int64_t K = (int64_t)N0 * N1 * N2, G = (int64_t)n0 * n1 * n2;
    const int64_t Bs = fftn_scratch_cells(*f);
    for (int v0 = 0; v0 < nv; v0 += 65535) {
        const int k = std::min(65535, nv - v0);
        float2* Gv = grid + v0 * G;
        float2* Bv = f->tmp + v0 * Bs;
        float2* Av = Gv;         // A'[m0][m1][z] in the grid's memory, dead after pass X
        float2* fv = modes + v0 * K;
        NUFFT_FFT_LEN_SWITCH(n0, {
            dim3 g((unsigned)(n2 / fftn_cols(L)), (unsigned)n1, (unsigned)k);
            if (inv) fftn_launch(k_fftn_crop_x<L, true>, g, fftn_smem<L>(), st, false,
                                 (const float2*)Gv, G, N0, n1, n2, fftn_tw(*f, 0), Bv, Bs);
            else fftn_launch(k_fftn_crop_x<L, false>, g, fftn_smem<L>(), st, false,
                             (const float2*)Gv, G, N0, n1, n2, fftn_tw(*f, 0), Bv, Bs);
        });
        NUFFT_LAUNCH("k_fftn_crop_x");
        NUFFT_FFT_LEN_SWITCH(n1, {
            dim3 g((unsigned)(n2 / fftn_cols(L)), (unsigned)N0, (unsigned)k);
            if (inv) fftn_launch(k_fftn_crop_y<L, true>, g, fftn_smem<L>(), st, true,
                                 (const float2*)Bv, Bs, N1, n2, fftn_tw(*f, 1), Av, G);
            else fftn_launch(k_fftn_crop_y<L, false>, g, fftn_smem<L>(), st, true,
                             (const float2*)Bv, Bs, N1, n2, fftn_tw(*f, 1), Av, G);
        });
        NUFFT_LAUNCH("k_fftn_crop_y");
        NUFFT_FFT_LEN_SWITCH(n2, {
            const int nrows = N0 * N1;
            dim3 g((unsigned)((nrows + fftn_cols(L) - 1) / fftn_cols(L)), (unsigned)k);
            if (inv) fftn_launch(k_fftn_crop_z<L, true>, g, fftn_smem<L>(), st, true,
                                 (const float2*)Av, G, dec[0], dec[1], dec[2], N1, N2,
                                 nrows, fftn_tw(*f, 2), fv, K);
            else fftn_launch(k_fftn_crop_z<L, false>, g, fftn_smem<L>(), st, true,
                             (const float2*)Av, G, dec[0], dec[1], dec[2], N1, N2, nrows,
                             fftn_tw(*f, 2), fv, K);
        });
        NUFFT_LAUNCH("k_fftn_crop_z");
    }
}

namespace {
}  // namespace

bool pdl_on() {
    static const bool on = [] {
        const char* e = std::getenv("NUFFT_PDL");
        return (e && *e) ? std::atoi(e) != 0 : true;
    }();
    return on;
}

bool fft1_supported(int64_t n) {
    return n >= (1 << 12) && n <= (1 << 22) && (n & (n - 1)) == 0;
}

void fft1_init(Fft1* f, int64_t n) {
    fft1_free(f);
    if (!fft1_supported(n)) fail(-1, "fft1: unsupported size");
    const int k = ilog2((int)n);
    f->n = (int)n;
    f->N1 = 1 << (k / 2);
    f->N2 = 1 << (k - k / 2);
    // [W_N1^m, m < N1][W_N2^m, m < N2][W_n^m, m < N2], forward sign, from
    // fp64 host cos/sin rounded once to fp32
    const double two_pi = 6.283185307179586476925286766559;
    std::vector<float2> h((size_t)f->N1 + 2 * (size_t)f->N2);
    auto fill = [&](float2* dst, int count, double len) {
        for (int m = 0; m < count; ++m) {
            const double a = two_pi * (double)m / len;
            dst[m] = make_float2((float)std::cos(a), (float)-std::sin(a));
        }
    };
    fill(h.data(), f->N1, f->N1);
    fill(h.data() + f->N1, f->N2, f->N2);
    fill(h.data() + f->N1 + f->N2, f->N2, (double)n);
    NUFFT_CUDA(cudaMalloc(&f->tw, sizeof(float2) * h.size()));
    NUFFT_CUDA(cudaMemcpy(f->tw, h.data(), sizeof(float2) * h.size(),
                          cudaMemcpyHostToDevice));
}

void fft1_free(Fft1* f) {
    if (f->tw) cudaFree(f->tw);
    if (f->tmp) cudaFree(f->tmp);
    *f = Fft1{};
}

void fft1_reserve(Fft1* f, int nv) {
    if (nv <= f->tmp_batch) return;
    if (f->tmp) {
        NUFFT_CUDA(cudaDeviceSynchronize());     // scratch may still be in use
        cudaFree(f->tmp);
        f->tmp = nullptr;
        f->tmp_batch = 0;
    }
    NUFFT_CUDA(cudaMalloc(&f->tmp, sizeof(float2) * (size_t)f->n * nv));
    f->tmp_batch = nv;
}

void fft1_cols(Fft1* f, const float2* in, int64_t N, const float* dec, int nv,
               bool inv, cudaStream_t st) {
    fft1_reserve(f, nv);
    const bool pad = dec != nullptr;
    const int64_t stride = pad ? N : f->n;
    for (int v0 = 0; v0 < nv; v0 += 65535) {
        const int k = std::min(65535, nv - v0);
        run_cols(*f, in + v0 * stride, stride, N, dec, pad, inv,
                 f->tmp + (int64_t)v0 * f->n, k, st);
    }
}

void fft1_rows(Fft1* f, float2* out, int64_t N, const float* dec, int nv, bool inv,
               cudaStream_t st) {
    const bool crop = dec != nullptr;
    const int64_t stride = crop ? N : f->n;
    for (int v0 = 0; v0 < nv; v0 += 65535) {
        const int k = std::min(65535, nv - v0);
        run_rows(*f, f->tmp + (int64_t)v0 * f->n, crop, inv, out + v0 * stride, stride,
                 N, dec, k, st);
    }
}

}  // namespace nufft
