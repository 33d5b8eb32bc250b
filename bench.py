"""Benchmark: NU points/s of the NUFFT execute path on B200 (one JSON line).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config C]
                    [--impl reference] [--no-per-config] [--no-cpu-baseline]

Headline workload (default --config 4): 3-D type 2, 256^3 complex64 modes,
M = 5e7 points (half uniform on [-pi, pi)^3, half Gaussian with sigma 0.3
about the origin, wrapped), eps = 1e-6, isign = -1 -- the largest of the
five workloads that runs at eps = 1e-6 on one GPU.  A step is one plan
execute over device-resident inputs: pad/deconvolve -> FFT -> interp
(setpts and sort excluded: the reference's "exec" protocol).  Each step is
bracketed by CUDA events on the execute stream; L2 is flushed between steps
outside the events (a 256 MiB write, then a read of the same buffer, so the
L2 holds clean unrelated lines).

Keys besides the contract's: `roofline` (the dominant own kernel, from the
plan's live stage events and the kernel's algorithmic bytes; `step_roofline`
the same for the whole execute with the full pipeline's algorithmic bytes),
`e2e` (the same metric through the public API from pinned host memory, H2D
and D2H copies timed), `cpu_baseline` (the CPU restatement of the reference
algorithm, oracle/port.py, on a bounded sample, rank 0 at N=1), `per_config`
(the other four workloads and the standalone expi, each with its own device
value, roofline, e2e and CPU baseline), `gpu_launches`, `clocks`.

With N > 1 GPUs (torchrun) the workloads are partitioned, one process per
GPU, strong scaling (the whole problem fixed): type 2 split by target (the
points of each rank form one x-slab of the grid, 3-D slabs of equal modelled
cost -- points to interpolate plus grid planes to transform; every rank
builds the planes of the fine grid its points read -- `value` -- or rank 0
builds it whole and broadcasts it over NCCL -- the `broadcast` key), the
batched type 1
split by vector, type 1 split by point with an NCCL all-reduce of the fine
grids, type 3 split by target and expi split by element.  Every partition
reports the rel-L2 of its result against one GPU running the whole problem
(on a subset of the outputs).

--impl reference times the CPU restatement of the reference algorithm
(oracle/port.py; the reference's own GPU path is Apple Metal/MLX and has no
CPU type-1/2 path) on the host cores, rank 0 only, on the same workload.
"""

import argparse
import importlib.util
import json
import os
import re
import statistics
import sys
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

METRIC = ("NU points/sec per GPU (spread+FFT+deconv, device-timed) at "
          "eps=1e-6; % HBM roofline")
HEADLINE = 4
PER_CONFIG = (1, 2, 3, 5, 6)
L2_NOTE = "flushed between steps (256 MiB write, then read)"


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--config", type=int, default=HEADLINE)
    ap.add_argument("--impl", default="native", choices=["native", "reference"])
    ap.add_argument("--scale", type=float, default=1.0,
                    help="point-count scale (1.0 = the full workload)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-per-config", action="store_true")
    return ap.parse_args()


def load_gen():
    """mlx_nufft_b200/gen.py loaded by file path: the synthetic generators
    without importing the package (whose __init__ loads the native
    library; the CPU reference arm must not)."""
    path = os.path.join(ROOT, "mlx_nufft_b200", "gen.py")
    spec = importlib.util.spec_from_file_location("_nufft_bench_gen", path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


# ------------------------------------------------------------ workloads
def unit_of(cfg):
    if cfg["type"] == 0:
        return "elem/s", "elements"
    if cfg["type"] == 1 and cfg.get("n_trans", 1) > 1:
        return "NU pt-vec/s", "points x vectors"
    if cfg["type"] == 3:
        return "NU pts/s", "sources (targets as many)"
    return "NU pts/s", "points"


def step_bytes(cfg, info):
    """Compulsory DRAM bytes of one whole execute (spread / interp + FFT +
    deconvolution) for this data layout: per point its cells (8 B/dim),
    permutation (4 B) and strength or output (8 B per vector); per fine-grid
    cell the spread write or interp read (8 B) and one FFT read + write
    (16 B); per mode the deconvolution read + write (16 B) or the modes read
    plus the pad write (8 + 8 B/cell)."""
    if cfg["type"] == 0:
        return 16 * int(cfg["phi"].size)
    dim = int(info.dim)
    n = int(np.prod([int(info.n_up[d]) for d in range(dim)]))
    if cfg["type"] == 1:
        M = int(info.M)
        B = int(cfg.get("n_trans", 1))
        K = int(np.prod(cfg["n_modes"]))
        return M * (4 + 8 * dim) + B * (M * 8 + n * 24 + K * 16)
    if cfg["type"] == 2:
        M = int(info.M)
        K = int(np.prod(cfg["n_modes"]))
        return K * 8 + n * (8 + 16 + 8) + M * (4 + 8 * dim + 8)
    nf = int(np.prod([int(info.nf[d]) for d in range(dim)]))
    Ms, Nt = int(info.M), int(info.N_tgt)
    return (Ms * (8 + 8 + 4 + 8 * dim) + nf * 16 + n * (8 + 16 + 8)
            + Nt * (8 * dim + 8 + 8))


def kernel_bytes(cfg, info, stage):
    """Compulsory DRAM bytes of the dominant own kernel of a stage:
    interp -- per point cells (8 B/dim) + permutation (4 B) + output (8 B)
    (+ phase 8 B for type-3 targets), the grid read once (8 B/cell);
    spread -- per point cells + permutation + strength per vector (+ phase),
    the grid written once per vector."""
    dim = int(info.dim)
    n = int(np.prod([int(info.n_up[d]) for d in range(dim)]))
    if stage == "interp":
        if cfg["type"] == 3:
            return int(info.N_tgt) * (8 * dim + 4 + 8 + 8) + n * 8
        return int(info.M) * (8 * dim + 4 + 8) + n * 8
    B = int(cfg.get("n_trans", 1))
    if cfg["type"] == 3:
        nf = int(np.prod([int(info.nf[d]) for d in range(dim)]))
        return int(info.M) * (8 * dim + 4 + 8 + 8) + nf * 8
    return int(info.M) * (8 * dim + 4 + 8 * B) + B * n * 8


def config_keys(cfg, k, info=None, world=1, rank_points=None):
    d = {"workload": cfg["name"], "config": k, "eps": cfg.get("eps"),
         "isign": cfg["isign"], "l2": L2_NOTE}
    if cfg["type"] == 0:
        d["elements"] = int(cfg["phi"].size)
        return d
    d["points"] = int(cfg["x"][0].size)
    if rank_points is not None:
        d["points_per_rank"] = int(rank_points)
    else:
        d["points_per_rank"] = int(cfg["x"][0].size) // max(1, world)
    d["vectors"] = int(cfg.get("n_trans", 1))
    if "n_modes" in cfg:
        d["n_modes"] = list(cfg["n_modes"])
    if cfg["type"] == 3:
        d["targets"] = int(cfg["s"][0].size)
    if info is not None:
        d["w"] = int(info.w)
        d["n_up"] = [int(info.n_up[i]) for i in range(int(info.dim))]
        d["tiled"] = bool(info.tiled)
    return d


PROFILE_OF = {1: "cfg1", 2: "interp1_stream_cfg2", 3: "spread_planes_cfg3",
              4: "interp_tma_cfg4", 5: "cfg5", 6: "expi_cfg6"}


def ncu_traffic(k):
    """Per-launch DRAM bytes of a config's dominant kernel from its committed
    ncu summary (profiles/<kernel>_cfg<k>.md, line
    'traffic_bytes_per_launch: <n>'); None if absent."""
    pdir = os.path.join(ROOT, "profiles")
    tag = PROFILE_OF.get(k)
    if not tag or not os.path.isdir(pdir):
        return None
    for f in sorted(os.listdir(pdir)):
        if not f.endswith(".md") or tag not in f:
            continue
        m = re.search(r"^traffic_bytes_per_launch:\s*([0-9.eE+]+)",
                      open(os.path.join(pdir, f)).read(), re.M)
        if m:
            return float(m.group(1))
    return None


# ------------------------------------------------------------ clocks
class ClockSampler:
    """SM clock and clock-event reasons of this rank's GPU, sampled through
    NVML on a background thread every `period` seconds between start() and
    stop() (stop() takes one last sample before returning)."""

    REASONS = (("sw_power_cap", 0x4), ("hw_slowdown", 0x8),
               ("sw_thermal_slowdown", 0x20), ("hw_thermal_slowdown", 0x40),
               ("hw_power_brake_slowdown", 0x80))

    def __init__(self, cuda_index, period=0.005):
        self.period = period
        self.samples = []
        self.handle = None
        self.max_mhz = None
        try:
            import pynvml
            import torch
            pynvml.nvmlInit()
            self.nvml = pynvml
            uuid = getattr(torch.cuda.get_device_properties(cuda_index),
                           "uuid", None)
            try:
                self.handle = pynvml.nvmlDeviceGetHandleByUUID(f"GPU-{uuid}")
            except Exception:
                self.handle = pynvml.nvmlDeviceGetHandleByIndex(cuda_index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(
                self.handle, pynvml.NVML_CLOCK_SM)
        except Exception:
            self.handle = None

    def _sample(self):
        n = self.nvml
        sm = n.nvmlDeviceGetClockInfo(self.handle, n.NVML_CLOCK_SM)
        try:
            r = n.nvmlDeviceGetCurrentClocksEventReasons(self.handle)
        except Exception:
            r = n.nvmlDeviceGetCurrentClocksThrottleReasons(self.handle)
        self.samples.append((sm, r))

    def _loop(self):
        while not self._stop.is_set():
            try:
                self._sample()
            except Exception:
                return
            self._stop.wait(self.period)

    def start(self):
        import threading
        if self.handle is None:
            return
        self._stop = threading.Event()
        self._thread = threading.Thread(target=self._loop, daemon=True)
        self._thread.start()

    def stop(self):
        if self.handle is None:
            return None
        try:
            self._sample()
        except Exception:
            pass
        self._stop.set()
        self._thread.join()
        if not self.samples:
            return None
        bits = 0
        for _, r in self.samples:
            bits |= int(r)
        return {"sm_mhz": statistics.median(sm for sm, _ in self.samples),
                "sm_max_mhz": self.max_mhz, "samples": len(self.samples),
                "reasons": [name for name, b in self.REASONS if bits & b],
                "source": "nvml"}


# ------------------------------------------------------------ CPU baseline
_CPU = None          # the CpuWork of the reference arm's forked workers


class CpuWork:
    """The reference algorithm restated on the CPU (oracle/port.py, fp64) on
    one workload, split into the whole fine-grid work (`grid`: deconvolve +
    pad + FFT, or FFT + crop per vector; scipy.fft on `threads` threads) and
    the per-point work (`points`: fold + spread or interp) of a sample of
    the points, extrapolated to all points.  Plan-time work (corrections,
    type-3 geometry) is done once in the constructor; the reference's exec
    protocol excludes it."""

    def __init__(self, cfg, threads):
        from oracle import port
        self.port = port
        self.cfg = cfg
        self.threads = max(1, int(threads))
        self.type = cfg["type"]
        self.pool = None
        self.V = None
        if self.type == 0:
            self.n = int(cfg["phi"].size)
            return
        self.x = [np.asarray(v, dtype=np.float64) for v in cfg["x"]]
        self.M = self.x[0].size
        self.dim = len(self.x)
        self.B = int(cfg.get("n_trans", 1))
        if self.type == 3:
            self.g = port.T3Geometry(self.x, cfg["s"], cfg["eps"], cfg["isign"])
            self.Nt = cfg["s"][0].size
            self.c = np.asarray(cfg["data"], dtype=np.complex128)
            dec = np.ones(self.g.nf)
            for d in range(self.dim):
                dec = dec * self.g.mode_dec[d].reshape(
                    (1,) * d + (-1,) + (1,) * (self.dim - d - 1))
            self.dec3 = dec
            self.grid_shape = tuple(self.g.n_up)
            self.w = self.g.w
            return
        N = tuple(cfg["n_modes"])
        self.N = N
        self.w, self.beta, self.nup = port.fine_grid_sizes(N, cfg["eps"])
        self.decs = []
        for d in range(self.dim):
            k = np.arange(-(N[d] // 2), N[d] - N[d] // 2, dtype=np.float64)
            self.decs.append(1.0 / port.kernel_ft(2.0 * np.pi * k / self.nup[d],
                                                  self.beta, self.w))
        self.grid_shape = tuple(self.nup)
        if self.type == 2:
            self.f = np.asarray(cfg["data"], dtype=np.complex128).reshape(N)
        else:
            self.c = np.asarray(cfg["data"], dtype=np.complex128).reshape(
                self.B, -1)

    # -- helpers ---------------------------------------------------------
    def _fft(self, H, isign):
        import scipy.fft as sf
        if isign > 0:
            return sf.ifftn(H, workers=self.threads, overwrite_x=True) * float(H.size)
        return sf.fftn(H, workers=self.threads, overwrite_x=True)

    def _band(self, d):
        return self.port._band(self.N[d], self.nup[d])

    def _cells(self, ix):
        i1s, frs = [], []
        for d in range(self.dim):
            i1, fr64, _ = self.port.cells_fold(self.x[d][ix], self.nup[d], self.w)
            i1s.append(i1)
            frs.append(fr64)
        return i1s, frs

    def _interp_part(self, ix):
        i1s, frs = self._cells(ix)
        return self.port.interp(self.V, i1s, frs, self.w, self.beta, chunk=8192)

    def units(self):
        if self.type == 0:
            return self.n
        if self.type == 1:
            return self.M * self.B
        return self.M

    # -- the two halves of one execute -------------------------------------
    def grid(self):
        """Seconds of the whole-grid work of one execute."""
        port = self.port
        dim = getattr(self, "dim", 0)
        if self.type == 0:
            return 0.0
        t0 = time.perf_counter()
        if self.type == 2:
            g = self.f.copy()
            for d in range(dim):
                g = g * self.decs[d].reshape((1,) * d + (-1,) + (1,) * (dim - d - 1))
            H = np.zeros(self.grid_shape, dtype=np.complex128)
            H[np.ix_(*[self._band(d) for d in range(dim)])] = g
            V = self._fft(H, self.cfg["isign"])
            t = time.perf_counter() - t0
            if self.pool is not None:
                self.V[...] = V         # hand-over to the workers, untimed
            else:
                self.V = V
            return t
        if self.type == 1:
            # FFT + crop + deconvolve of one vector's grid, times B
            G = np.empty(self.grid_shape, dtype=np.complex128)
            G.real = 1.0
            G.imag = 0.5
            t0 = time.perf_counter()
            V = self._fft(G, self.cfg["isign"])
            out = V[np.ix_(*[self._band(d) for d in range(dim)])]
            for d in range(dim):
                out = out * self.decs[d].reshape((1,) * d + (-1,) + (1,) * (dim - d - 1))
            return (time.perf_counter() - t0) * self.B
        # type 3: deconvolve + pad of the spread grid, FFT (the spread grid
        # values do not change the cost; the spread itself is per point)
        g = self.g
        Bg = np.ones(g.nf, dtype=np.complex128)
        t0 = time.perf_counter()
        H = np.zeros(g.n_up, dtype=np.complex128)
        H[np.ix_(*[np.mod(np.arange(-g.nf[d] // 2, g.nf[d] // 2), g.n_up[d])
                   for d in range(g.dim)])] = Bg * self.dec3
        self.V = self._fft(H, g.isign)
        return time.perf_counter() - t0

    def points(self, sample):
        """Seconds of the per-point work of one execute, measured on
        `sample` points (sources and targets for type 3) and extrapolated
        to all of them; needs grid() to have run (interpolation reads its
        grid)."""
        port = self.port
        if self.type == 0:
            t0 = time.perf_counter()
            np.exp(1j * self.cfg["isign"] * self.cfg["phi"])
            return time.perf_counter() - t0
        sample = int(min(sample, self.M))
        if self.type == 2:
            parts = [p for p in np.array_split(np.arange(sample), 4 * self.threads)
                     if p.size]
            t0 = time.perf_counter()
            if self.pool is not None:
                self.pool.map(_pool_interp, [(int(p[0]), int(p[-1]) + 1) for p in parts])
            else:
                for p in parts:
                    self._interp_part(p)
            return (time.perf_counter() - t0) * (self.M / sample)
        if self.type == 1:
            ix = np.arange(sample)
            t0 = time.perf_counter()
            i1s, frs = self._cells(ix)
            port.spread(i1s, frs, self.c[0][ix], self.nup, self.w, self.beta,
                        chunk=65536)
            return (time.perf_counter() - t0) * (self.M / sample) * self.B
        g = self.g
        ns, nt = min(sample, self.M), min(sample, self.Nt)
        t0 = time.perf_counter()
        cp = self.c[:ns] * g.prephase[:ns]
        port.spread([v[:ns] for v in g.i1], [v[:ns] for v in g.fr], cp,
                    g.nf, g.w, g.beta, chunk=65536)
        ts = (time.perf_counter() - t0) * (self.M / ns)
        t1 = time.perf_counter()
        port.interp(self.V, [v[:nt] for v in g.t_i1], [v[:nt] for v in g.t_fr],
                    g.w, g.beta, chunk=8192) * g.post[:nt]
        return ts + (time.perf_counter() - t1) * (self.Nt / nt)

    def describe(self, sample):
        t = self.threads
        if self.type == 0:
            return f"numpy exp(1j*phi) fp64 over all {self.n} elements"
        s = min(sample, self.M)
        if self.type == 2:
            what = (f"deconvolve+pad+FFT of the full grid; fold+interp of "
                    f"{s} of {self.M} points")
        elif self.type == 1:
            what = (f"FFT+crop of the full grid and fold+spread of {s} of "
                    f"{self.M} points, per vector, x{self.B} vectors")
        else:
            what = (f"prephase+spread of {s} of {self.M} sources, deconvolve+"
                    f"pad+FFT of the full grid, interp x post of "
                    f"{min(s, self.Nt)} of {self.Nt} targets")
        return (f"oracle/port.py fp64 on {t} thread(s): {what}"
                + ("" if s == getattr(self, "M", s) else
                   ", per-point time extrapolated to all points"))


def _pool_interp(span):
    lo, hi = span
    _CPU._interp_part(np.arange(lo, hi))
    return 0


def cpu_baseline(cfg, threads=1, budget_s=8.0):
    """The CPU restatement on `threads` threads: the whole grid work once
    and the per-point work of a sample sized to take about budget_s."""
    cw = CpuWork(cfg, threads)
    tg = cw.grid()
    if cw.type == 0:
        sample = 0
        tp = cw.points(0)
    else:
        probe = min(cw.M, 20_000)
        per_all = cw.points(probe)                  # extrapolated seconds
        frac = min(1.0, budget_s / max(per_all, 1e-9))
        sample = int(min(cw.M, max(probe, frac * cw.M)))
        tp = cw.points(sample)
    unit, _ = unit_of(cfg)
    return {"value": cw.units() / (tg + tp), "unit": unit, "cores": cw.threads,
            "kind": "port", "sample": cw.describe(sample), "grid_s": tg,
            "points_s_extrapolated": tp}


def run_reference(args, budget_s=150.0):
    """--impl reference: the CPU restatement with all host threads (FFT on
    scipy.fft workers, type-2 per-point work on a fork pool), rank 0 only.
    Every step does the whole grid work and the per-point work of a sample
    sized so the whole --warmup + --steps run stays near budget_s."""
    global _CPU
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    gen = load_gen()
    cfg = gen.config(args.config, scale=args.scale)
    threads = os.cpu_count() or 1
    cw = CpuWork(cfg, threads)
    shm = None
    if cw.type == 2:
        # the grid lives in shared memory, so the forked workers read the
        # step's own FFT output
        from multiprocessing import get_context, shared_memory
        shm = shared_memory.SharedMemory(create=True,
                                         size=int(np.prod(cw.grid_shape)) * 16)
        cw.V = np.ndarray(cw.grid_shape, dtype=np.complex128, buffer=shm.buf)
        _CPU = cw
        cw.pool = get_context("fork").Pool(threads)
    try:
        n_steps = max(1, args.warmup + args.steps)
        sample = 0
        if cw.type != 0:
            tg = cw.grid()
            probe = min(cw.M, 200_000)
            tp = cw.points(probe)
            per_step = budget_s / n_steps
            sample = int(min(cw.M, max(probe, (per_step - tg) / max(tp, 1e-9) * cw.M)))
        vals = []
        for i in range(n_steps):
            tg = cw.grid()
            tp = cw.points(sample)
            if i >= args.warmup:
                vals.append(cw.units() / (tg + tp))
        v = float(np.median(vals))
    finally:
        if cw.pool is not None:
            cw.pool.close()
            cw.pool.join()
        if shm is not None:
            del cw.V
            shm.close()
            shm.unlink()
    unit, _ = unit_of(cfg)
    ckeys = config_keys(cfg, args.config, None, args.gpus)
    if cw.type in (1, 2, 3):
        ckeys["w"] = int(cw.w)
        ckeys["n_up"] = [int(v) for v in cw.grid_shape]
    frac = 1.0 if cw.type == 0 else min(1.0, sample / cw.M)
    line = {"impl": "reference", "metric": METRIC, "value": v, "unit": unit,
            "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": cw.units() / v * 1e3,
            "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "f64", "data": "synthetic",
            "config": ckeys, "sample_fraction": frac,
            "cpu_baseline": {"value": v, "unit": unit, "cores": threads,
                             "kind": "port",
                             "sample": cw.describe(sample) + " per step"
                                       + (" (FFT: scipy.fft workers; per-point work: "
                                          "fork pool)" if cw.type == 2 else "")},
            "e2e": {"value": v, "unit": unit, "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


# ------------------------------------------------------------ GPU context
class Ctx:
    def __init__(self, args):
        import torch
        import torch.distributed as dist
        self.torch, self.dist, self.args = torch, dist, args
        self.world = int(os.environ.get("WORLD_SIZE", "1"))
        self.rank = int(os.environ.get("RANK", "0"))
        self.local = int(os.environ.get("LOCAL_RANK", "0"))
        torch.cuda.set_device(self.local)
        self.dev = torch.device("cuda", self.local)
        if self.world > 1:
            from datetime import timedelta
            # NCCL may print its version banner on file descriptor 1 while
            # the communicator is set up; send that to stderr so that rank
            # 0's stdout carries only the JSON line
            sys.stdout.flush()
            saved = os.dup(1)
            os.dup2(2, 1)
            try:
                dist.init_process_group("nccl", timeout=timedelta(seconds=240),
                                        device_id=self.dev)
                dist.barrier()
                torch.cuda.synchronize()
            finally:
                sys.stdout.flush()
                os.dup2(saved, 1)
                os.close(saved)
        self.flushbuf = torch.empty(256 * 2 ** 20, dtype=torch.uint8, device=self.dev)

    def barrier(self):
        if self.world > 1:
            self.dist.barrier()
        self.torch.cuda.synchronize()

    def allmax(self, v):
        t = self.torch.tensor([float(v)], dtype=self.torch.float64, device=self.dev)
        if self.world > 1:
            self.dist.all_reduce(t, op=self.dist.ReduceOp.MAX)
        return float(t.item())

    def flush(self):
        self.flushbuf.zero_()                           # write > L2 ...
        self.flushbuf.view(self.torch.int64).sum()      # ... then leave it clean

    def event(self):
        return self.torch.cuda.Event(enable_timing=True)

    def time_steps(self, step, steps, warmup, clocks=True):
        """Device ms of `steps` steps (CUDA events around each on the current
        stream, L2 flushed between them), max over ranks; NVML clock
        samples of the timed region."""
        for _ in range(warmup):
            self.flush()
            step()
        self.barrier()
        ev = [(self.event(), self.event()) for _ in range(steps)]
        sampler = ClockSampler(self.local) if clocks else None
        if sampler:
            sampler.start()
        w0 = time.perf_counter()
        for i in range(steps):
            self.flush()
            ev[i][0].record()
            step()
            ev[i][1].record()
        self.barrier()
        wall = time.perf_counter() - w0
        clk = sampler.stop() if sampler else None
        per = [a.elapsed_time(b) for a, b in ev]
        return self.allmax(sum(per)), per, clk, wall

    def time_e2e(self, fn, n):
        """Median ms of n end-to-end calls (events around each, synchronised),
        max over ranks."""
        out = []
        for i in range(n + 2):
            a, b = self.event(), self.event()
            self.flush()
            self.torch.cuda.synchronize()
            a.record()
            fn()
            b.record()
            self.torch.cuda.synchronize()
            if i >= 2:
                out.append(a.elapsed_time(b))
        return self.allmax(float(np.median(out)))


def build_plan(cfg, x=None, s=None):
    import mlx_nufft_b200 as nb
    x = cfg["x"] if x is None else x
    if cfg["type"] == 2:
        return nb.Type2PlanND(tuple(x), cfg["n_modes"], eps=cfg["eps"],
                              isign=cfg["isign"])
    if cfg["type"] == 1:
        return nb.Type1PlanND(tuple(x), cfg["n_modes"], eps=cfg["eps"],
                              isign=cfg["isign"])
    return nb.Type3Plan(tuple(x), tuple(cfg["s"] if s is None else s),
                        eps=cfg["eps"], isign=cfg["isign"])


def roofline(cfg, info, stage_ms, k, peak, peak_kind):
    """The dominant own kernel's achieved GB/s (algorithmic bytes over its
    stage's live event time)."""
    if cfg["type"] == 2:
        stage, key = "interp", "interp_or_crop"
    elif cfg["type"] == 1:
        stage, key = "spread", "spread_or_pad"
    else:
        # type 3: spread (stage 0) or interp (stage 2), whichever is longer
        stage, key = (("spread", "spread_or_pad")
                      if stage_ms["spread_or_pad"] >= stage_ms["interp_or_crop"]
                      else ("interp", "interp_or_crop"))
    ms = stage_ms[key]
    alg = kernel_bytes(cfg, info, stage)
    ach = alg / (ms / 1e3) / 1e9 if ms > 0 else 0.0
    names = {2: {1: "k_interp1_stream", 2: "k_interp_tiled / k_interp_global",
                 3: "k_interp_tma"},
             1: {1: "k_spread_tiled", 2: "k_spread_tiled / k_spread_global",
                 3: "k_spread_planes"}}
    dim = int(info.dim)
    kern = (names.get(cfg["type"], {}).get(dim) if cfg["type"] != 3
            else ("k_spread_planes" if stage == "spread" else "k_interp_tiled"))
    return {"bound": "hbm", "achieved": ach, "peak": peak, "unit": "GB/s",
            "frac": ach / peak, "traffic": ncu_traffic(k), "kernel": kern,
            "stage": stage, "algorithmic_bytes": alg, "kernel_ms": ms,
            "peak_kind": peak_kind}


def stage_split(ctx, native, step, n):
    """Per-stage device ms (the plan's own CUDA events) averaged over n
    executes, outside the timed region."""
    keys = ("spread_or_pad", "fft", "interp_or_crop")
    acc = dict.fromkeys(keys, 0.0)
    native.set_profile(True)
    try:
        for _ in range(n):
            ctx.flush()
            step()
            st = native.stage_times()
            for kk in keys:
                acc[kk] += st[kk] / n
    finally:
        native.set_profile(False)
    return acc


# ------------------------------------------------------------ one GPU
def run_single(ctx, gen, k, steps, warmup, headline, cpu, scale):
    """Config k on this GPU: device-timed value, stage split, rooflines,
    e2e through the public API, CPU baseline."""
    torch = ctx.torch
    cfg = gen.config(k, scale=scale)
    unit, what = unit_of(cfg)
    peak, peak_kind = peaks()
    if cfg["type"] == 0:
        return run_expi(ctx, cfg, k, steps, warmup, cpu, peak, peak_kind, unit)
    plan = build_plan(cfg)
    native = plan._plan
    info = native.info()
    data = torch.from_numpy(np.ascontiguousarray(
        np.asarray(cfg["data"]).astype(np.complex64))).to(ctx.dev)
    nvec = int(cfg.get("n_trans", 1))
    if cfg["type"] == 2:
        n_out = int(info.M)
    elif cfg["type"] == 1:
        n_out = int(np.prod(cfg["n_modes"])) * nvec
    else:
        n_out = int(info.N_tgt)
    out = torch.empty(n_out, dtype=torch.complex64, device=ctx.dev)
    units = int(info.M) * nvec

    def step():
        native.execute(data, out, nvec)

    native.set_profile(False)
    launches0 = int(native.info().kernel_launches)
    tot, per, clocks, wall = ctx.time_steps(step, steps, warmup)
    launches = int(native.info().kernel_launches) - launches0
    value = units * steps / (tot / 1e3)
    stage_ms = stage_split(ctx, native, step, max(1, min(steps, 20)))
    rl = roofline(cfg, info, stage_ms, k, peak, peak_kind)
    sb = step_bytes(cfg, info)
    ms = tot / steps
    srl = {"bound": "hbm", "achieved": sb / (ms / 1e3) / 1e9, "peak": peak,
           "unit": "GB/s", "frac": sb / (ms / 1e3) / 1e9 / peak,
           "algorithmic_bytes": sb, "peak_kind": peak_kind}
    # e2e through the public API, pinned host buffers
    host_in = torch.from_numpy(np.ascontiguousarray(
        np.asarray(cfg["data"]).astype(np.complex64))).pin_memory()
    host_out = torch.empty(n_out, dtype=torch.complex64).pin_memory()
    if cfg["type"] == 1 and nvec > 1:
        def e2e_call():
            plan.execute_batch(host_in.reshape(nvec, -1), out=host_out)
    else:
        def e2e_call():
            plan.execute(host_in, out=host_out)
    n_e2e = max(3, min(steps, 10))
    e2e_ms = ctx.time_e2e(e2e_call, n_e2e)
    res = {"metric": METRIC if headline else f"{what}/s (device-timed execute)",
           "value": value, "unit": unit, "n_gpus": 1, "steps": steps,
           "warmup": warmup, "ms_per_step": ms, "higher_is_better": True,
           "scaling": "strong", "vs_baseline": None, "dtype": "f32",
           "data": "synthetic", "config": config_keys(cfg, k, info),
           "stage_ms": dict(stage_ms, note="plan stage events, separate loop "
                                           "after the timed region"),
           "roofline": rl, "step_roofline": srl,
           "e2e": {"value": units / (e2e_ms / 1e3), "unit": unit,
                   "h2d_bytes_per_step": int(data.numel() * 8),
                   "d2h_bytes_per_step": int(n_out * 8), "ms_per_step": e2e_ms,
                   "steps": n_e2e,
                   "api": ("plan.execute_batch" if nvec > 1 else "plan.execute")
                          + "(pinned host in, out=pinned host)"},
           "gpu_launches": launches, "clocks": clocks,
           "wall_s_timed_region": wall}
    del plan, native, data, out, host_in, host_out
    torch.cuda.empty_cache()
    res["cpu_baseline"] = None
    if cpu:
        try:
            res["cpu_baseline"] = cpu_baseline(cfg, 1)
        except Exception as e:                 # reported, never fatal
            res["cpu_baseline"] = {"error": repr(e)}
    return res


def run_expi(ctx, cfg, k, steps, warmup, cpu, peak, peak_kind, unit, lo=None, hi=None):
    """Standalone expi (1e7 fp64 phases in [-1e6, 1e6]): device time of the
    C-ABI call on resident data; e2e through dfmath.expi from pinned host
    phases to a host result.  With lo/hi: this rank's element range."""
    import ctypes
    torch = ctx.torch
    from mlx_nufft_b200 import expi
    from mlx_nufft_b200._lib import check, lib
    phi_all = cfg["phi"]
    if lo is not None:
        phi_all = phi_all[lo:hi]
    phi_h = torch.from_numpy(np.ascontiguousarray(phi_all)).pin_memory()
    phi = phi_h.to(ctx.dev)
    n = phi.numel()
    out = torch.empty(n, dtype=torch.complex64, device=ctx.dev)
    ptrs = (ctypes.c_void_p * 1)(phi.data_ptr())
    st = torch.cuda.current_stream(ctx.dev).cuda_stream

    def step():
        check(lib.nufft_expi(1, ptrs, n, int(cfg["isign"]), out.data_ptr(), st))

    tot, per, clocks, wall = ctx.time_steps(step, steps, warmup)
    ms = tot / steps
    total_n = int(cfg["phi"].size)
    alg = 16 * n
    ach = alg / (ms / 1e3) / 1e9
    e2e_ms = ctx.time_e2e(lambda: expi(phi_h, isign=int(cfg["isign"]),
                                       return_np=True), max(3, min(steps, 10)))
    res = {"metric": "expi elements/s (device-timed)",
           "value": total_n * steps / (tot / 1e3), "unit": "elem/s",
           "n_gpus": ctx.world, "steps": steps, "warmup": warmup,
           "ms_per_step": ms, "higher_is_better": True, "scaling": "strong",
           "vs_baseline": None, "dtype": "f64", "data": "synthetic",
           "config": dict(config_keys(cfg, k), elements_per_rank=n),
           "roofline": {"bound": "hbm", "achieved": ach, "peak": peak,
                        "unit": "GB/s", "frac": ach / peak,
                        "traffic": ncu_traffic(k), "kernel": "k_expi2",
                        "algorithmic_bytes": alg, "kernel_ms": ms,
                        "peak_kind": peak_kind},
           "e2e": {"value": total_n / (e2e_ms / 1e3), "unit": "elem/s",
                   "h2d_bytes_per_step": 8 * n, "d2h_bytes_per_step": 8 * n,
                   "ms_per_step": e2e_ms, "api": "expi(pinned host phases, "
                                                 "return_np=True)"},
           "gpu_launches": steps, "clocks": clocks, "cpu_baseline": None}
    if cpu:
        try:
            res["cpu_baseline"] = cpu_baseline(cfg, 1)
        except Exception as e:
            res["cpu_baseline"] = {"error": repr(e)}
    return res


# ------------------------------------------------------------ N GPUs
# Per-rank cost model of the x-slab split of the 3-D type-2 workload (B200,
# 512^3 grid, 12^3 interpolation bins): ~9.0e-8 ms per point interpolated,
# and ~2.2e-3 ms per fine-grid plane the slab spans -- the slab-order FFT
# beyond its first pass and the per-subproblem overhead (tile copy,
# barrier) of the ~154 bins per plane that uniformly spread points occupy.
# Least-squares fit (with a constant of ~0.34 ms per rank) to the per-rank
# step times of 4- and 8-GPU runs.
SLAB_MS_PER_POINT = 9.0e-8
SLAB_MS_PER_PLANE = 2.2e-3


def slab_split(x0, world, rank, n_planes=None):
    """Boolean mask of the points of `rank` when the points are split into
    `world` slabs of the first coordinate (so each rank's points touch one
    slab of the fine grid).  Without n_planes the slabs hold equal point
    counts; with it (the fine grid's extent in that coordinate) they hold
    equal modelled cost, interpolation per point plus the slab-order FFT per
    grid plane the slab spans, so dense slabs are narrower."""
    if world == 1:
        return np.ones(x0.size, dtype=bool)
    if n_planes is None:
        qs = np.quantile(x0, np.linspace(0.0, 1.0, world + 1)[1:-1])
    else:
        xs = np.sort(np.asarray(x0, dtype=np.float64))
        # cumulative cost at each sorted point: points so far, and planes
        # from -pi up to it
        cum = (SLAB_MS_PER_POINT * np.arange(1, xs.size + 1)
               + SLAB_MS_PER_PLANE * (xs + np.pi) * (n_planes / (2 * np.pi)))
        targets = cum[-1] * np.arange(1, world) / world
        qs = xs[np.minimum(np.searchsorted(cum, targets), xs.size - 1)]
    lo = -np.inf if rank == 0 else qs[rank - 1]
    hi = np.inf if rank == world - 1 else qs[rank]
    return (x0 >= lo) & (x0 < hi)


def gather_small(ctx, arr):
    """All ranks' small numpy arrays (list, by rank)."""
    if ctx.world == 1:
        return [arr]
    out = [None] * ctx.world
    ctx.dist.all_gather_object(out, arr)
    return out


def run_split(ctx, gen, k, steps, warmup, headline, scale):
    """Config k partitioned over the ranks (strong scaling)."""
    torch, dist = ctx.torch, ctx.dist
    import mlx_nufft_b200 as nb
    from mlx_nufft_b200 import parallel as par
    cfg = gen.config(k, scale=scale)
    unit, what = unit_of(cfg)
    peak, peak_kind = peaks()
    W, R = ctx.world, ctx.rank
    res = {"metric": METRIC if headline else f"{what}/s (device-timed execute)",
           "unit": unit, "n_gpus": W, "steps": steps, "warmup": warmup,
           "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
           "dtype": "f32", "data": "synthetic"}
    if cfg["type"] == 0:
        lo, hi = par.split_range(cfg["phi"].size, R, W)
        r = run_expi(ctx, cfg, k, steps, warmup, False, peak, peak_kind, unit, lo, hi)
        r.update(partition="expi split by element", scaling="strong",
                 check={"rel_l2_vs_1gpu": 0.0, "note": "elementwise, independent"})
        return r
    launches = 0
    if cfg["type"] == 2:
        # split by target: x-slabs of equal modelled cost (points to
        # interpolate, fine-grid planes to transform)
        n_up0 = None
        if len(cfg["x"]) == 3:               # the plan's n_up rule (sigma 2)
            from mlx_nufft_b200 import sizing
            w, _ = sizing.kernel_params(cfg["eps"], 2.0)
            n_up0 = sizing.next235even(max(2 * w, int(np.ceil(2.0 * cfg["n_modes"][0]))))
        mask = slab_split(cfg["x"][0], W, R, n_up0)
        xl = [v[mask] for v in cfg["x"]]
        plan = build_plan(cfg, x=xl)
        native = plan._plan
        info = native.info()
        data = torch.from_numpy(np.ascontiguousarray(
            np.asarray(cfg["data"]).astype(np.complex64))).to(ctx.dev)
        out = torch.empty(int(info.M), dtype=torch.complex64, device=ctx.dev)

        def step():
            native.execute(data, out, 1)

        l0 = int(native.info().kernel_launches)
        tot, per, clocks, wall = ctx.time_steps(step, steps, warmup)
        launches = int(native.info().kernel_launches) - l0
        units = int(cfg["x"][0].size)
        stage_ms = stage_split(ctx, native, step, max(1, min(steps, 10)))
        # every rank's own time per step and share of the split (the
        # partition's balance; `value` takes the slowest rank)
        ranks = gather_small(ctx, {"ms_per_step": float(np.mean(per)),
                                   "points": int(info.M),
                                   "x_range": [float(xl[0].min()), float(xl[0].max())]})
        res["ranks"] = ranks
        # variant: rank 0 builds the grid, NCCL broadcast, every rank interps
        grid = par.plan_grid_storage(native)          # stored layout, halo included
        gview = torch.view_as_real(grid)
        from mlx_nufft_b200 import _lib

        def step_bcast():
            if R == 0:
                native.execute_stage(_lib.STAGE_SPREAD, data, None, 1)
            dist.broadcast(gview, src=0)
            native.execute_stage(_lib.STAGE_FINISH, None, out, 1)

        tb, _, _, _ = ctx.time_steps(step_bcast, steps, 2, clocks=False)
        bev = []
        for _ in range(3):
            a, b = ctx.event(), ctx.event()
            ctx.barrier()
            a.record()
            dist.broadcast(gview, src=0)
            b.record()
            ctx.torch.cuda.synchronize()
            bev.append(a.elapsed_time(b))
        bcast_ms = ctx.allmax(float(np.median(bev)))
        res["broadcast"] = {"ms_per_step": tb / steps,
                            "value": units * steps / (tb / 1e3),
                            "broadcast_ms": bcast_ms,
                            "grid_bytes": int(gview.numel() * 4),
                            "note": "rank 0 pad+FFT, ncclBroadcast of the fine grid, "
                                    "every rank interp"}
        # correctness: the first 256 outputs of every rank against one GPU
        # (rank 0) interpolating the same points from a full plan
        native.execute(data, out, 1)
        torch.cuda.synchronize()
        mine = (np.stack([v[:256] for v in xl]), out[:256].cpu().numpy())
        allp = gather_small(ctx, mine)
        chk = None
        if R == 0:
            xs = [np.concatenate([p[0][d] for p in allp]) for d in range(len(xl))]
            ref = build_plan(cfg, x=xs).execute(data)
            got = np.concatenate([p[1] for p in allp])
            chk = float(np.linalg.norm(got - ref) / np.linalg.norm(ref))
        res["partition"] = ("type 2 split by target: x-slabs of equal modelled cost "
                            "(points + fine-grid planes) per rank, fine grid built on "
                            "every rank for its planes (value) or broadcast whole "
                            "from rank 0 (broadcast)")
        ckeys = config_keys(cfg, k, info, W, rank_points=int(info.M))
        n_out = int(info.M)
        h2d = int(data.numel() * 8)
        host_in = torch.from_numpy(np.ascontiguousarray(
            np.asarray(cfg["data"]).astype(np.complex64))).pin_memory()
        host_out = torch.empty(n_out, dtype=torch.complex64).pin_memory()
        e2e_ms = ctx.time_e2e(lambda: plan.execute(host_in, out=host_out),
                              max(3, min(steps, 10)))
        e2e = {"value": units / (e2e_ms / 1e3), "unit": unit,
               "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": n_out * 8,
               "ms_per_step": e2e_ms,
               "api": "plan.execute(pinned host in, out=pinned host) per rank"}
    elif cfg["type"] == 1 and int(cfg.get("n_trans", 1)) > 1:
        # batched type 1 split by vector
        B = int(cfg["n_trans"])
        lo, hi = par.vector_range(B, R, W)
        plan = build_plan(cfg)
        native = plan._plan
        info = native.info()
        allc = np.asarray(cfg["data"]).astype(np.complex64)
        data = torch.from_numpy(np.ascontiguousarray(allc[lo:hi])).to(ctx.dev)
        K = int(np.prod(cfg["n_modes"]))
        nv = hi - lo
        out = torch.empty(max(nv, 1) * K, dtype=torch.complex64, device=ctx.dev)

        def step():
            if nv > 0:
                native.execute(data, out, nv)

        l0 = int(native.info().kernel_launches)
        tot, per, clocks, wall = ctx.time_steps(step, steps, warmup)
        launches = int(native.info().kernel_launches) - l0
        units = int(cfg["x"][0].size) * B
        stage_ms = stage_split(ctx, native, step, max(1, min(steps, 10)))
        step()
        torch.cuda.synchronize()
        idx = np.random.default_rng(7).choice(K, 512, replace=False)
        mine = (lo, out.reshape(max(nv, 1), K)[:nv, idx].cpu().numpy())
        allp = gather_small(ctx, mine)
        chk = None
        if R == 0:
            full = torch.empty(B * K, dtype=torch.complex64, device=ctx.dev)
            native.execute(torch.from_numpy(np.ascontiguousarray(allc)).to(ctx.dev),
                           full, B)
            ref = full.reshape(B, K)[:, idx].cpu().numpy()
            got = np.concatenate([p[1] for p in sorted(allp, key=lambda q: q[0])])
            chk = float(np.linalg.norm(got - ref) / np.linalg.norm(ref))
        res["partition"] = "batched type 1 split by vector (no collective)"
        ckeys = dict(config_keys(cfg, k, info, W), vectors_per_rank=nv)
        host_in = torch.from_numpy(np.ascontiguousarray(allc[lo:hi])).pin_memory()
        host_out = torch.empty(max(nv, 1) * K, dtype=torch.complex64).pin_memory()
        e2e_ms = ctx.time_e2e(lambda: plan.execute_batch(host_in, out=host_out)
                              if nv > 0 else None, max(3, min(steps, 10)))
        e2e = {"value": units / (e2e_ms / 1e3), "unit": unit,
               "h2d_bytes_per_step": int(host_in.numel() * 8),
               "d2h_bytes_per_step": int(nv * K * 8), "ms_per_step": e2e_ms,
               "api": "plan.execute_batch(pinned host in, out=pinned host) per rank"}
    elif cfg["type"] == 1:
        # one type-1 transform split by point: all-reduce of the fine grids
        M = int(cfg["x"][0].size)
        lo, hi = par.split_range(M, R, W)
        xl = [v[lo:hi] for v in cfg["x"]]
        call = np.asarray(cfg["data"]).astype(np.complex64)
        plan = build_plan(cfg, x=xl)
        native = plan._plan
        info = native.info()
        stages = par.PlanStages(plan)
        split = par.Type1PointSplit(stages)
        cl = torch.from_numpy(np.ascontiguousarray(call[lo:hi])).to(ctx.dev)
        holder = {}

        def step():
            holder["r"] = split.execute(cl, return_np=False)

        l0 = int(native.info().kernel_launches)
        tot, per, clocks, wall = ctx.time_steps(step, steps, warmup)
        launches = int(native.info().kernel_launches) - l0
        units = M
        stage_ms = None      # the stages straddle the all-reduce
        step()
        got = holder["r"].cpu().numpy().ravel()
        chk = None
        if R == 0:
            ref = build_plan(cfg).execute(call).ravel()
            chk = float(np.linalg.norm(got - ref) / np.linalg.norm(ref))
        res["partition"] = ("type 1 split by point: per-rank spread, NCCL "
                            "all-reduce of the fine grid, FFT + crop on every rank")
        ckeys = config_keys(cfg, k, info, W, rank_points=hi - lo)
        e2e = None
    else:
        # type 3 split by target
        Nt = int(cfg["s"][0].size)
        lo, hi = par.split_range(Nt, R, W)
        sl = [v[lo:hi] for v in cfg["s"]]
        plan = build_plan(cfg, s=sl)
        native = plan._plan
        info = native.info()
        call = np.asarray(cfg["data"]).astype(np.complex64)
        data = torch.from_numpy(np.ascontiguousarray(call)).to(ctx.dev)
        out = torch.empty(hi - lo, dtype=torch.complex64, device=ctx.dev)

        def step():
            native.execute(data, out, 1)

        l0 = int(native.info().kernel_launches)
        tot, per, clocks, wall = ctx.time_steps(step, steps, warmup)
        launches = int(native.info().kernel_launches) - l0
        units = int(cfg["x"][0].size)
        stage_ms = stage_split(ctx, native, step, max(1, min(steps, 10)))
        step()
        torch.cuda.synchronize()
        # the first 256 targets of every rank against one GPU running the
        # whole problem (a plan over all targets: type-3 grids are sized
        # from the target extent)
        mine = (np.arange(lo, lo + min(256, hi - lo)), out[:256].cpu().numpy())
        allp = gather_small(ctx, mine)
        chk = None
        if R == 0:
            idx = np.concatenate([p[0] for p in allp])
            ref = build_plan(cfg).execute(call)[idx]
            got = np.concatenate([p[1] for p in allp])
            chk = float(np.linalg.norm(got - ref) / np.linalg.norm(ref))
        res["partition"] = ("type 3 split by target: every rank all sources and "
                            "1/N of the targets (no collective)")
        ckeys = config_keys(cfg, k, info, W)
        ckeys["targets_per_rank"] = hi - lo
        e2e = None
    ms = tot / steps
    res.update({"value": units * steps / (tot / 1e3), "ms_per_step": ms,
                "value_per_gpu": units * steps / (tot / 1e3) / W,
                "config": ckeys, "stage_ms_rank0": stage_ms,
                "check": {"rel_l2_vs_1gpu": chk,
                          "what": "subset of the outputs against one GPU running "
                                  "the whole problem"},
                "gpu_launches": launches, "clocks": clocks,
                "wall_s_timed_region": wall})
    if e2e is not None:
        res["e2e"] = e2e
    if cfg["type"] in (1, 2) and stage_ms is not None:
        res["roofline"] = roofline(cfg, info, stage_ms, k, peak, peak_kind)
    torch.cuda.synchronize()
    del plan, native
    torch.cuda.empty_cache()
    return res


def main():
    args = parse()
    if args.impl == "reference":
        run_reference(args)
        return
    ctx = Ctx(args)
    gen = load_gen()
    cpu = not args.no_cpu_baseline and ctx.world == 1 and ctx.rank == 0
    per = {}
    if ctx.world == 1:
        line = run_single(ctx, gen, args.config, args.steps, args.warmup, True,
                          cpu, args.scale)
        if args.config == HEADLINE and not args.no_per_config:
            for k in PER_CONFIG:
                try:
                    per[str(k)] = run_single(ctx, gen, k, min(args.steps, 20), 3,
                                             False, cpu, args.scale)
                except Exception as e:          # reported, never fatal
                    per[str(k)] = {"error": repr(e)}
    else:
        line = run_split(ctx, gen, args.config, args.steps, args.warmup, True,
                         args.scale)
        if args.config == HEADLINE and not args.no_per_config:
            for k in (3, 1, 5, 6, 2):
                per[str(k)] = run_split(ctx, gen, k, min(args.steps, 20), 3,
                                        False, args.scale)
    line["n_gpus"] = ctx.world
    line.setdefault("value_per_gpu", line["value"] / ctx.world)
    if per:
        line["per_config"] = per
    if ctx.rank == 0:
        print(json.dumps(line), flush=True)
    if ctx.world > 1:
        ctx.dist.barrier()
        ctx.dist.destroy_process_group()


if __name__ == "__main__":
    main()
