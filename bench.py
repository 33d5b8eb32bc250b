"""Benchmark: NU points/s of the NUFFT execute path on B200 (one JSON line).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config C]
                    [--impl reference]

Workload (default --config 2, the configuration BASELINE.json's metric is
quoted on): 1D type 2, N = 2^20 complex64 modes, M = 1e7 points uniform in
[-pi, pi), eps = 1e-6, isign = -1.  A step is one plan execute over resident
device inputs: pad/deconvolve -> cuFFT -> interp (setpts / sort excluded, the
reference's "exec" protocol).  Each step is bracketed by CUDA events on the
execute stream; L2 is flushed between steps, outside the events: a 256 MiB
write, then a read of the same buffer, so the L2 holds clean unrelated
lines (the write alone would leave ~126 MB of dirty lines whose write-back
would land inside the next timed step).  `value` = points of all ranks / max-over-ranks device time.

Other keys: `roofline` (the dominant own kernel, from the plan's live stage
events and the algorithmic bytes of the stage), `e2e` (same metric through
the public API from pinned host memory with the H2D / D2H copies timed),
`cpu_baseline` (the CPU oracle port on a bounded sample, rank 0),
`gpu_launches` (own kernels launched in the timed region), `clocks`
(NVML samples taken during the timed region).

--impl reference times the CPU port of the reference algorithm
(oracle/port.py; the reference itself has no CPU type-1/2 path and its Metal
GPU path cannot run here) with all host threads, on rank 0 only.
"""

import argparse
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
UNIT = "NU pts/s"


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=300)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--config", type=int, default=2)
    ap.add_argument("--impl", default="native", choices=["native", "reference"])
    ap.add_argument("--scale", type=float, default=1.0,
                    help="point-count scale (1.0 = the BASELINE size)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    return ap.parse_args()


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


# ---------------------------------------------------------------- clocks
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


# ---------------------------------------------------------------- traffic
def ncu_traffic(kernel_tag):
    """Per-launch DRAM bytes of the dominant kernel from the committed ncu
    summary (profiles/*.md line 'traffic_bytes_per_launch: <n>' under the
    heading for this workload); None if absent."""
    pdir = os.path.join(ROOT, "profiles")
    if not os.path.isdir(pdir):
        return None
    for f in sorted(os.listdir(pdir)):
        if not f.endswith(".md") or kernel_tag not in f:
            continue
        m = re.search(r"traffic_bytes_per_launch:\s*([0-9.eE+]+)",
                      open(os.path.join(pdir, f)).read())
        if m:
            return float(m.group(1))
    return None


# ---------------------------------------------------------------- workload
def algorithmic_bytes(cfg, info, stage):
    """Compulsory DRAM bytes of one launch of the given stage's own kernel.
    interp (type 2): per point cell (8 B/dim) + output (8 B) + permutation
    (4 B, when sorted); grid read once (8 B/cell).  pad: modes read (8 B) +
    grid written (8 B/cell).  spread (type 1): per point cell + strength
    (8 B) + permutation; grid written once per vector."""
    dim = info.dim
    M = int(info.M)
    ncell = int(np.prod([info.n_up[d] for d in range(dim)]))
    K = int(np.prod([info.n_modes[d] for d in range(dim)]))
    perm = 4 if info.tiled or info.nsub > 0 else 0
    if stage == "interp":
        return M * (8 * dim + 8 + perm) + ncell * 8
    if stage == "pad":
        return K * 8 + ncell * 8
    if stage == "spread":
        return M * (8 * dim + 8 + perm) + ncell * 8
    raise ValueError(stage)


def build_plan(cfg, torch):
    import mlx_nufft_b200 as nb
    if cfg["type"] == 2:
        plan = nb.Type2PlanND(tuple(cfg["x"]), cfg["n_modes"], eps=cfg["eps"],
                              isign=cfg["isign"])
    elif cfg["type"] == 1:
        plan = nb.Type1PlanND(tuple(cfg["x"]), cfg["n_modes"], eps=cfg["eps"],
                              isign=cfg["isign"])
    else:
        plan = nb.Type3Plan(tuple(cfg["x"]), tuple(cfg["s"]), eps=cfg["eps"],
                            isign=cfg["isign"])
    return plan


class CpuPort:
    """The CPU oracle port of the reference algorithm (oracle/port.py, fp64)
    on the same type-2 workload: deconvolve + pad + FFT of the full grid,
    then fold + interp of a sample of the points on `threads` threads.
    Plan-time work (deconvolution factors) is done once in the constructor,
    as the reference's exec protocol excludes it."""

    def __init__(self, cfg, threads):
        from oracle import port
        if cfg["type"] != 2:
            raise NotImplementedError("CPU baseline implemented for type-2 "
                                      "configs")
        self.port = port
        self.cfg = cfg
        self.threads = threads
        self.x = cfg["x"]
        self.M = self.x[0].size
        self.dim = len(self.x)
        self.f = np.asarray(cfg["data"], dtype=np.complex128)
        N = self.f.shape
        self.w, self.beta, self.nup = port.fine_grid_sizes(N, cfg["eps"])
        self.decs = []
        for d in range(self.dim):
            k = np.arange(-(N[d] // 2), N[d] - N[d] // 2, dtype=np.float64)
            self.decs.append(1.0 / port.kernel_ft(2.0 * np.pi * k / self.nup[d],
                                                  self.beta, self.w))

    def step(self, sample):
        """One pass: full grid work + interp of the first `sample` points.
        Returns (grid seconds, point seconds)."""
        from concurrent.futures import ThreadPoolExecutor
        port, dim, N = self.port, self.dim, self.f.shape
        t0 = time.perf_counter()
        g = self.f.copy()
        for d in range(dim):
            g = g * self.decs[d].reshape((1,) * d + (-1,) + (1,) * (dim - d - 1))
        H = np.zeros(self.nup, dtype=np.complex128)
        H[np.ix_(*[port._band(N[d], self.nup[d]) for d in range(dim)])] = g
        V = port._fft(H, self.cfg["isign"])
        t_grid = time.perf_counter() - t0

        def work(ix):
            i1s, frs = [], []
            for d in range(dim):
                i1, fr64, _ = port.cells_fold(self.x[d][ix], self.nup[d], self.w)
                i1s.append(i1)
                frs.append(fr64)
            return port.interp(V, i1s, frs, self.w, self.beta, chunk=65536)

        parts = [p for p in np.array_split(np.arange(sample), 4 * self.threads)
                 if p.size]
        t1 = time.perf_counter()
        with ThreadPoolExecutor(self.threads) as ex:
            list(ex.map(work, parts))
        return t_grid, time.perf_counter() - t1

    def rate(self, t_grid, t_pts, sample):
        """Points/s of the full workload from one step's times."""
        return self.M / (t_grid + t_pts * (self.M / sample))

    def describe(self, t_grid, t_pts, sample):
        return (f"oracle/port.py fp64 on {self.threads} thread(s): "
                f"deconvolve+pad+FFT of the full grid ({t_grid:.3f} s) + "
                f"fold+interp of {sample} of {self.M} points ({t_pts:.3f} s)"
                + ("" if sample == self.M else ", extrapolated to all points"))


def cpu_baseline(cfg, threads):
    """One single-threaded pass of the CPU port over the whole workload."""
    cp = CpuPort(cfg, threads)
    sample = cp.M
    tg, tp = cp.step(sample)
    return {"value": cp.rate(tg, tp, sample), "unit": UNIT, "cores": threads,
            "kind": "port", "sample": cp.describe(tg, tp, sample)}


def run_reference(args, budget_s=150.0):
    """--impl reference: the CPU port with all host threads, rank 0 only.
    The first warm-up step calibrates the point rate; every step then
    interpolates a sample sized so the whole run stays near `budget_s`."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    from mlx_nufft_b200 import gen
    cfg = gen.config(args.config, scale=args.scale)
    threads = os.cpu_count() or 1
    cp = CpuPort(cfg, threads)
    probe = min(cp.M, 200_000)
    tg, tp = cp.step(probe)
    per_step = budget_s / max(1, args.warmup + args.steps)
    pts_rate = probe / max(tp, 1e-9)
    sample = int(min(cp.M, max(20_000, (per_step - tg) * pts_rate)))
    vals, last = [], None
    for i in range(args.warmup + args.steps):
        tg, tp = cp.step(sample)
        if i >= args.warmup:
            vals.append(cp.rate(tg, tp, sample))
            last = (tg, tp)
    v = float(np.median(vals))
    line = {"impl": "reference", "metric": METRIC, "value": v, "unit": UNIT,
            "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": cp.M / v * 1e3,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "f64", "data": "synthetic",
            "config": {"workload": cfg["name"], "config": args.config},
            "cpu_baseline": {"value": v, "unit": UNIT, "cores": threads,
                             "kind": "port",
                             "sample": cp.describe(*last, sample) + " (per step)"},
            "e2e": {"value": v, "unit": UNIT, "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def run_expi(args, cfg, torch, dist, world, rank, local, barrier):
    """--config 6: the standalone expi of BASELINE cfg 5 (1e7 fp64 phases
    in [-1e6, 1e6]); metric elements/s.  Device time: CUDA events around
    the C-ABI call on resident data; e2e: dfmath.expi from pinned host
    phases to a host result."""
    import ctypes
    from mlx_nufft_b200 import expi
    from mlx_nufft_b200._lib import check, lib
    dev = torch.device("cuda", local)
    phi_h = torch.from_numpy(np.ascontiguousarray(cfg["phi"])).pin_memory()
    phi = phi_h.to(dev)
    n = phi.numel()
    out = torch.empty(n, dtype=torch.complex64, device=dev)
    ptrs = (ctypes.c_void_p * 1)(phi.data_ptr())
    flush = torch.empty(256 * 2 ** 20, dtype=torch.uint8, device=dev)
    st = torch.cuda.current_stream(dev).cuda_stream

    def step():
        check(lib.nufft_expi(1, ptrs, n, int(cfg["isign"]), out.data_ptr(), st))

    for _ in range(args.warmup):
        step()
    barrier()
    sampler = ClockSampler(local)
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
          for _ in range(args.steps)]
    sampler.start()
    for i in range(args.steps):
        flush.zero_()
        flush.view(torch.int64).sum()
        ev[i][0].record()
        step()
        ev[i][1].record()
    barrier()
    clocks = sampler.stop()
    ms = sum(a.elapsed_time(b) for a, b in ev)
    t = torch.tensor([ms], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    tmax = float(t.item())
    value = world * n * args.steps / (tmax / 1e3)
    e2e = []
    for i in range(max(3, min(args.steps, 20)) + 2):
        a = torch.cuda.Event(enable_timing=True)
        b = torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        a.record()
        expi(phi_h, isign=int(cfg["isign"]), return_np=True)
        b.record()
        torch.cuda.synchronize()
        if i >= 2:
            e2e.append(a.elapsed_time(b))
    e2e_t = torch.tensor([float(np.median(e2e))], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(e2e_t, op=dist.ReduceOp.MAX)
    peak, peak_kind = peaks()
    kern_ms = tmax / args.steps
    alg = 16 * n
    if rank == 0:
        print(json.dumps({
            "metric": "expi elements/sec per GPU (device-timed)", "value": value,
            "unit": "elem/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": kern_ms,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "f64", "data": "synthetic",
            "config": {"workload": cfg["name"], "config": args.config,
                       "elements_per_rank": n,
                       "l2": "flushed between steps (256 MiB write, then read)"},
            "roofline": {"bound": "hbm", "achieved": alg / (kern_ms / 1e3) / 1e9,
                         "peak": peak, "unit": "GB/s",
                         "frac": alg / (kern_ms / 1e3) / 1e9 / peak,
                         "traffic": ncu_traffic(f"cfg{args.config}"),
                         "kernel": "k_expi2",
                         "algorithmic_bytes": alg, "peak_kind": peak_kind},
            "e2e": {"value": world * n / (float(e2e_t.item()) / 1e3), "unit": "elem/s",
                    "h2d_bytes_per_step": 8 * n, "d2h_bytes_per_step": 8 * n,
                    "ms_per_step": float(e2e_t.item())},
            "gpu_launches": args.steps, "clocks": clocks, "cpu_baseline": None,
        }), flush=True)


def main():
    args = parse()
    if args.impl == "reference":
        run_reference(args)
        return
    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if world > 1:
        from datetime import timedelta
        # NCCL may print its version banner on file descriptor 1 while the
        # communicator is set up; send that to stderr so that rank 0's
        # stdout carries only the JSON line
        sys.stdout.flush()
        saved_fd = os.dup(1)
        os.dup2(2, 1)
        try:
            dist.init_process_group("nccl", timeout=timedelta(seconds=300),
                                    device_id=torch.device("cuda", local))
            dist.barrier()
            torch.cuda.synchronize()
        finally:
            sys.stdout.flush()
            os.dup2(saved_fd, 1)
            os.close(saved_fd)

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    from mlx_nufft_b200 import gen
    # weak scaling: every rank owns its own point set (seed = rank)
    cfg = gen.config(args.config, scale=args.scale, seed=rank)
    if cfg["type"] == 0:
        run_expi(args, cfg, torch, dist, world, rank, local, barrier)
        if world > 1:
            dist.barrier()
            dist.destroy_process_group()
        return
    plan = build_plan(cfg, torch)
    native = plan._plan
    info = native.info()
    dev = torch.device("cuda", local)
    data = torch.from_numpy(np.ascontiguousarray(
        np.asarray(cfg["data"]).astype(np.complex64))).to(dev)
    ndata = data.numel()
    if cfg["type"] == 2:
        n_out, nvec = int(info.M), 1
        stage_own = "interp"
    elif cfg["type"] == 1:
        nvec = int(cfg.get("n_trans", 1))
        n_out = int(np.prod(cfg["n_modes"])) * nvec
        stage_own = "spread"
    else:
        n_out, nvec = int(info.N_tgt), 1
        stage_own = "interp"
    out = torch.empty(n_out, dtype=torch.complex64, device=dev)
    flush = torch.empty(256 * 2 ** 20, dtype=torch.uint8, device=dev)

    def flush_l2():
        flush.zero_()                              # write > L2 ...
        flush.view(torch.int64).sum()              # ... then leave it clean
    npts = int(info.M) * nvec

    def step():
        native.execute(data, out, nvec)

    # The timed steps run without the plan's per-stage events (they would
    # sit between the kernels); the stage split comes from a separate
    # profiled loop after the timed region.
    native.set_profile(False)
    for _ in range(args.warmup):
        flush_l2()
        step()
    barrier()
    ev = [(torch.cuda.Event(enable_timing=True),
           torch.cuda.Event(enable_timing=True)) for _ in range(args.steps)]
    sampler = ClockSampler(local)
    launches0 = int(native.info().kernel_launches)
    barrier()
    sampler.start()
    w0 = time.perf_counter()
    for i in range(args.steps):
        flush_l2()
        ev[i][0].record()
        step()
        ev[i][1].record()
    barrier()
    wall = time.perf_counter() - w0
    clocks = sampler.stop()
    launches = int(native.info().kernel_launches) - launches0
    dev_ms = sum(a.elapsed_time(b) for a, b in ev)
    # per-stage device times (plan events), outside the timed region
    n_prof = max(1, min(args.steps, 50))
    stage_ms = {"spread_or_pad": 0.0, "fft": 0.0, "interp_or_crop": 0.0}
    native.set_profile(True)
    for _ in range(n_prof):
        flush_l2()
        step()
        st = native.stage_times()
        for k in stage_ms:
            stage_ms[k] += st[k] / n_prof
    native.set_profile(False)
    t = torch.tensor([dev_ms], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    tmax_ms = float(t.item())
    value = world * npts * args.steps / (tmax_ms / 1e3)

    # ---- e2e through the public API, pinned host buffers -----------------
    # Each step: H2D copy of the step's input from pinned memory, execute,
    # D2H copy of the result into a pinned host array, all inside the events.
    host_in = torch.from_numpy(np.ascontiguousarray(
        np.asarray(cfg["data"]).astype(np.complex64))).pin_memory()
    host_out = torch.empty(n_out, dtype=torch.complex64).pin_memory()
    e2e_ms = []
    n_e2e = max(3, min(args.steps, 30))
    for i in range(n_e2e + 2):
        a = torch.cuda.Event(enable_timing=True)
        b = torch.cuda.Event(enable_timing=True)
        flush_l2()
        torch.cuda.synchronize()
        a.record()
        if cfg["type"] == 1 and nvec > 1:
            plan.execute_batch(host_in.reshape(nvec, -1), out=host_out)
        else:
            plan.execute(host_in, out=host_out)
        b.record()
        torch.cuda.synchronize()
        if i >= 2:
            e2e_ms.append(a.elapsed_time(b))
    e2e_t = torch.tensor([float(np.median(e2e_ms))], dtype=torch.float64,
                         device=dev)
    if world > 1:
        dist.all_reduce(e2e_t, op=dist.ReduceOp.MAX)
    e2e_val = world * npts / (float(e2e_t.item()) / 1e3)

    # ---- roofline of the dominant own kernel ------------------------------
    peak, peak_kind = peaks()
    key = "interp_or_crop" if stage_own == "interp" else "spread_or_pad"
    kern_ms = stage_ms[key]
    alg = algorithmic_bytes(cfg, info, stage_own)
    achieved = alg / (kern_ms / 1e3) / 1e9
    traffic = ncu_traffic(f"cfg{args.config}")

    if rank == 0:
        cpu = None
        if not args.no_cpu_baseline and world == 1 and cfg["type"] == 2:
            try:
                cpu = cpu_baseline(cfg, 1)
            except Exception as e:          # reported, never fatal
                cpu = {"error": str(e)}
        line = {
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": tmax_ms / args.steps, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic",
            "config": {"workload": cfg["name"], "config": args.config,
                       "points_per_rank": int(info.M), "vectors": nvec,
                       "eps": cfg["eps"], "isign": cfg["isign"],
                       "w": int(info.w),
                       "n_up": [int(info.n_up[d]) for d in range(info.dim)],
                       "tiled": bool(info.tiled),
                       "l2": "flushed between steps (256 MiB write, then read)",
                       "wall_s_timed_region": wall},
            "stage_ms": dict(stage_ms, steps=n_prof,
                             note="plan stage events, separate loop after the timed region"),
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak,
                         "unit": "GB/s", "frac": achieved / peak,
                         "traffic": traffic, "kernel": stage_own,
                         "algorithmic_bytes": alg, "kernel_ms": kern_ms,
                         "peak_kind": peak_kind},
            "e2e": {"value": e2e_val, "unit": UNIT,
                    "h2d_bytes_per_step": int(ndata * 8),
                    "d2h_bytes_per_step": int(n_out * 8),
                    "ms_per_step": float(e2e_t.item()), "steps": n_e2e,
                    "api": "plan.execute(pinned host in, out=pinned host)"},
            "gpu_launches": launches,
            "clocks": clocks,
            "cpu_baseline": cpu,
        }
        print(json.dumps(line), flush=True)
    del plan, native
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
