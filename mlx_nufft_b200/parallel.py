"""Multi-GPU execution within one box: one process per GPU, torch.distributed
for the plumbing (NCCL over NVLink on the GPUs; the same code runs over gloo
in the CPU tests).

Only the partitions the transforms have naturally are provided:

* batched transforms split by vector -- each rank runs its own slice of the
  n_trans vectors through one plan over the shared points; no collective
  during execute (`vector_range`, `ShardedBatch`);
* type 2 split by target point -- every rank interpolates its own points
  from the same fine grid, which every rank computes from its copy of the
  modes (replicate, no collective) or one rank computes (pad/deconvolve +
  FFT) and broadcasts (`Type2TargetSplit`);
* type 1 split by point -- every rank spreads its own points onto a full
  fine grid, the grids are summed with one all-reduce, and every rank (or
  one root) finishes with FFT + deconvolution (`Type1PointSplit`);
* type 3 split by target point -- sources replicated, each rank a plan over
  its targets (`Type3TargetSplit`).

The reference is single-GPU; its closest counterparts are the batched
execute (mlx_nufft/nd.py:744-794, gpu_t3.py:941-1041) and the stage order of
Type1PlanND.execute / Type2PlanND.execute (nd.py:581-625, 1075-1119).

The split classes drive a small "stages" interface -- `first(data)` runs the
first stage and returns the fine grid as a tensor, `grid()` returns that
grid without computing it, `second()` runs the second stage and returns the
result -- implemented here over the native plans' staged execute
(nufft_execute_stage + nufft_get_grid).  Tests substitute a CPU
implementation to run the same orchestration on gloo ranks.
"""

import numpy as np
import torch
import torch.distributed as dist

from . import _lib
from ._device import as_c64, finish


def split_range(n, rank, world):
    """Contiguous, balanced [lo, hi) share of n items for `rank`."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside world of size {world}")
    base, extra = divmod(int(n), int(world))
    lo = rank * base + min(rank, extra)
    return lo, lo + base + (1 if rank < extra else 0)


vector_range = split_range


def _world(group):
    if not dist.is_available() or not dist.is_initialized():
        return 0, 1
    return dist.get_rank(group), dist.get_world_size(group)


def gather_rows(local, n_total, group=None):
    """All-gather per-rank row blocks (each rank holds rows [lo, hi) of a
    split_range partition of n_total along dim 0) into the full array on
    every rank.  Blocks are padded to the largest share for the collective."""
    rank, world = _world(group)
    if world == 1:
        return local
    shares = [split_range(n_total, r, world) for r in range(world)]
    width = max(hi - lo for lo, hi in shares)
    pad = torch.zeros((width,) + tuple(local.shape[1:]), dtype=local.dtype,
                      device=local.device)
    pad[: local.shape[0]] = local
    # complex tensors travel as their real view (all backends)
    send = torch.view_as_real(pad) if pad.is_complex() else pad
    bufs = [torch.empty_like(send) for _ in range(world)]
    dist.all_gather(bufs, send, group=group)
    parts = []
    for (lo, hi), b in zip(shares, bufs):
        b = torch.view_as_complex(b) if pad.is_complex() else b
        parts.append(b[: hi - lo])
    return torch.cat(parts, dim=0)


class _DeviceArray:
    """Zero-copy torch view of a device buffer owned by a native plan."""

    def __init__(self, ptr, shape, typestr):
        self.__cuda_array_interface__ = {
            "shape": tuple(int(s) for s in shape), "typestr": typestr,
            "data": (int(ptr), False), "version": 3, "strides": None}


def plan_grid_storage(native, nvec=1, fp64=False):
    """The native plan's stored fine grid(s) as a contiguous (nvec, *ext)
    complex CUDA tensor sharing its memory (nufft_get_grid; ext = the fine
    grid's extents plus the periodic halo of a 3-D type-2 grid, the fine
    grid itself otherwise): what a broadcast or reduction of the grid
    moves."""
    info = native.info()
    ptr, n = native.grid()
    cells = int(info.grid_cells)
    if nvec * cells > n:
        raise ValueError("plan grid holds fewer vectors than requested")
    ext = tuple(int(info.grid_ext[d]) for d in range(int(info.dim)))
    arr = _DeviceArray(ptr, (nvec,) + ext, "<c16" if fp64 else "<c8")
    return torch.as_tensor(arr, device=torch.device("cuda", native.device))


def plan_grid_view(native, n_up, nvec=1, fp64=False):
    """The native plan's fine grid(s) as a (nvec, *n_up) complex CUDA tensor
    sharing its memory: a strided view that skips the periodic halo of a
    3-D type-2 grid (nufft_plan_info grid_ext / grid_lo)."""
    info = native.info()
    flat = plan_grid_storage(native, nvec, fp64)
    if tuple(flat.shape[1:]) == tuple(int(v) for v in n_up):
        return flat                                    # no halo
    dim = len(n_up)
    ext = [int(info.grid_ext[d]) for d in range(dim)]
    lo = [int(info.grid_lo[d]) for d in range(dim)]
    strides, acc = [], 1
    for e in reversed(ext):
        strides.insert(0, acc)
        acc *= e
    off = sum(l * st for l, st in zip(lo, strides))
    return torch.as_strided(flat, (nvec,) + tuple(int(v) for v in n_up),
                            (int(info.grid_cells),) + tuple(strides), off)


class PlanStages:
    """Stages interface over a Type1PlanND / Type2PlanND (one vector)."""

    def __init__(self, plan):
        self.plan = plan
        self.native = plan._plan
        info = self.native.info()
        self.type = int(info.type)
        self.fp64 = bool(info.fft64)
        self.n_up = tuple(int(info.n_up[d]) for d in range(info.dim))

    def grid(self):
        return plan_grid_storage(self.native, 1, fp64=self.fp64 and self.type == 2)

    def first(self, data):
        d = as_c64(data, self.native.device).reshape(-1)
        self.native.execute_stage(_lib.STAGE_SPREAD, d, None, 1)
        return self.grid()

    def second(self):
        if self.type == 1:
            out = torch.empty(tuple(self.plan.N), dtype=torch.complex64,
                              device=torch.device("cuda", self.native.device))
        else:
            out = torch.empty(self.plan.P, dtype=torch.complex64,
                              device=torch.device("cuda", self.native.device))
        self.native.execute_stage(_lib.STAGE_FINISH, None, out, 1)
        return out


def _real(t):
    return torch.view_as_real(t) if t.is_complex() else t


class Type1PointSplit:
    """One type-1 transform whose points are split across the ranks of
    `group`: each rank spreads its own points (its `stages` object owns a
    plan over them), the fine grids are summed with one all-reduce, and each
    rank -- or only `root` -- runs FFT + deconvolution.  The sum of the
    ranks' spread grids is the single-GPU spread grid (spreading is linear),
    so the result matches one plan over all points up to float summation
    order."""

    def __init__(self, stages, group=None, root=None):
        self.stages = stages
        self.group = group
        self.root = root

    def execute(self, c_local, return_np=True):
        rank, world = _world(self.group)
        g = self.stages.first(c_local)
        if world > 1:
            if self.root is None:
                dist.all_reduce(_real(g), op=dist.ReduceOp.SUM, group=self.group)
            else:
                dist.reduce(_real(g), dst=self.root, op=dist.ReduceOp.SUM,
                            group=self.group)
        if self.root is not None and rank != self.root:
            return None
        return finish(self.stages.second(), return_np)


class Type2TargetSplit:
    """Type 2 with the target points split across the ranks of `group`;
    every rank interpolates its own points from the same fine grid.  With
    `replicate=True` every rank builds the grid (pad/deconvolve + FFT) from
    its own copy of the modes, with no collective; otherwise `root` builds
    it once and broadcasts it (modes held by one rank).  `gather=True`
    assembles the caller-order output of all points (each rank holding the
    split_range share of the global point list) on every rank."""

    def __init__(self, stages, n_points_total=None, group=None, root=0,
                 replicate=False):
        self.stages = stages
        self.group = group
        self.root = root
        self.n_total = n_points_total
        self.replicate = replicate

    def execute(self, fk, return_np=True, gather=False):
        rank, world = _world(self.group)
        if world == 1 or rank == self.root or self.replicate:
            g = self.stages.first(fk)
        else:
            g = self.stages.grid()
        if world > 1 and not self.replicate:
            dist.broadcast(_real(g), src=self.root, group=self.group)
        out = self.stages.second()
        if gather:
            out = gather_rows(out, self.n_total, self.group)
        return finish(out, return_np)


class ShardedBatch:
    """Batched transform split by vector: this rank runs vectors
    vector_range(n_trans, rank, world) of `cs` through `plan.execute_batch`
    (any plan class with execute_batch); `gather=True` all-gathers the
    (n_trans, ...) result on every rank."""

    def __init__(self, plan, group=None):
        self.plan = plan
        self.group = group

    def local_range(self, n_trans):
        rank, world = _world(self.group)
        return vector_range(n_trans, rank, world)

    def execute_batch(self, cs, return_np=True, gather=False):
        n = int(cs.shape[0])
        lo, hi = self.local_range(n)
        res = self.plan.execute_batch(cs[lo:hi], return_np=False)
        if gather:
            res = gather_rows(res, n, self.group)
        return finish(res, return_np)


class Type3TargetSplit:
    """Type 3 with the targets split across ranks: every rank plans over all
    sources and its split_range share of the targets (`plan` built by the
    caller on those targets); `gather=True` assembles all targets."""

    def __init__(self, plan, n_targets_total, group=None):
        self.plan = plan
        self.group = group
        self.n_total = n_targets_total

    def execute(self, c, return_np=True, gather=False):
        out = self.plan.execute(c, return_np=False)
        if gather:
            out = gather_rows(out, self.n_total, self.group)
        return finish(out, return_np)
