"""Row-sharded multi-GPU SpMV: one process per GPU, torch.distributed (NCCL)
for the plumbing.

Layout (no counterpart in the reference, which is single-GPU):
  * rows are split at equal-nnz boundaries (``shard_bounds``); rank k owns
    rows [b_k, b_{k+1}) with its own CSR slice (row_ptr rebased to 0), a full
    replica of x, and writes the disjoint slice y[b_k, b_{k+1});
  * a single multiply needs no collective (each rank's y slice is final);
  * the iterated multiply y <- A*y/||y|| (benchmark config 5) re-assembles y
    into every rank's next x with an all-gather over NVLink and reduces the
    8-byte partial ||y||^2 with an all-reduce.

The local multiply is the library's CUDA kernel on the rank's slice; the
iteration logic here is written against a ``local_spmv`` callable and a
process group so that the same code runs on CPU ``gloo`` ranks in the tests.
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import numpy as np


def equal_nnz_bounds(row_lengths_prefix: np.ndarray, parts: int) -> np.ndarray:
    """bounds[k] = first row r with prefix[r] >= k*nnz/parts (prefix = row_ptr)."""
    rp = np.asarray(row_lengths_prefix, dtype=np.int64)
    m = len(rp) - 1
    z = int(rp[-1] - rp[0])
    b = np.zeros(parts + 1, dtype=np.int64)
    for k in range(1, parts):
        b[k] = max(int(np.searchsorted(rp, int(rp[0]) + (z * k) // parts, side="left")), b[k - 1])
    b[parts] = m
    return b


def gen_bounds(pf, spec, parts: int) -> np.ndarray:
    """Equal-nnz row bounds of a generated config without materialising it:
    fixed-length configs split by rows; others through the row-length prefix."""
    s = spec.resolved()
    if s.cfg in (1, 4, 5):
        return np.array([(s.m * k) // parts for k in range(parts + 1)], dtype=np.int64)
    lens = np.zeros(s.m, dtype=np.int64)
    import ctypes as C
    pf._check(pf.lib.pf_gen_row_lengths_host(C.byref(s.c()), 0, s.m, lens.ctypes.data))
    rp = np.zeros(s.m + 1, dtype=np.int64)
    np.cumsum(lens, out=rp[1:])
    return equal_nnz_bounds(rp, parts)


@dataclass
class StepStats:
    norm_sq: float


class PowerIteration:
    """x_{k+1} = A x_k / ||A x_k|| over row shards.

    ``local_spmv(x_full, y_local, alpha)`` computes y_local = alpha * A_k x_full
    for this rank's rows. ``x`` holds the previous (unnormalised) iterate on
    every rank, and the normalisation 1/||x|| is applied as the next multiply's
    alpha, so no extra pass over x is needed.
    """

    def __init__(self, local_spmv, x_full, y_local, bounds, rank: int, world: int,
                 group=None, torch_mod=None):
        import torch
        import torch.distributed as dist
        self.torch = torch_mod or torch
        self.dist = dist
        self.local_spmv = local_spmv
        self.x = x_full
        self.y = y_local
        self.bounds = bounds
        self.rank, self.world, self.group = rank, world, group
        self.equal = len(set(int(bounds[k + 1] - bounds[k]) for k in range(world))) == 1
        # 1/||x0||
        nsq = float(self.torch.dot(x_full, x_full).item())
        self.alpha = 1.0 / math.sqrt(nsq) if nsq > 0 else 1.0

    def step(self) -> StepStats:
        torch, dist = self.torch, self.dist
        self.local_spmv(self.x, self.y, self.alpha)
        sq = torch.dot(self.y, self.y).reshape(1)
        if self.world > 1:
            dist.all_reduce(sq, group=self.group)
            if self.equal and dist.get_backend(self.group) == "nccl":
                dist.all_gather_into_tensor(self.x, self.y, group=self.group)
            else:
                # all-gather-v: each rank broadcasts its slice of y into x
                b = self.bounds
                self.x[int(b[self.rank]):int(b[self.rank + 1])].copy_(self.y)
                for k in range(self.world):
                    dist.broadcast(self.x[int(b[k]):int(b[k + 1])], src=k, group=self.group)
        else:
            self.x.copy_(self.y)
        nsq = float(sq.item())
        self.alpha = 1.0 / math.sqrt(nsq) if nsq > 0 else 1.0
        return StepStats(nsq)


class FusedPowerIteration:
    """x_{k+1} = A x_k / ||A x_k|| with the all-gather fused into the multiply.

    The kernel (pf_spmv_dist_*) stores every finished row of this rank
    straight into every rank's next-x buffer over NVLink and reduces ||y||^2
    in the same pass; alpha = 1/||x_k|| is taken on the device from the norm
    slots, and the kernel is also the step barrier (step counters in the same
    memory), so a step is one kernel launch and the host never waits for the
    GPU or for the other ranks.

    Buffers: one symmetric-memory allocation per rank (torch symmetric
    memory: every rank can address every other rank's copy) holding two x
    buffers, two norm-slot arrays and the step counters. Step k reads x[k%2]
    and slots[k%2] and writes x[(k+1)%2] and slots[(k+1)%2] on every rank; it
    starts reading only when every rank has finished step k-1, which makes
    peers' stores visible and keeps any rank from overwriting a buffer that
    another rank still reads. With one rank the buffers are ordinary device
    memory and there is nothing to wait for.
    """

    SLOTS = 64

    def __init__(self, pf, handle, row_ptr, col, val, x0, bounds, rank: int, world: int,
                 group=None, stream=None):
        import torch
        self.torch, self.pf, self.h = torch, pf, handle
        self.rp, self.col, self.val = row_ptr, col, val
        self.rank, self.world = rank, world
        self.n = int(x0.numel())
        self.m = int(bounds[rank + 1] - bounds[rank])
        self.row_offset = int(bounds[rank])
        self.nnz = int(col.numel())
        self.stream = stream or torch.cuda.current_stream(x0.device)
        dev = x0.device
        total = 2 * self.n + 3 * self.SLOTS  # x0, x1, slots0, slots1, step counters
        if world > 1:
            import torch.distributed as dist
            import torch.distributed._symmetric_memory as symm_mem
            self.buf = symm_mem.empty(total, dtype=torch.float64, device=dev)
            g = group or dist.group.WORLD
            self.hdl = symm_mem.rendezvous(self.buf, g)
            bases = [int(p) for p in self.hdl.buffer_ptrs]
        else:
            self.buf = torch.empty(total, dtype=torch.float64, device=dev)
            self.hdl = None
            bases = [self.buf.data_ptr()]
        self.xs = [self.buf[0:self.n], self.buf[self.n:2 * self.n]]
        self.slots = [self.buf[2 * self.n:2 * self.n + self.SLOTS],
                      self.buf[2 * self.n + self.SLOTS:2 * self.n + 2 * self.SLOTS]]
        self.out_ptrs = [torch.tensor([b + 8 * k * self.n for b in bases], dtype=torch.int64,
                                      device=dev) for k in (0, 1)]
        self.slot_ptrs = [torch.tensor([b + 8 * (2 * self.n + k * self.SLOTS) for b in bases],
                                       dtype=torch.int64, device=dev) for k in (0, 1)]
        # step counters: uint64 words after the slots (zero: no step finished)
        self.flags = self.buf[2 * self.n + 2 * self.SLOTS:2 * self.n + 3 * self.SLOTS]
        self.flags.zero_()
        self.flag_ptrs = torch.tensor([b + 8 * (2 * self.n + 2 * self.SLOTS) for b in bases],
                                      dtype=torch.int64, device=dev) if world > 1 else None
        self.xs[0].copy_(x0)
        self.slots[0].zero_()
        self.slots[1].zero_()
        self.slots[0][0] = torch.dot(x0, x0)       # every rank holds the full x0
        self.k = 0
        torch.cuda.synchronize(dev)
        if self.hdl is not None:
            self.hdl.barrier(channel=0)

    def step(self):
        k = self.k
        self.pf.spmv_dist(self.h, self.m, self.n, self.nnz, self.rp, self.col, self.val,
                          self.xs[k % 2], self.slots[k % 2], self.world, self.rank,
                          self.out_ptrs[(k + 1) % 2].data_ptr(),
                          self.slot_ptrs[(k + 1) % 2].data_ptr(), self.row_offset,
                          stream=self.stream,
                          flag_ptrs_dev=self.flag_ptrs.data_ptr() if self.flag_ptrs is not None else 0,
                          step=k)
        self.k += 1

    @property
    def x(self):
        """The current (unnormalised) iterate."""
        return self.xs[self.k % 2]

    def sync(self):
        """Wait until every rank has finished its steps so far (a collective:
        every rank calls it): afterwards x and the norm slots are complete."""
        self.torch.cuda.synchronize(self.buf.device)
        if self.hdl is not None:
            self.hdl.barrier(channel=0)

    def norm_sq(self) -> float:
        """||A x_{k-1}||^2 of the last step (a collective: see sync)."""
        self.sync()
        return float(self.slots[self.k % 2][:self.world].sum().item())
