"""Level-sharded generate / generate_grad_xi over several GPUs, one process per GPU.

The reference shards its distributed path by points with MPI (src/distributed.jl:129-247,
293-322); here the depth batches themselves are split.  Every rank holds the whole problem (graph,
table, dense factor) and the whole field.  For each depth batch b = [lo, hi) the points are cut
into `world` contiguous chunks of c = ceil((hi - lo) / world) points; rank g computes chunk g and
an in-place all-gather over NCCL, values[lo : lo + world*c] <- chunks, completes the batch on
every rank before batch b+1 starts.  The gather may spill past `hi` into the next batch's slots
(overwritten when that batch is computed) and past N into a slack region.  Batches smaller than
`min_shard` points are computed by every rank with no exchange.

The reverse sweep (generate_grad_xi) keeps a partial cotangent per rank: before batch b is
processed (latest first) its segment is summed over the ranks (reduce-scatter for sharded
batches, all-reduce for small ones), each rank then scatters the contributions of its own chunk
into its partial cotangent, and at the end the dense block's cotangents are all-reduced and the
per-rank xbar pieces summed.

The per-batch work goes through the C ABI's range entry points (gpb2_refine_range,
gpb2_refine_reverse_range, gpb2_dense_apply); `ops` can be replaced (the CPU tests run the
orchestration under gloo with a numpy implementation of the same ranges).
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass

import numpy as np
import torch
import torch.distributed as dist

from . import _lib
from .problem import GraphGPProblem


@dataclass(frozen=True)
class Batch:
    lo: int        # first tree position of the batch
    hi: int        # one past the last
    chunk: int     # points per rank (sharded batches)
    sharded: bool

    def mine(self, rank: int) -> tuple[int, int]:
        """This rank's slice [a, b) of the batch (all of it when not sharded)."""
        if not self.sharded:
            return self.lo, self.hi
        a = min(self.hi, self.lo + rank * self.chunk)
        return a, min(self.hi, a + self.chunk)


def plan_batches(offsets, world: int, min_shard: int) -> tuple[list[Batch], int]:
    """Per-batch sharding plan and the slack (entries past N) the gathers may touch."""
    batches, slack = [], 0
    offs = [int(o) for o in offsets]
    n = offs[-1]
    for lo, hi in zip(offs[:-1], offs[1:]):
        size = hi - lo
        sharded = world > 1 and size >= max(min_shard, world)
        chunk = -(-size // world) if sharded else size
        batches.append(Batch(lo, hi, chunk, sharded))
        if sharded:
            slack = max(slack, lo + world * chunk - n)
    return batches, max(slack, 0)


class DeviceOps:
    """The per-batch work on this rank's GPU, through the C ABI (asynchronous on the current
    stream except dense_apply)."""

    def __init__(self, prob: GraphGPProblem):
        self.prob = prob
        self.lib = _lib.lib()

    def _s(self):
        return C.c_void_p(torch.cuda.current_stream(self.prob.device).cuda_stream)

    def refine_range(self, values, xi_ref, lo, hi):
        _lib.check(self.lib.gpb2_refine_range(self.prob.handle, C.c_void_p(values.data_ptr()),
                                              C.c_void_p(xi_ref.data_ptr()), lo, hi, self._s()),
                   "refine_range")

    def reverse_range(self, xg, vb, lo, hi):
        _lib.check(self.lib.gpb2_refine_reverse_range(
            self.prob.handle, C.c_void_p(xg.data_ptr()), C.c_void_p(vb.data_ptr()), lo, hi,
            self._s()), "refine_reverse_range")

    def dense_apply(self, trans, x, y):
        _lib.check(self.lib.gpb2_dense_apply(self.prob.handle, 1 if trans else 0,
                                             C.c_void_p(x.data_ptr()), C.c_void_p(y.data_ptr()),
                                             self._s()), "dense_apply")


class ShardedGenerate:
    """generate / generate_grad_xi of `prob` with every depth batch split over the ranks of
    `group` (default: the world).  Inputs and outputs are full-length tensors (original point
    order) on every rank."""

    def __init__(self, prob: GraphGPProblem, group=None, min_shard: int = 65536, ops=None,
                 device=None):
        self.prob = prob
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.min_shard = int(min_shard)
        self.batches, self.slack = plan_batches(prob.offsets, self.world, self.min_shard)
        self.ops = ops if ops is not None else DeviceOps(prob)
        self.device = torch.device(device) if device is not None else prob.device
        self.dtype = prob.torch_dtype
        self.n, self.n0 = prob.npoints(), int(prob.n0)
        idx = prob.indices
        self.indices = None if idx is None else torch.as_tensor(np.asarray(idx, np.int64),
                                                                device=self.device)
        self.nccl = dist.get_backend(group) == "nccl"

    # -- collectives --------------------------------------------------------------------------
    def _gather_batch(self, buf: torch.Tensor, b: Batch):
        """buf[lo : lo + world*chunk] <- the ranks' chunks, in place."""
        c, lo = b.chunk, b.lo
        out = buf[lo: lo + self.world * c]
        mine = buf[lo + self.rank * c: lo + (self.rank + 1) * c]
        if self.nccl:
            dist.all_gather_into_tensor(out, mine, group=self.group)
        else:
            parts = [torch.empty_like(mine) for _ in range(self.world)]
            dist.all_gather(parts, mine.clone(), group=self.group)
            out.copy_(torch.cat(parts))

    def _reduce_batch(self, buf: torch.Tensor, b: Batch):
        """Sum the batch's segment of the partial cotangents over the ranks (each rank needs at
        least its own chunk; small batches get the whole segment)."""
        if not b.sharded:
            dist.all_reduce(buf[b.lo: b.hi], group=self.group)
            return
        c, lo = b.chunk, b.lo
        seg = buf[lo: lo + self.world * c]
        mine = buf[lo + self.rank * c: lo + (self.rank + 1) * c]
        if self.nccl:
            tmp = seg.clone()
            dist.reduce_scatter_tensor(mine, tmp, group=self.group)
        else:
            dist.all_reduce(seg, group=self.group)

    # -- permutation ----------------------------------------------------------------------------
    def _to_tree(self, x):
        x = torch.as_tensor(x, dtype=self.dtype, device=self.device)
        return x if self.indices is None else x.index_select(0, self.indices)

    def _to_orig(self, t):
        if self.indices is None:
            return t.clone()
        out = torch.empty_like(t)
        out[self.indices] = t
        return out

    # -- operations ------------------------------------------------------------------------------
    def generate(self, xi) -> torch.Tensor:
        """generate (src/orchestrate.jl:19-42) with level-sharded batches; bit-identical to the
        single-GPU path (the same per-point arithmetic)."""
        xt = self._to_tree(xi).contiguous()
        values = torch.zeros(self.n + self.slack, dtype=self.dtype, device=self.device)
        self.ops.dense_apply(False, xt, values)          # values[:n0] = L xt[:n0]
        xi_ref = xt[self.n0:].contiguous()
        for b in self.batches:
            a, e = b.mine(self.rank)
            self.ops.refine_range(values, xi_ref, a, e)
            if b.sharded:
                self._gather_batch(values, b)
        return self._to_orig(values[: self.n])

    def generate_grad_xi(self, vbar) -> torch.Tensor:
        """generate_grad_xi (src/grad.jl:392-506) with level-sharded batches."""
        vt = self._to_tree(vbar)
        vb = torch.zeros(self.n + self.slack, dtype=self.dtype, device=self.device)
        if self.rank == 0:
            vb[: self.n] = vt  # the upstream cotangent enters once
        xg = torch.zeros(self.n + self.slack, dtype=self.dtype, device=self.device)
        for b in reversed(self.batches):
            self._reduce_batch(vb, b)
            a, e = b.mine(self.rank) if b.sharded else self._small_share(b)
            self.ops.reverse_range(xg, vb, a, e)
        dist.all_reduce(vb[: self.n0], group=self.group)
        dist.all_reduce(xg[self.n0: self.n], group=self.group)
        dense = torch.zeros(self.n0, dtype=self.dtype, device=self.device)
        self.ops.dense_apply(True, vb[: self.n0].contiguous(), dense)
        xg[: self.n0] = dense
        return self._to_orig(xg[: self.n])

    def _small_share(self, b: Batch) -> tuple[int, int]:
        """A small batch's cotangent is complete on every rank after its all-reduce; its points
        are still split so that each contribution is scattered exactly once."""
        size = b.hi - b.lo
        c = -(-size // self.world)
        a = min(b.hi, b.lo + self.rank * c)
        return a, min(b.hi, a + c)
