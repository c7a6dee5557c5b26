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

Two forms:
* ``LevelSharded`` (the product path): the whole per-batch schedule runs inside the library
  (gpb2_*_sharded), with the library's own NCCL communicator (``Comm``) issuing the collectives
  on the caller's stream between the batch kernels; one C call per operation.
* ``ShardedGenerate``: the same schedule written out in Python over torch.distributed
  collectives and the C ABI's range entry points (gpb2_refine_range, gpb2_refine_reverse_range,
  gpb2_dense_apply).  Its `ops` can be replaced: the CPU tests run it under gloo with a numpy
  implementation of the ranges, which checks the plan and the orchestration without a GPU.

``DistributedGraphGPProblem`` is the reference's scheme-A fitting view (src/distributed.jl:34-44,
129-247): generate_logdet, generate_logdet(_and)_grad_vals and generate_inv_loss_grad_vals over
contiguous per-rank ranges of the refined points, with one all-reduce.
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
        if ops is None:
            # The library's range entry points index in its internal order (every depth batch
            # sorted by Morton code): map original <-> library positions.
            self.indices = prob.library_order()[1].to(device=self.device, dtype=torch.int64)
        else:
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



# ---------------------------------------------------------------------------------------------
# The library path: NCCL inside libgraphgp_b200.so
# ---------------------------------------------------------------------------------------------

class Comm:
    """The library's NCCL communicator (gpb2_comm) over the ranks of a torch.distributed group:
    rank 0 of the group makes the unique id, the group broadcasts it, every rank joins."""

    def __init__(self, group=None, device=None, min_shard: int = 65536, timeout_s: float = 300.0):
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.device = torch.device(device) if device is not None else torch.device(
            "cuda", torch.cuda.current_device())
        L = _lib.lib()
        uid = C.create_string_buffer(128)
        if self.rank == 0:
            _lib.check(L.gpb2_comm_unique_id(uid), "gpb2_comm_unique_id")
        obj = [bytes(uid.raw) if self.rank == 0 else None]
        src = dist.get_global_rank(group, 0) if group is not None else 0
        dist.broadcast_object_list(obj, src=src, group=group)
        uid = C.create_string_buffer(obj[0], 128)
        h = C.c_void_p()
        _lib.check(L.gpb2_comm_create(C.byref(h), self.world, self.rank, uid,
                                      self.device.index or 0, float(timeout_s)),
                   "gpb2_comm_create")
        self._h = h
        self.set_min_shard(min_shard)

    @property
    def handle(self) -> C.c_void_p:
        if self._h is None:
            raise RuntimeError("communicator is closed")
        return self._h

    def set_min_shard(self, min_shard: int) -> None:
        _lib.check(_lib.lib().gpb2_comm_set_min_shard(self.handle, int(min_shard)),
                   "gpb2_comm_set_min_shard")
        self.min_shard = int(min_shard)

    def close(self) -> None:
        if self._h is not None:
            _lib.check(_lib.lib().gpb2_comm_destroy(self._h), "gpb2_comm_destroy")
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def library_plan(offsets, world: int, rank: int, min_shard: int):
    """The library's sharding plan of a rank (gpb2_shard_plan, host only): per depth batch
    (forward range, own range, sharded) and the slack."""
    offs = np.ascontiguousarray(offsets, np.int64)
    nb = len(offs) - 1
    fl, fh, ol, oh = (np.empty(nb, np.int64) for _ in range(4))
    sh = np.empty(nb, np.int32)
    slack = C.c_int64()
    _lib.check(_lib.lib().gpb2_shard_plan(
        offs.ctypes.data_as(_lib.PI64), len(offs), world, rank, int(min_shard),
        fl.ctypes.data_as(_lib.PI64), fh.ctypes.data_as(_lib.PI64),
        ol.ctypes.data_as(_lib.PI64), oh.ctypes.data_as(_lib.PI64),
        sh.ctypes.data_as(C.POINTER(C.c_int)), C.byref(slack)), "gpb2_shard_plan")
    return [((int(a), int(b)), (int(c), int(d)), bool(e))
            for a, b, c, d, e in zip(fl, fh, ol, oh, sh)], int(slack.value)


class LevelSharded:
    """generate / generate_grad_xi / generate_grad_vals of `prob` with every depth batch split
    over the ranks of `comm` (a library ``Comm``); the per-batch kernels and collectives run
    inside the library, one C call per operation.  Inputs and outputs are full-length device
    tensors in original order on every rank; the results equal the single-GPU operations'."""

    def __init__(self, prob: GraphGPProblem, comm: Comm):
        self.prob = prob
        self.comm = comm

    def _s(self):
        return C.c_void_p(torch.cuda.current_stream(self.prob.device).cuda_stream)

    def _vec(self, x, name):
        t = torch.as_tensor(x, dtype=self.prob.torch_dtype, device=self.prob.device).contiguous()
        if t.ndim != 1 or t.shape[0] != self.prob.npoints():
            raise ValueError(f"{name} must have length {self.prob.npoints()}")
        return t

    def generate(self, xi, out=None) -> torch.Tensor:
        x = self._vec(xi, "xi")
        out = torch.empty_like(x) if out is None else out
        _lib.check(_lib.lib().gpb2_generate_sharded(self.prob.handle, self.comm.handle,
                                                    C.c_void_p(x.data_ptr()),
                                                    C.c_void_p(out.data_ptr()), self._s()),
                   "generate_sharded")
        return out

    def generate_grad_xi(self, vbar, out=None) -> torch.Tensor:
        v = self._vec(vbar, "vbar")
        out = torch.empty_like(v) if out is None else out
        _lib.check(_lib.lib().gpb2_generate_grad_xi_sharded(
            self.prob.handle, self.comm.handle, C.c_void_p(v.data_ptr()),
            C.c_void_p(out.data_ptr()), self._s()), "generate_grad_xi_sharded")
        return out

    def generate_grad_vals(self, xi, vbar, out=None) -> torch.Tensor:
        x = self._vec(xi, "xi")
        v = self._vec(vbar, "vbar")
        out = torch.empty(self.prob.nbins(), dtype=self.prob.torch_dtype,
                          device=self.prob.device) if out is None else out
        _lib.check(_lib.lib().gpb2_generate_grad_vals_sharded(
            self.prob.handle, self.comm.handle, C.c_void_p(x.data_ptr()),
            C.c_void_p(v.data_ptr()), C.c_void_p(out.data_ptr()), self._s()),
            "generate_grad_vals_sharded")
        return out


class DistributedGraphGPProblem:
    """Scheme-A fitting view of a problem (src/distributed.jl:34-44, 129-247): every rank holds
    the whole problem; the refined points are split into contiguous per-rank ranges (the first
    M mod ranks ranks take one more, _balanced_range, ext/GraphGPMPIExt.jl:25-36), rank 0 adds
    the dense first layer, and one all-reduce of nbins + 4 doubles (the histogram and the
    scalars, accumulated in float64) gives every rank the global result."""

    def __init__(self, prob: GraphGPProblem, comm: Comm):
        self.prob = prob
        self.comm = comm
        M, W, r = prob.nrefined(), comm.world, comm.rank
        base, rem = divmod(M, W)
        self.m_lo = r * (base + 1) if r < rem else rem * (base + 1) + (r - rem) * base
        self.m_hi = self.m_lo + (base + 1 if r < rem else base)   # exclusive
        self.is_root = r == 0

    def nrefined_local(self) -> int:
        return self.m_hi - self.m_lo

    def _s(self):
        return C.c_void_p(torch.cuda.current_stream(self.prob.device).cuda_stream)

    def generate_logdet(self) -> float:
        out = C.c_double()
        _lib.check(_lib.lib().gpb2_generate_logdet_sharded(self.prob.handle, self.comm.handle,
                                                           C.byref(out), self._s()),
                   "generate_logdet_sharded")
        return out.value

    def generate_logdet_and_grad_vals(self):
        out = torch.empty(self.prob.nbins(), dtype=self.prob.torch_dtype, device=self.prob.device)
        ld = C.c_double()
        _lib.check(_lib.lib().gpb2_generate_logdet_grad_vals_sharded(
            self.prob.handle, self.comm.handle, C.c_void_p(out.data_ptr()), C.byref(ld),
            self._s()), "generate_logdet_grad_vals_sharded")
        return ld.value, out

    def generate_logdet_grad_vals(self):
        return self.generate_logdet_and_grad_vals()[1]

    def generate_inv_loss_grad_vals(self, data):
        d = torch.as_tensor(data, dtype=self.prob.torch_dtype, device=self.prob.device).contiguous()
        out = torch.empty(self.prob.nbins(), dtype=self.prob.torch_dtype, device=self.prob.device)
        loss = C.c_double()
        _lib.check(_lib.lib().gpb2_generate_inv_loss_grad_vals_sharded(
            self.prob.handle, self.comm.handle, C.c_void_p(d.data_ptr()),
            C.c_void_p(out.data_ptr()), C.byref(loss), self._s()),
            "generate_inv_loss_grad_vals_sharded")
        return loss.value, out


def distribute(prob: GraphGPProblem, comm: Comm) -> DistributedGraphGPProblem:
    """``distribute(prob, comm)`` (ext/GraphGPMPIExt.jl:46-67): the scheme-A view of `prob`."""
    return DistributedGraphGPProblem(prob, comm)
