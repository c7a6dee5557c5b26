"""GraphGPProblem: the container the whole API dispatches on (src/types.jl:22-60).

Memory layout is the reference's: ``coords`` holds a point's D lattice coordinates contiguously
(Julia's (D, N) column-major UInt32 == numpy (N, D) row-major), ``neighbors`` holds a refined
point's K neighbour indices contiguously (Julia's (K, M) column-major == numpy (M, K)).  The
Python mirror uses 0-based neighbour and permutation indices (the convention of the Python
``graphgp`` package and of the reference's .npz fixtures); the Julia binding passes its 1-based
arrays to the same C entry points with ``neighbor_base = 1``.

``offsets`` are the batch ends with ``offsets[0] == n0`` and ``offsets[-1] == N``; batch b covers
tree positions ``[offsets[b-1], offsets[b])``.  ``indices[tree_pos] = original_pos`` (or None for
the identity), as ``GraphGPProblem.indices``.

The device-side state lives in a library handle (``gpb2_problem``) created on first use: it holds
int32 neighbours, padded coordinates and the interpolation table, and validates the graph
(check_graph's invariants) on the device.
"""
from __future__ import annotations

import ctypes as C
import weakref

import numpy as np
import torch

from . import _lib

_DT = {np.dtype(np.float32): _lib.GPB2_F32, np.dtype(np.float64): _lib.GPB2_F64}
_TORCH_DT = {np.dtype(np.float32): torch.float32, np.dtype(np.float64): torch.float64}


def _np_dtype(x) -> np.dtype:
    if isinstance(x, torch.Tensor):
        return np.dtype(str(x.dtype).replace("torch.", ""))
    return np.asarray(x).dtype


def _host(x, dtype=None) -> np.ndarray:
    if isinstance(x, torch.Tensor):
        x = x.detach().cpu().numpy()
    return np.ascontiguousarray(x, dtype=dtype)


def _destroy(handle_value: int) -> None:
    try:
        _lib.lib().gpb2_problem_destroy(C.c_void_p(handle_value))
    except Exception:  # interpreter shutdown: the library may already be gone
        pass


class GraphGPProblem:
    """GraphGPProblem(coords, neighbors, offsets, n0, scale, bins, vals, indices=None), or with
    an anisotropic covariance ``GraphGPProblem.anisotropic(coords, neighbors, offsets, n0,
    scale, cov, indices=None)`` (src/types.jl:62-68; forward operations only)."""

    @classmethod
    def anisotropic(cls, coords, neighbors, offsets, n0, scale, cov, indices=None, **kw):
        # The table holds the covariance's axes as placeholders, as in the reference.
        prob = cls(coords, neighbors, offsets, n0, scale, cov.spatial_bins, cov.z_bins, indices,
                   dtype=kw.pop("dtype", cov.grid.dtype), **kw)
        prob.cov = cov
        return prob

    def __init__(self, coords, neighbors, offsets, n0, scale, bins, vals, indices=None, *,
                 dtype=None, device=None, neighbor_base: int = 0):
        self.cov = None
        dt = np.dtype(dtype) if dtype is not None else _np_dtype(vals)
        if dt not in _DT:
            raise TypeError(f"vals must be float32 or float64 (got {dt})")
        self.dtype = dt
        self.coords = coords
        self.neighbors = neighbors
        self.offsets = _host(offsets, np.int64)
        self.n0 = int(n0)
        self.scale = float(scale)
        self.bins = bins
        self.vals = vals
        # A permutation already on the device (a graph built by build_graph_device) stays there.
        self.indices = None if indices is None else (
            indices if isinstance(indices, torch.Tensor) and indices.is_cuda
            else _host(indices, np.int64))
        self.neighbor_base = int(neighbor_base)
        if device is None:
            device = coords.device if isinstance(coords, torch.Tensor) and coords.is_cuda \
                else torch.device("cuda", torch.cuda.current_device() if torch.cuda.is_available() else 0)
        self.device = torch.device(device)
        self.host_arrays = not isinstance(coords, torch.Tensor)
        shape_c = tuple(coords.shape)
        shape_n = tuple(neighbors.shape)
        if len(shape_c) != 2 or len(shape_n) != 2:
            raise ValueError("coords must be (N, D) and neighbors (M, K)")
        self._N, self._D = shape_c
        self._M, self._K = shape_n
        if self._N - self._M != self.n0:
            raise ValueError(f"n0 ({self.n0}) must equal npoints - nrefined ({self._N - self._M})")
        self._handle = None
        self._finalizer = None

    # -- sizes (src/types.jl:72-76) ----------------------------------------------------------
    def npoints(self) -> int:
        return self._N

    def ndims_space(self) -> int:
        return self._D

    def nneighbors(self) -> int:
        return self._K

    def nrefined(self) -> int:
        return self._M

    def nbins(self) -> int:
        return int(len(self.bins))

    @property
    def torch_dtype(self):
        return _TORCH_DT[self.dtype]

    def n_batches(self) -> int:
        return len(self.offsets) - 1

    # -- device handle -------------------------------------------------------------------------
    def _dev(self, x, dtype):
        if isinstance(x, torch.Tensor):
            return x.to(device=self.device, dtype=dtype).contiguous()
        return torch.from_numpy(np.ascontiguousarray(x)).to(device=self.device, dtype=dtype)

    @property
    def handle(self) -> C.c_void_p:
        if self._handle is None:
            self._handle = self._create()
            self._finalizer = weakref.finalize(self, _destroy, self._handle.value)
        return self._handle

    def _create(self) -> C.c_void_p:
        L = _lib.lib()
        with torch.cuda.device(self.device):
            c = self.coords
            if isinstance(c, torch.Tensor):
                c = c.view(torch.int32) if c.dtype == torch.uint32 else c
                coords = c.to(device=self.device, dtype=torch.int32).contiguous()
            else:
                coords = torch.from_numpy(
                    np.ascontiguousarray(c, dtype=np.uint32).view(np.int32)).to(self.device)
            nb = self.neighbors
            nb_dt = torch.int32 if _np_dtype(nb) in (np.dtype(np.int32), np.dtype(np.uint32)) \
                else torch.int64
            nbd = self._dev(nb, nb_dt)
            bins = self._dev(self.bins, self.torch_dtype)
            vals = self._dev(self.vals, self.torch_dtype)
            offs = np.ascontiguousarray(self.offsets, dtype=np.int64)
            stream = torch.cuda.current_stream(self.device).cuda_stream
            h = C.c_void_p()
            common = (C.byref(h), _DT[self.dtype], self.device.index or 0,
                      C.c_void_p(coords.data_ptr()), self._D, self._N,
                      C.c_void_p(nbd.data_ptr()), 4 if nb_dt == torch.int32 else 8,
                      self.neighbor_base, self._K, offs.ctypes.data_as(_lib.PI64), len(offs),
                      self.n0, self.scale, C.c_void_p(bins.data_ptr()),
                      C.c_void_p(vals.data_ptr()), self.nbins())
            if isinstance(self.indices, torch.Tensor):
                idx = self.indices.to(self.device).contiguous()
                if idx.dtype not in (torch.int32, torch.int64):
                    raise TypeError("indices must be int32 or int64")
                st = L.gpb2_problem_create_dev(*common, C.c_void_p(idx.data_ptr()),
                                               4 if idx.dtype == torch.int32 else 8, 0,
                                               C.c_void_p(stream))
            else:
                idx = None if self.indices is None else np.ascontiguousarray(self.indices,
                                                                             np.int64)
                st = L.gpb2_problem_create(*common,
                                           None if idx is None else idx.ctypes.data_as(_lib.PI64),
                                           0, C.c_void_p(stream))
            _lib.check(st, "GraphGPProblem upload")
            if self.cov is not None:
                cv = self.cov
                sb = self._dev(cv.spatial_bins, self.torch_dtype)
                zb = self._dev(cv.z_bins, self.torch_dtype)
                # (ns, nz) column-major, as the reference's Matrix.
                g = self._dev(np.asarray(cv.grid).ravel(order="F"), self.torch_dtype)
                st = L.gpb2_problem_set_aniso(h, C.c_void_p(sb.data_ptr()), sb.numel(),
                                              C.c_void_p(zb.data_ptr()), zb.numel(),
                                              C.c_void_p(g.data_ptr()), float(cv.alpha),
                                              C.c_void_p(stream))
                if st != 0:
                    L.gpb2_problem_destroy(h)
                    _lib.check(st, "GraphGPProblem anisotropic covariance")
        return h

    def update_vals(self, vals) -> "GraphGPProblem":
        """Replace the covariance table in place (same bins; the handle and its device graph are
        kept).  The dense block is refactorised by the next call that needs it; until then every
        call reuses the factor of the current table."""
        if self._handle is None:
            self.vals = vals
            return self
        v = self._dev(vals, self.torch_dtype)
        if v.numel() != self.nbins():
            raise ValueError(f"vals has {v.numel()} entries, the table has {self.nbins()} bins")
        st = _lib.lib().gpb2_problem_set_vals(
            self.handle, C.c_void_p(v.data_ptr()),
            C.c_void_p(torch.cuda.current_stream(self.device).cuda_stream))
        _lib.check(st, "update_vals")
        self.vals = vals
        return self

    def prefactor(self) -> "GraphGPProblem":
        """Queue the current table's factorisations (dense block and per-point factors) on the
        current stream without waiting, so they overlap whatever the caller does next (e.g.
        copying the next inputs in).  Operations factor an unfactorised table themselves; a
        dense block that no jitter step factorises is reported by the next operation."""
        st = _lib.lib().gpb2_problem_prefactor(
            self.handle, C.c_void_p(torch.cuda.current_stream(self.device).cuda_stream))
        _lib.check(st, "prefactor")
        return self

    def set_factor_cache(self, mode: int) -> "GraphGPProblem":
        """Per-point factor cache (the packed Cholesky factor and pair weights of every refined
        point, read by the vals-gradient kernels instead of recomputing them): 0 off (frees
        it), 1 always, 2 (default) from the first generate_grad_vals when the device keeps a
        margin of free memory beyond it.  Results are the same in every mode."""
        _lib.check(_lib.lib().gpb2_problem_set_factor_cache(self.handle, int(mode)),
                   "set_factor_cache")
        return self

    def factor_cache(self) -> dict:
        """{"mode", "valid" (0: nothing current, 1: the current table's factors of every point,
        2: those of this rank's level-sharded ranges), "bytes"} of the factor cache."""
        mode, valid, nbytes = C.c_int32(), C.c_int32(), C.c_int64()
        _lib.check(_lib.lib().gpb2_problem_factor_cache(self.handle, C.byref(mode),
                                                         C.byref(valid), C.byref(nbytes)),
                   "factor_cache")
        return {"mode": mode.value, "valid": valid.value, "bytes": nbytes.value}

    def set_reverse_mode(self, mode: int) -> "GraphGPProblem":
        """Reverse sweep form: 0 atomic push (sums in no fixed order), 1 pull through the
        transposed graph (the serial sweep's sums bit for bit), 2 (default) pull from 2e7
        refined points up (below, the push is faster) when the graph fits in free device
        memory with a margin."""
        _lib.check(_lib.lib().gpb2_problem_set_reverse_mode(self.handle, int(mode)),
                   "set_reverse_mode")
        return self

    def reverse_mode(self) -> dict:
        """{"mode", "built" (the transposed graph exists), "bytes"}."""
        mode, built, nbytes = C.c_int32(), C.c_int32(), C.c_int64()
        _lib.check(_lib.lib().gpb2_problem_reverse_mode(self.handle, C.byref(mode),
                                                         C.byref(built), C.byref(nbytes)),
                   "reverse_mode")
        return {"mode": mode.value, "built": bool(built.value), "bytes": nbytes.value}

    def check(self) -> "GraphGPProblem":
        """Wait for this handle's queued work on the current stream and raise its status (in
        the asynchronous call mode, `set_synchronous(False)`, operations do not wait)."""
        st = _lib.lib().gpb2_problem_check(
            self.handle, C.c_void_p(torch.cuda.current_stream(self.device).cuda_stream))
        _lib.check(st, "check")
        return self

    def library_order(self):
        """(lib_tree, lib_orig): the library's internal point order (gpb2_problem_order) as two
        int32 device tensors, library position -> tree position and -> original index.  Inside
        the handle every depth batch is sorted by Morton code; the range entry points
        (gpb2_refine_range, gpb2_refine_reverse_range) index in this order."""
        lt = torch.empty(self._N, dtype=torch.int32, device=self.device)
        lo = torch.empty(self._N, dtype=torch.int32, device=self.device)
        st = _lib.lib().gpb2_problem_order(
            self.handle, C.c_void_p(lt.data_ptr()), C.c_void_p(lo.data_ptr()),
            C.c_void_p(torch.cuda.current_stream(self.device).cuda_stream))
        _lib.check(st, "library_order")
        return lt, lo

    def dense_jitter(self) -> float:
        """Relative jitter of the dense block's last factorisation (0.0 = none needed, -1.0 =
        not factorised yet), the ladder of src/dense.jl:46-67."""
        out = C.c_double()
        _lib.check(_lib.lib().gpb2_problem_dense_jitter(self.handle, C.byref(out)))
        return out.value

    def dense_factor(self) -> np.ndarray:
        """The dense block's last Cholesky factor (n0 x n0 lower triangle) as a host array."""
        n = self.n0
        out = torch.empty((n, n), dtype=self.torch_dtype, device=self.device)
        st = _lib.lib().gpb2_problem_dense_factor(
            self.handle, C.c_void_p(out.data_ptr()),
            C.c_void_p(torch.cuda.current_stream(self.device).cuda_stream))
        _lib.check(st, "dense_factor")
        return np.tril(out.cpu().numpy().T)  # column-major on the device

    def release(self) -> None:
        """Free the device handle now (it is otherwise freed with the object)."""
        if self._finalizer is not None:
            self._finalizer()
        self._handle = None
        self._finalizer = None

    def __repr__(self) -> str:
        return (f"GraphGPProblem(N={self._N}, D={self._D}, K={self._K}, n0={self.n0}, "
                f"batches={self.n_batches()}, nbins={self.nbins()}, dtype={self.dtype.name}, "
                f"indices={'yes' if self.indices is not None else 'no'})")


def to_backend(prob: GraphGPProblem, device) -> GraphGPProblem:
    """A copy of ``prob`` bound to ``device`` (src/types.jl:97-106)."""
    return GraphGPProblem(prob.coords, prob.neighbors, prob.offsets, prob.n0, prob.scale,
                          prob.bins, prob.vals, prob.indices, dtype=prob.dtype, device=device,
                          neighbor_base=prob.neighbor_base)


def set_vals(prob: GraphGPProblem, vals) -> GraphGPProblem:
    """``_set_vals`` (src/chainrules.jl:18-21): the same problem with ``vals`` replaced."""
    return GraphGPProblem(prob.coords, prob.neighbors, prob.offsets, prob.n0, prob.scale,
                          prob.bins, vals, prob.indices, dtype=prob.dtype, device=prob.device,
                          neighbor_base=prob.neighbor_base)
