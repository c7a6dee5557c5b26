"""build_graph (src/graph_build.jl:256-288) through the library's host builder.

The builder (csrc/graph_build.cpp) restates the reference's CPU pipeline -- special-order heap
k-d tree, preceding k-NN by the stackless traversal, longest-path depths, stable re-sort by depth,
21-bit lattice quantisation, offsets -- so its graph is byte-identical to the reference's.  It is
the input producer of the refine path, not part of the accelerated path.
"""
from __future__ import annotations

import ctypes as C
import hashlib
import os

import numpy as np

from . import _lib
from .problem import GraphGPProblem


def build_graph_arrays(points, n0: int, k: int, lattice_bits: int = 21, nthreads: int = 0):
    """Run the builder; returns dict(coords (N,D) uint32, neighbors (M,K) int64 0-based,
    offsets int64, n0, scale float, indices int64 0-based tree->original)."""
    pts = np.asarray(points, dtype=np.float64)
    if pts.ndim != 2:
        raise ValueError("points must be (N, D)")
    N, D = pts.shape
    # Dim-major (Julia's (N, D) column-major) is what the builder reads natively.
    pf = np.asfortranarray(pts)
    L = _lib.lib()
    g = C.c_void_p()
    st = L.gpb2_build_graph(pf.ctypes.data_as(C.c_void_p), N, D, 1, int(n0), int(k),
                            int(lattice_bits), int(nthreads), C.byref(g))
    _lib.check(st, "build_graph")
    try:
        n_off = L.gpb2_graph_n_offsets(g)
        n0f = L.gpb2_graph_n0(g)
        coords = np.empty((N, D), np.uint32)
        nbrs = np.empty((N - n0f, k), np.int64)
        indices = np.empty(N, np.int64)
        offsets = np.empty(n_off, np.int64)
        scale = C.c_double()
        _lib.check(L.gpb2_graph_export(g, coords.ctypes.data_as(C.c_void_p),
                                       nbrs.ctypes.data_as(C.c_void_p),
                                       indices.ctypes.data_as(C.c_void_p),
                                       offsets.ctypes.data_as(C.c_void_p), C.byref(scale)),
                   "graph export")
    finally:
        L.gpb2_graph_free(g)
    return dict(coords=coords, neighbors=nbrs, offsets=offsets, n0=int(n0f), scale=scale.value,
                indices=indices)


def build_graph_device(points, n0: int, k: int, lattice_bits: int = 21, device=None):
    """build_graph on the GPU (gpb2_build_graph_device): the same graph, byte for byte, as
    ``build_graph_arrays``.  ``points`` is an (N, D) float64 torch tensor on the device (or a host
    array, copied there).  Returns dict(coords (N, D) int32 tensor holding the uint32 lattice
    coordinates, neighbors (M, K) int32 tensor 0-based, indices (N) int32 tensor 0-based
    tree->original, offsets int64 numpy array, n0, scale), all tensors on the device."""
    import torch
    if isinstance(points, torch.Tensor):
        dev = points.device if points.is_cuda else torch.device(
            "cuda", torch.cuda.current_device() if device is None else torch.device(device).index)
    else:
        dev = torch.device(device) if device is not None else torch.device(
            "cuda", torch.cuda.current_device())
    pts = torch.as_tensor(points, dtype=torch.float64).to(dev).contiguous()
    if pts.ndim != 2:
        raise ValueError("points must be (N, D)")
    N, D = pts.shape
    L = _lib.lib()
    g = C.c_void_p()
    with torch.cuda.device(dev):
        stream = C.c_void_p(torch.cuda.current_stream(dev).cuda_stream)
        _lib.check(L.gpb2_build_graph_device(C.c_void_p(pts.data_ptr()), N, D, 0, int(n0), int(k),
                                             int(lattice_bits), dev.index or 0, stream,
                                             C.byref(g)), "build_graph_device")
        try:
            n_off = L.gpb2_dgraph_n_offsets(g)
            n0f = L.gpb2_dgraph_n0(g)
            coords = torch.empty((N, D), dtype=torch.int32, device=dev)
            nbrs = torch.empty((N - n0f, k), dtype=torch.int32, device=dev)
            indices = torch.empty(N, dtype=torch.int32, device=dev)
            offsets = np.empty(n_off, np.int64)
            scale = C.c_double()
            _lib.check(L.gpb2_dgraph_export(g, C.c_void_p(coords.data_ptr()),
                                            C.c_void_p(nbrs.data_ptr()),
                                            C.c_void_p(indices.data_ptr()),
                                            offsets.ctypes.data_as(_lib.PI64), C.byref(scale),
                                            stream), "graph export")
            torch.cuda.current_stream(dev).synchronize()
        finally:
            L.gpb2_dgraph_free(g)
    return dict(coords=coords, neighbors=nbrs, offsets=offsets, n0=int(n0f), scale=scale.value,
                indices=indices)


def build_graph(points, n0: int, k: int, bins, vals, lattice_bits: int = 21, nthreads: int = 0,
                dtype=None, device=None) -> GraphGPProblem:
    """``build_graph(points, n0, k, bins, vals; lattice_bits=21)`` -> GraphGPProblem with the
    ``indices`` permutation set; ``scale`` is stored in the table's precision as the reference's
    ``eltype(vals)(scale)``."""
    g = build_graph_arrays(points, n0, k, lattice_bits, nthreads)
    dt = np.dtype(dtype) if dtype is not None else np.asarray(vals).dtype
    scale = float(dt.type(g["scale"]))
    return GraphGPProblem(g["coords"], g["neighbors"], g["offsets"], g["n0"], scale,
                          np.asarray(bins, dt), np.asarray(vals, dt), g["indices"], dtype=dt,
                          device=device)


def cached_graph(points_fn, key: str, n0: int, k: int, cache_dir: str | None = None,
                 nthreads: int = 0):
    """Build once and keep the arrays on disk (an .npz per key), so large configurations are
    built a single time.  ``points_fn()`` produces the points only when the cache misses."""
    cache_dir = cache_dir or os.environ.get("GPB2_GRAPH_CACHE",
                                            os.path.join(os.path.expanduser("~"), ".cache",
                                                         "graphgp_b200"))
    os.makedirs(cache_dir, exist_ok=True)
    h = hashlib.sha1(f"{key}|n0={n0}|k={k}".encode()).hexdigest()[:16]
    path = os.path.join(cache_dir, f"graph_{h}.npz")
    if os.path.exists(path):
        with np.load(path) as d:
            return {name: (d[name] if d[name].ndim else d[name].item()) for name in d.files}
    g = build_graph_arrays(points_fn(), n0, k, nthreads=nthreads)
    tmp = path + f".tmp{os.getpid()}.npz"
    np.savez(tmp, **g)
    os.replace(tmp, path)
    return g
