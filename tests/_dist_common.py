"""Shared pieces of the level-sharded tests: a small problem and a numpy implementation of the
per-batch ranges (the oracle's arithmetic, for the CPU/gloo runs)."""
import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
for p in (ROOT, os.path.join(ROOT, "graphgp.jl_b200")):
    if p not in sys.path:
        sys.path.insert(0, p)

import graphgp_b200 as gp  # noqa: E402
from oracle import oracle as O  # noqa: E402


def small_problem(dt, N=3000, n0=64, k=8, seed=17):
    rng = np.random.default_rng(seed)
    pts = rng.standard_normal((N, 2))
    bins, vals = gp.rbf_kernel(1.0, 0.3, 1e-4, 10.0, 1000, jitter=1e-5)
    g = gp.build_graph_arrays(pts, n0, k)
    args = (g["coords"], g["neighbors"], g["offsets"], g["n0"], dt(g["scale"]), bins.astype(dt),
            vals.astype(dt), g["indices"])
    return args


class NumpyOps:
    """refine_range / reverse_range / dense_apply on CPU torch tensors, with the oracle's
    per-point factors and dense factor (test infrastructure)."""

    def __init__(self, orc, dt):
        self.dt = dt
        self.mv, self.sd = O.meanvec_std(orc)
        self.nbrs = np.asarray(orc.nbrs, np.int64)
        self.n0 = int(orc.n0)
        self.K = self.nbrs.shape[1]
        self.L, _ = O.dense_chol(orc)

    def refine_range(self, values, xi_ref, lo, hi):
        if hi <= lo:
            return
        v = values.numpy()
        x = xi_ref.numpy()
        m = np.arange(lo - self.n0, hi - self.n0)
        acc = (self.sd[m] * x[m]).astype(self.dt)
        for j in range(self.K):  # std*xi first, then the K products in neighbour order
            acc = (acc + (self.mv[m, j] * v[self.nbrs[m, j]]).astype(self.dt)).astype(self.dt)
        v[lo:hi] = acc

    def reverse_range(self, xg, vb, lo, hi):
        if hi <= lo:
            return
        g = xg.numpy()
        b = vb.numpy()
        m = np.arange(lo - self.n0, hi - self.n0)
        vp = b[lo:hi].copy()
        g[lo:hi] = self.sd[m] * vp
        for j in range(self.K):
            np.add.at(b, self.nbrs[m, j], (self.mv[m, j] * vp).astype(self.dt))

    def dense_apply(self, trans, x, y):
        xd = np.ascontiguousarray(x.numpy()[: self.n0])
        y.numpy()[: self.n0] = O.dense_adjoint(self.L, xd) if trans else O.generate_dense(self.L, xd)
