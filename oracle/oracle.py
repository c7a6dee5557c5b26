"""CPU oracle for the GraphGP.jl refine path -- TEST INFRASTRUCTURE ONLY.

Thin numpy/ctypes layer over ``libgp_oracle.so`` (the C restatement in ``gp_oracle.c``).  Only
``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline legs may import this
module; the product path (``graphgp_b200``) never does.

Problems are duck-typed: any object with the attributes
``coords`` (N, D) uint32, ``nbrs`` (M, K) int64 0-based, ``offsets`` (int64, offsets[0] == n0),
``n0``, ``scale``, ``bins``, ``vals``, ``indices`` (0-based tree->original or None) and ``dtype``
(numpy float32 / float64).  This is the memory layout of the reference's ``GraphGPProblem``
(``src/types.jl:22-60``): Julia's column-major (D, N) coords and (K, M) neighbours.

Orchestration follows ``src/orchestrate.jl:19-97`` (gather xi original->tree, dense block,
refine, scatter tree->original) and the gradient drivers of ``src/grad.jl`` and
``src/grad_generate_vals.jl``.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess
from types import SimpleNamespace

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "libgp_oracle.so")
_lib = None

P = C.c_void_p
I64 = C.c_int64
I32 = C.c_int


def build() -> str:
    """Compile libgp_oracle.so with the committed Makefile (gcc, -ffp-contract=off)."""
    subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _LIB_PATH


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH) or (
            os.path.getmtime(_LIB_PATH) < os.path.getmtime(os.path.join(_HERE, "gp_oracle.c"))
        ):
            build()
        _lib = C.CDLL(_LIB_PATH)
    return _lib


def _sfx(dtype) -> str:
    return "_f32" if np.dtype(dtype) == np.float32 else "_f64"


def _ct(dtype):
    return C.c_float if np.dtype(dtype) == np.float32 else C.c_double


def _p(a: np.ndarray):
    return a.ctypes.data_as(P)


def _fn(name, dtype):
    return getattr(lib(), name + _sfx(dtype))


def make_problem(coords, nbrs, offsets, n0, scale, bins, vals, indices=None, dtype=np.float64):
    """Bundle arrays in the oracle's layout (see module docstring)."""
    dt = np.dtype(dtype)
    return SimpleNamespace(
        coords=np.ascontiguousarray(coords, dtype=np.uint32),
        nbrs=np.ascontiguousarray(nbrs, dtype=np.int64),
        offsets=np.ascontiguousarray(offsets, dtype=np.int64),
        n0=int(n0),
        scale=dt.type(scale),
        bins=np.ascontiguousarray(bins, dtype=dt),
        vals=np.ascontiguousarray(vals, dtype=dt),
        indices=None if indices is None else np.ascontiguousarray(indices, dtype=np.int64),
        dtype=dt,
    )


def _dims(p):
    N, D = p.coords.shape
    M, K = p.nbrs.shape
    return N, D, M, K


def _common(p):
    N, D, M, K = _dims(p)
    return (I64(p.n0), I32(K), I32(D), _ct(p.dtype)(p.scale), _p(p.bins), _p(p.vals),
            I64(len(p.bins)))


# ---------------------------------------------------------------------------------------------
# L0 scalar numerics
# ---------------------------------------------------------------------------------------------

def cov_lookup(r, bins, vals):
    """src/interp.jl:10-34 on an array of radii."""
    dt = np.asarray(bins).dtype
    r = np.ascontiguousarray(np.atleast_1d(r), dtype=dt)
    bins = np.ascontiguousarray(bins, dtype=dt)
    vals = np.ascontiguousarray(vals, dtype=dt)
    out = np.empty_like(r)
    _fn("gpo_cov_lookup", dt)(_p(r), I64(r.size), _p(bins), _p(vals), I64(bins.size), _p(out))
    return out


def cov_lookup_weights(r, bins):
    """src/interp.jl:62-83: (lo 0-based, w_lo, w_hi)."""
    dt = np.asarray(bins).dtype
    r = np.ascontiguousarray(np.atleast_1d(r), dtype=dt)
    bins = np.ascontiguousarray(bins, dtype=dt)
    lo = np.empty(r.size, np.int64)
    wlo = np.empty_like(r)
    whi = np.empty_like(r)
    _fn("gpo_cov_lookup_weights", dt)(_p(r), I64(r.size), _p(bins), I64(bins.size), _p(lo),
                                      _p(wlo), _p(whi))
    return lo, wlo, whi


def chol_solve(A, K):
    """chol_lower! + mean_vec_solve! (src/linalg.jl:38-103) on one (K+1)x(K+1) matrix."""
    A = np.ascontiguousarray(A).copy()
    mv = np.empty(K, A.dtype)
    _fn("gpo_chol_solve", A.dtype)(_p(A), I32(K + 1), _p(mv))
    return np.tril(A), mv


# ---------------------------------------------------------------------------------------------
# Refine layer (tree order)
# ---------------------------------------------------------------------------------------------

def refine(p, initial_values, xi_ref, nthreads=0):
    """refine(prob, initial_values, xi) (src/api.jl:176-182)."""
    N, D, M, K = _dims(p)
    values = np.zeros(N, p.dtype)
    values[: p.n0] = initial_values
    xi_ref = np.ascontiguousarray(xi_ref, dtype=p.dtype)
    rc = _fn("gpo_refine", p.dtype)(_p(values), _p(xi_ref), _p(p.coords), _p(p.nbrs),
                                    _p(p.offsets), I64(len(p.offsets)), *_common(p), I32(nthreads))
    assert rc == 0
    return values


def meanvec_std(p, nthreads=0):
    N, D, M, K = _dims(p)
    mv = np.empty((M, K), p.dtype)
    sd = np.empty(M, p.dtype)
    rc = _fn("gpo_meanvec_std", p.dtype)(_p(mv), _p(sd), _p(p.coords), _p(p.nbrs), I64(M),
                                         *_common(p), I32(nthreads))
    assert rc == 0
    return mv, sd


def refine_inv(p, values, nthreads=0):
    """refine_inv (src/api.jl:66-103)."""
    N, D, M, K = _dims(p)
    values = np.ascontiguousarray(values, dtype=p.dtype)
    xi = np.empty(M, p.dtype)
    rc = _fn("gpo_refine_inv", p.dtype)(_p(xi), _p(values), _p(p.coords), _p(p.nbrs), I64(M),
                                        *_common(p), I32(nthreads))
    assert rc == 0
    return xi


def refine_logdet_terms(p, nthreads=0):
    N, D, M, K = _dims(p)
    terms = np.empty(M, p.dtype)
    rc = _fn("gpo_refine_logdet_terms", p.dtype)(_p(terms), _p(p.coords), _p(p.nbrs), I64(M),
                                                 *_common(p), I32(nthreads))
    assert rc == 0
    return terms


def refine_logdet(p, nthreads=0):
    """refine_logdet (src/api.jl:24-28); the sum is taken in float64."""
    return float(np.sum(refine_logdet_terms(p, nthreads).astype(np.float64)))


def refine_logdet_grad_vals(p, nthreads=0, acc_t=False):
    """refine_logdet_grad_vals (src/grad.jl:96-119) + the fused logdet sum.

    Returns (logdet_refine, dvals float64).  acc_t=True accumulates in T like the reference."""
    N, D, M, K = _dims(p)
    dv = np.zeros(len(p.bins), np.float64)
    ld = C.c_double(0.0)
    rc = _fn("gpo_refine_logdet_grad_vals", p.dtype)(
        _p(dv), C.byref(ld), _p(p.coords), _p(p.nbrs), I64(M), *_common(p), I32(nthreads),
        I32(1 if acc_t else 0))
    assert rc == 0
    return ld.value, dv


def refine_inv_loss_grad_vals(p, values, nthreads=0, acc_t=False):
    """refine_inv_loss_grad_vals (src/grad.jl:643-678): (loss, dvals float64)."""
    N, D, M, K = _dims(p)
    values = np.ascontiguousarray(values, dtype=p.dtype)
    dv = np.zeros(len(p.bins), np.float64)
    loss = C.c_double(0.0)
    rc = _fn("gpo_refine_inv_loss_grad_vals", p.dtype)(
        _p(dv), C.byref(loss), _p(values), _p(p.coords), _p(p.nbrs), I64(M), *_common(p),
        I32(nthreads), I32(1 if acc_t else 0))
    assert rc == 0
    return loss.value, dv


# ---------------------------------------------------------------------------------------------
# Dense first layer (src/dense.jl)
# ---------------------------------------------------------------------------------------------

def dense_cov(p, n=None):
    n = p.n0 if n is None else n
    N, D, M, K = _dims(p)
    Km = np.empty((n, n), p.dtype)
    _fn("gpo_dense_cov", p.dtype)(_p(Km), _p(p.coords), I64(n), I32(D),
                                  _ct(p.dtype)(p.scale), _p(p.bins), _p(p.vals), I64(len(p.bins)))
    return Km


_ANISO = None  # the anisotropic covariance in force (see `anisotropic`), or None


class anisotropic:
    """Context in which the assembly functions of the C restatement use an anisotropic
    covariance (src/aniso.jl) instead of the table: ``with anisotropic(p, cov): generate(p, xi)``.
    cov has spatial_bins (ns), z_bins (nz), grid (ns, nz) and alpha, in the problem's type."""

    def __init__(self, p, cov):
        self.p = p
        dt = p.dtype
        self.sb = np.ascontiguousarray(cov.spatial_bins, dt)
        self.zb = np.ascontiguousarray(cov.z_bins, dt)
        self.g = np.ascontiguousarray(np.asarray(cov.grid, dt).ravel(order="F"))
        self.alpha = float(cov.alpha)

    def __enter__(self):
        global _ANISO
        _fn("gpo_set_aniso", self.p.dtype)(_p(self.sb), I64(self.sb.size), _p(self.zb),
                                            I64(self.zb.size), _p(self.g),
                                            _ct(self.p.dtype)(self.alpha), I32(1))
        _ANISO = hash((self.sb.tobytes(), self.zb.tobytes(), self.g.tobytes(), self.alpha))
        return self

    def __exit__(self, *exc):
        global _ANISO
        _fn("gpo_set_aniso", self.p.dtype)(None, I64(0), None, I64(0), None,
                                            _ct(self.p.dtype)(1.0), I32(0))
        _ANISO = None


def aniso_lookup(p, ds, dz):
    """aniso_lookup (src/aniso.jl:67-85) of the model in force, on arrays."""
    ds = np.ascontiguousarray(np.atleast_1d(ds), p.dtype)
    dz = np.ascontiguousarray(np.atleast_1d(dz), p.dtype)
    out = np.empty_like(ds)
    _fn("gpo_aniso_lookup", p.dtype)(_p(ds), _p(dz), I64(ds.size), _p(out))
    return out


def dense_chol(p):
    """_dense_chol_L (src/dense.jl:46-67) -> (L, jitter_used).  The factor is kept on the
    problem object for its table (a large first layer takes minutes on the host)."""
    key = hash((p.vals.tobytes(), _ANISO))
    cached = getattr(p, "_dense_cache", None)
    if cached is not None and cached[0] == key:
        return cached[1], cached[2]
    L, jit = _dense_chol(p)
    p._dense_cache = (key, L, jit)
    return L, jit


def _dense_chol(p):
    Km = dense_cov(p)
    n = Km.shape[0]
    L = np.empty_like(Km)
    jit = _ct(p.dtype)(0)
    rc = _fn("gpo_dense_chol", p.dtype)(_p(L), _p(Km), I64(n), C.byref(jit))
    if rc != 0:
        raise RuntimeError("dense first-layer covariance is not positive definite even with "
                           "1e-2 relative jitter")
    return L, float(jit.value)


def _tri(fn, L, x):
    x = np.ascontiguousarray(x, dtype=L.dtype)
    out = np.empty_like(x)
    _fn(fn, L.dtype)(_p(out), _p(L), _p(x), I64(L.shape[0]))
    return out


def generate_dense(L, xi):
    return _tri("gpo_trmv_lower", L, xi)


def generate_dense_inv(L, values):
    return _tri("gpo_trsv_lower", L, values)


def dense_adjoint(L, vb):
    return _tri("gpo_trmv_lower_t", L, vb)


def dense_logdet(L):
    """sum(log, diag(L)) (src/dense.jl:142-147)."""
    f = _fn("gpo_dense_logdet", L.dtype)
    f.restype = C.c_double
    return float(f(_p(L), I64(L.shape[0])))


def chol_pullback_dense(L, Lbar):
    """chol_pullback_dyn! (src/grad_generate_vals.jl:18-39); returns Abar (lower)."""
    L = np.ascontiguousarray(L)
    Lbar = np.ascontiguousarray(Lbar, dtype=L.dtype).copy()
    Abar = np.zeros_like(L)
    _fn("gpo_chol_pullback_dense", L.dtype)(_p(Abar), _p(Lbar), _p(L), I64(L.shape[0]))
    return Abar


# ---------------------------------------------------------------------------------------------
# Orchestration (original order in / out)
# ---------------------------------------------------------------------------------------------

def _gather(p, x):
    x = np.asarray(x, dtype=p.dtype)
    return x if p.indices is None else x[p.indices]


def _scatter(p, x):
    if p.indices is None:
        return x
    out = np.empty_like(x)
    out[p.indices] = x
    return out


def generate(p, xi, nthreads=0):
    """generate (src/orchestrate.jl:19-42)."""
    xo = _gather(p, xi)
    L, _ = dense_chol(p)
    v0 = generate_dense(L, xo[: p.n0])
    values = refine(p, v0, xo[p.n0:], nthreads)
    return _scatter(p, values)


def generate_inv(p, values, nthreads=0):
    """generate_inv (src/orchestrate.jl:53-81)."""
    vo = _gather(p, values)
    xi_ref = refine_inv(p, vo, nthreads)
    L, _ = dense_chol(p)
    xi_d = generate_dense_inv(L, vo[: p.n0])
    return _scatter(p, np.concatenate([xi_d, xi_ref]).astype(p.dtype))


def generate_logdet(p, nthreads=0):
    """generate_logdet (src/orchestrate.jl:89-97)."""
    L, _ = dense_chol(p)
    return dense_logdet(L) + refine_logdet(p, nthreads)


def generate_grad_xi(p, vbar, nthreads=0):
    """generate_grad_xi, CPU branch (src/grad.jl:392-465)."""
    N, D, M, K = _dims(p)
    mv, sd = meanvec_std(p, nthreads)
    vb = np.array(_gather(p, vbar), dtype=p.dtype)
    xg = np.zeros(N, p.dtype)
    _fn("gpo_reverse_sweep", p.dtype)(_p(xg), _p(vb), _p(mv), _p(sd), _p(p.nbrs), _p(p.offsets),
                                      I64(len(p.offsets)), I64(p.n0), I32(K))
    L, _ = dense_chol(p)
    xg[: p.n0] = dense_adjoint(L, vb[: p.n0])
    return _scatter(p, xg)


def generate_grad_vals(p, xi, vbar, nthreads=0, acc_t=False):
    """generate_grad_vals (src/grad_generate_vals.jl:111-213) -> float64 d_vals.

    The forward field is recomputed with refine (the operation order of the device branch,
    src/grad_generate_vals.jl:227-234)."""
    N, D, M, K = _dims(p)
    xih = _gather(p, xi).copy()
    L, _ = dense_chol(p)
    v0 = generate_dense(L, xih[: p.n0])
    v = refine(p, v0, xih[p.n0:], nthreads)
    vb = np.array(_gather(p, vbar), dtype=p.dtype)
    mv, sd = meanvec_std(p, nthreads)
    dv = np.zeros(len(p.bins), np.float64)
    rc = _fn("gpo_generate_grad_vals_refine", p.dtype)(
        _p(dv), _p(vb), _p(v), _p(xih), _p(mv), _p(p.coords), _p(p.nbrs), _p(p.offsets),
        I64(len(p.offsets)), I64(p.n0), I32(K), I32(D), _ct(p.dtype)(p.scale), _p(p.bins),
        _p(p.vals), I64(len(p.bins)), I32(1 if acc_t else 0))
    assert rc == 0
    vbd = np.ascontiguousarray(vb[: p.n0])
    xid = np.ascontiguousarray(xih[: p.n0])
    if p.n0 > DENSE_BLOCKED_MIN:
        dense_grad_vals_blocked(p, L, vbd, xid, dv)
        return dv
    _fn("gpo_dense_grad_vals", p.dtype)(_p(dv), _p(L), _p(vbd), _p(xid), _p(p.coords),
                                        I64(p.n0), I32(D), _ct(p.dtype)(p.scale), _p(p.bins),
                                        I64(len(p.bins)), I32(1 if acc_t else 0))
    return dv


# First layers larger than this take the blocked dense pullback (the scalar recurrence is
# O(n0^3) on one thread, and on the host slow in the subnormal range a short correlation
# length drives the factor into).
DENSE_BLOCKED_MIN = 2048


def dense_grad_vals_blocked(p, L, vb, xi, dv):
    """Dense block of generate_grad_vals (src/grad_generate_vals.jl:252-280) for a large first
    layer, in float64: with Lbar = tril(vb xi^T), the pullback of chol_pullback_dyn!
    (src/grad_generate_vals.jl:18-39) is the lower triangle of S = L^-T Phi(L^T Lbar) L^-1
    (Phi: lower triangle, halved diagonal); the pair cotangent is S_ij + S_ji off the diagonal and
    S_ii on it.  Accumulated into dv (float64, nbins)."""
    from scipy.linalg import solve_triangular
    N, D, M, K = _dims(p)
    Lf = np.tril(np.asarray(L, np.float64))
    X = Lf.T @ np.tril(np.outer(np.asarray(vb, np.float64), np.asarray(xi, np.float64)))
    X = np.tril(X)
    X[np.diag_indices_from(X)] *= 0.5
    Y = solve_triangular(Lf, X, trans="T", lower=True)        # L^-T Phi
    S = solve_triangular(Lf, Y.T, trans="T", lower=True).T    # (L^-T Phi) L^-1
    G = np.tril(S, -1) + np.triu(S, 1).T
    G[np.diag_indices_from(G)] = np.diag(S)
    G = np.ascontiguousarray(G)
    _fn("gpo_dense_scatter", p.dtype)(_p(dv), _p(G), _p(p.coords), I64(p.n0), I32(D),
                                      _ct(p.dtype)(p.scale), _p(p.bins), I64(len(p.bins)))
    return dv


def dense_logdet_grad_vals(p, acc_t=False):
    """_dense_logdet_grad_vals (src/dense.jl:153-183) -> float64."""
    N, D, M, K = _dims(p)
    L, _ = dense_chol(p)
    dv = np.zeros(len(p.bins), np.float64)
    _fn("gpo_dense_logdet_grad_vals", p.dtype)(_p(dv), _p(L), _p(p.coords), I64(p.n0), I32(D),
                                               _ct(p.dtype)(p.scale), _p(p.bins),
                                               I64(len(p.bins)), I32(1 if acc_t else 0))
    return dv


def generate_logdet_grad_vals(p, nthreads=0, acc_t=False):
    """generate_logdet_grad_vals (src/grad.jl:149-154)."""
    _, dv = refine_logdet_grad_vals(p, nthreads, acc_t)
    return dv + dense_logdet_grad_vals(p, acc_t)


# ---------------------------------------------------------------------------------------------
# Point-position gradients (src/grad.jl:168-377, src/dense.jl:184-297): (N, D) in tree order,
# d(.)/dx for the continuous positions x = scale * coords (Julia's (D, N))
# ---------------------------------------------------------------------------------------------

def refine_logdet_grad_points(p):
    """refine_logdet_grad_points (src/grad.jl:168-233)."""
    N, D, M, K = _dims(p)
    dp = np.zeros((N, D), np.float64)
    rc = _fn("gpo_refine_logdet_grad_points", p.dtype)(_p(dp), _p(p.coords), _p(p.nbrs), I64(M),
                                                        *_common(p))
    assert rc == 0
    return dp.astype(p.dtype)


def refine_inv_loss_grad_points(p, values):
    """refine_inv_loss_grad_points (src/grad.jl:259-358); values in tree order."""
    N, D, M, K = _dims(p)
    values = np.ascontiguousarray(values, dtype=p.dtype)
    dp = np.zeros((N, D), np.float64)
    rc = _fn("gpo_refine_inv_loss_grad_points", p.dtype)(_p(dp), _p(values), _p(p.coords),
                                                          _p(p.nbrs), I64(M), *_common(p))
    assert rc == 0
    return dp.astype(p.dtype)


def dense_grad_points(p, y=None):
    """_dense_logdet_grad_points (y None) / _dense_inv_loss_grad_points (y = the first n0
    values in tree order) (src/dense.jl:188-225, 271-297): (N, D), zero past n0."""
    N, D, M, K = _dims(p)
    L, _ = dense_chol(p)
    dp = np.zeros((N, D), np.float64)
    yy = np.zeros(p.n0, p.dtype) if y is None else np.ascontiguousarray(y, dtype=p.dtype)
    _fn("gpo_dense_grad_points", p.dtype)(_p(dp), _p(L), _p(yy), _p(p.coords), I64(p.n0),
                                          I32(D), _ct(p.dtype)(p.scale), _p(p.bins), _p(p.vals),
                                          I64(len(p.bins)), I32(0 if y is None else 1))
    return dp.astype(p.dtype)


def generate_logdet_grad_points(p):
    """generate_logdet_grad_points (src/grad.jl:234-247): refinement + dense block."""
    return refine_logdet_grad_points(p) + dense_grad_points(p)


def generate_inv_loss_grad_points(p, data):
    """generate_inv_loss_grad_points (src/grad.jl:360-377); data in the original order."""
    d = np.asarray(data, p.dtype)
    dord = d if p.indices is None else d[p.indices]
    return refine_inv_loss_grad_points(p, dord) + dense_grad_points(p, dord[: p.n0])


# ---------------------------------------------------------------------------------------------
# Inputs: graph build and covariance tables, without the product library
# ---------------------------------------------------------------------------------------------

_GRAPH_PATH = os.path.join(_HERE, "libgp_graph.so")
_glib = None


def _graph_lib():
    global _glib
    if _glib is None:
        if not os.path.exists(_GRAPH_PATH):
            build()
        g = C.CDLL(_GRAPH_PATH)
        g.gpb2_build_graph.restype = I32
        g.gpb2_build_graph.argtypes = [P, I64, I64, I64, I64, I64, I64, I64, C.POINTER(P)]
        g.gpb2_graph_n_offsets.restype = I64
        g.gpb2_graph_n_offsets.argtypes = [P]
        g.gpb2_graph_n0.restype = I64
        g.gpb2_graph_n0.argtypes = [P]
        g.gpb2_graph_export.restype = I32
        g.gpb2_graph_export.argtypes = [P, P, P, P, P, C.POINTER(C.c_double)]
        g.gpb2_graph_free.restype = None
        g.gpb2_graph_free.argtypes = [P]
        g.gpo_graph_last_error.restype = C.c_char_p
        _glib = g
    return _glib


def build_graph(points, n0, k, lattice_bits=21, nthreads=0):
    """build_graph (src/graph_build.jl:256-288) on the host cores, through the oracle's own
    copy of the host builder (libgp_graph.so): returns dict(coords (N,D) uint32, neighbors
    (M,K) int64 0-based, offsets, n0, scale, indices 0-based tree->original)."""
    pts = np.asfortranarray(np.asarray(points, dtype=np.float64))
    N, D = pts.shape
    L = _graph_lib()
    g = P()
    st = L.gpb2_build_graph(pts.ctypes.data_as(P), N, D, 1, int(n0), int(k), int(lattice_bits),
                            int(nthreads), C.byref(g))
    if st != 0:
        raise RuntimeError(f"build_graph failed ({st}): {L.gpo_graph_last_error().decode()}")
    try:
        n_off = L.gpb2_graph_n_offsets(g)
        n0f = L.gpb2_graph_n0(g)
        coords = np.empty((N, D), np.uint32)
        nbrs = np.empty((N - n0f, k), np.int64)
        indices = np.empty(N, np.int64)
        offsets = np.empty(n_off, np.int64)
        scale = C.c_double()
        L.gpb2_graph_export(g, coords.ctypes.data_as(P), nbrs.ctypes.data_as(P),
                            indices.ctypes.data_as(P), offsets.ctypes.data_as(P), C.byref(scale))
    finally:
        L.gpb2_graph_free(g)
    return dict(coords=coords, neighbors=nbrs, offsets=offsets, n0=int(n0f), scale=scale.value,
                indices=indices)


def make_cov_bins(r_min, r_max, n_bins):
    """make_cov_bins (src/extras.jl:14-17): [0; 10 .^ range(log10 r_min, log10 r_max, n-1)]."""
    import math
    inner = 10.0 ** np.linspace(math.log10(float(r_min)), math.log10(float(r_max)), n_bins - 1)
    return np.concatenate([[0.0], inner])


def rbf_kernel(variance, scale, r_min, r_max, n_bins, jitter=0.0, dtype=np.float64):
    """rbf_kernel (src/extras.jl:26-38): variance*exp(-r^2/(2 scale^2)), vals[0] *= 1+jitter."""
    bins = make_cov_bins(r_min, r_max, n_bins)
    r = bins.astype(dtype)
    v = (np.asarray(variance, dtype) * np.exp(np.asarray(-0.5, dtype) * (r / np.asarray(scale, dtype)) ** 2)).astype(dtype)
    v[0] = v[0] * (1 + np.asarray(jitter, dtype))
    return bins, v


def matern_kernel(p, variance, cutoff, r_min, r_max, n_bins, jitter=0.0, dtype=np.float64):
    """matern_kernel (src/extras.jl:57-73), nu = p + 1/2: variance*exp(-x)*polyval(c, 2x) with
    x = sqrt(2p+1) r / cutoff and c_i = exp(lgamma(p+1) + lgamma(p+i+1) - lgamma(i+1)
    - lgamma(p-i+1) - lgamma(2p+1))."""
    import math
    bins = make_cov_bins(r_min, r_max, n_bins)
    c = [math.exp(math.lgamma(p + 1.0) + math.lgamma(p + i + 1.0) - math.lgamma(i + 1.0)
                  - math.lgamma(p - i + 1.0) - math.lgamma(2 * p + 1.0)) for i in range(p + 1)]
    r = bins.astype(dtype)
    x = dtype(math.sqrt(float(2 * p + 1))) * r / np.asarray(cutoff, dtype)
    z = 2 * x
    acc = np.full_like(z, c[0])
    for ci in c[1:]:
        acc = acc * z + dtype(ci)
    v = (np.asarray(variance, dtype) * np.exp(-x) * acc).astype(dtype)
    v[0] = v[0] * (1 + np.asarray(jitter, dtype))
    return bins, v


def clamp_stats(p, nthreads=0):
    """Near-singular diagnostics over the refined points: dict(points_clamped, pivots_clamped,
    collisions, weights_zeroed) (see gpo_clamp_stats in gp_oracle.c)."""
    N, D, M, K = _dims(p)
    out = np.zeros(4, np.int64)
    _fn("gpo_clamp_stats", p.dtype)(_p(out), _p(p.coords), _p(p.nbrs), I64(M), I64(p.n0), I32(K),
                                    I32(D), _ct(p.dtype)(p.scale), _p(p.bins), _p(p.vals),
                                    I64(len(p.bins)), I32(nthreads))
    return dict(points_clamped=int(out[0]), pivots_clamped=int(out[1]), collisions=int(out[2]),
                weights_zeroed=int(out[3]))
