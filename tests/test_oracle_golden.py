"""The CPU oracle against the reference's golden vectors and known-answer tests.

Fixtures: test/reference/{small,medium,generate_parity}.npz of the reference (copied into
tests/golden by tests/golden/make_golden.py).  Tolerances are the reference's own
(test/test_refine.jl:1-30, test/test_gradients.jl:1-26, test/python_parity_generate.jl:35),
tightened where the restatement is closer than they require.
"""
import numpy as np
import pytest
import scipy.linalg as sl

from conftest import relerr
from oracle import oracle as O


def _prob(d, tag, dtype, with_indices=False):
    return O.make_problem(d["coords"], d["neighbors"], d["offsets"], d["n0"], d["scale"],
                          d["cov_bins" + tag], d["cov_vals" + tag],
                          d["indices"] if with_indices else None, dtype)


@pytest.mark.parametrize("name", ["small", "medium"])
def test_refine_f64_vs_jax(golden, name):
    d = golden(name)
    p = _prob(d, "64", np.float64)
    ld = O.refine_logdet(p)
    assert abs(ld - d["logdet64"]) <= 1e-12 * abs(d["logdet64"])
    assert relerr(O.refine_inv(p, d["values64"]), d["xi64"]) < 1e-12
    v = O.refine(p, d["initial_values64"], d["xi_ref64"])
    assert relerr(v, d["refine_values64"]) < 1e-12


@pytest.mark.parametrize("name", ["small", "medium"])
def test_refine_f32_vs_jax(golden, name):
    # f32 vs an independent f32 implementation: the reference's own tolerances (rtol 2e-3 on
    # logdet, 1e-2 on xi/values) -- f32 rounding-order differences are amplified by the
    # near-singular (k+1) blocks.
    d = golden(name)
    p = _prob(d, "32", np.float32)
    assert abs(O.refine_logdet(p) - d["logdet32"]) <= 2e-3 * abs(d["logdet32"])
    assert relerr(O.refine_inv(p, d["values32"]), d["xi32"]) < 1e-3
    assert relerr(O.refine(p, d["initial_values32"], d["xi_ref32"]), d["refine_values32"]) < 1e-4


@pytest.mark.parametrize("name", ["small", "medium"])
def test_gradients_vs_jax(golden, name):
    d = golden(name)
    p = _prob(d, "64", np.float64)
    ld, g = O.refine_logdet_grad_vals(p)
    assert abs(ld - d["logdet64"]) <= 1e-12 * abs(d["logdet64"])
    nz = d["grad_logdet_vals64"] != 0
    assert relerr(g[nz], d["grad_logdet_vals64"][nz]) < 1e-12
    assert np.allclose(g[nz], d["grad_logdet_vals64"][nz], rtol=1e-5, atol=1e-8)
    loss, gi = O.refine_inv_loss_grad_vals(p, d["values64"])
    assert abs(loss - d["inv_loss64"]) <= 1e-12 * abs(d["inv_loss64"])
    nz = d["grad_inv_loss_vals64"] != 0
    assert relerr(gi[nz], d["grad_inv_loss_vals64"][nz]) < 1e-12


def test_generate_parity_f64(golden):
    # test/python_parity_generate.jl: norm-relerr < 1e-12 in ORIGINAL order, non-identity indices.
    d = golden("generate_parity")
    p = _prob(d, "64", np.float64, with_indices=True)
    assert not np.array_equal(d["indices"], np.arange(len(d["indices"])))
    f = O.generate(p, d["xi"])
    assert relerr(f, d["generate_field"]) < 1e-12
    assert relerr(O.generate_inv(p, d["values"]), d["generate_inv_xi"]) < 1e-12
    assert relerr(O.generate_inv(p, f), d["xi"]) < 1e-10


def test_cov_lookup_known_answers():
    # test/test_interp.jl:2-20
    bins = np.array([0.0, 1.0, 2.0, 4.0], np.float32)
    vals = np.array([1.0, 0.5, 0.2, 0.05], np.float32)
    r = np.array([0.0, -3.0, 4.0, 99.0, 1.0, 2.0, 1.5, 3.0], np.float32)
    out = O.cov_lookup(r, bins, vals)
    assert list(out[:6]) == [1.0, 1.0, 0.05, 0.05, 0.5, 0.2]
    assert np.isclose(out[6], 0.35) and np.isclose(out[7], 0.125)
    lbins = np.concatenate([[0.0], 10.0 ** np.linspace(-4, 1, 199)]).astype(np.float32)
    lvals = np.exp(-(lbins.astype(np.float64) / 0.3) ** 2).astype(np.float32)
    rr = (10.0 ** np.linspace(-5, 1.3, 500)).astype(np.float32)
    ref = np.interp(rr.astype(np.float64), lbins.astype(np.float64), lvals.astype(np.float64))
    assert np.allclose(O.cov_lookup(rr, lbins, lvals), ref, rtol=1e-4, atol=1e-20)
    lo, wlo, whi = O.cov_lookup_weights(np.array([0.0, 1.5, 5.0], np.float32), bins)
    assert list(lo) == [0, 1, 2] and list(wlo) == [1.0, 0.5, 0.0] and list(whi) == [0.0, 0.5, 1.0]


@pytest.mark.parametrize("kp1", [2, 5, 11])
def test_chol_solve_vs_lapack(kp1):
    # test/test_linalg.jl:3-27
    rng = np.random.default_rng(42 + kp1)
    B = rng.standard_normal((kp1, kp1))
    S = B @ B.T + kp1 * np.eye(kp1)
    L, mv = O.chol_solve(S, kp1 - 1)
    Lref = np.linalg.cholesky(S)
    assert np.allclose(L, Lref, rtol=1e-10)
    if kp1 > 1:
        xref = sl.solve_triangular(Lref[:-1, :-1].T, Lref[-1, :-1], lower=False)
        assert np.allclose(mv, xref, rtol=1e-10)


def test_chol_indefinite_clamped():
    # test/test_linalg.jl:29-33: an indefinite 2x2 is regularised, not NaN-propagated.
    L, _ = O.chol_solve(np.array([[1.0, 2.0], [2.0, 1.0]], np.float32), 1)
    assert np.isfinite(L[1, 1]) and 0 < L[1, 1] <= 1e-3


def test_dense_roundtrip_and_logdet(golden):
    # test/test_dense.jl:1-40
    d = golden("small")
    p = _prob(d, "64", np.float64)
    L, jit = O.dense_chol(p)
    assert jit == 0.0
    xi = np.random.default_rng(42).standard_normal(p.n0)
    v = O.generate_dense(L, xi)
    assert np.allclose(O.generate_dense_inv(L, v), xi, rtol=1e-10, atol=1e-12)
    Km = O.dense_cov(p)
    assert np.isclose(O.dense_logdet(L), 0.5 * np.linalg.slogdet(Km)[1], rtol=1e-12)
    assert np.allclose(L, np.linalg.cholesky(Km), rtol=1e-12, atol=1e-14)


def test_generate_logdet_is_dense_plus_refine(golden):
    # test/test_orchestrate.jl:30-40
    d = golden("small")
    p = _prob(d, "64", np.float64)
    L, _ = O.dense_chol(p)
    assert np.isclose(O.generate_logdet(p), O.dense_logdet(L) + O.refine_logdet(p), rtol=1e-12)


def test_blocked_cholesky_adjoint_matches_scalar(golden):
    # The device computes chol_pullback_dyn! in the blocked form S = L^-T Phi(L^T Lbar) L^-1;
    # pin that identity against the scalar recurrence on the fixture's dense block.
    d = golden("generate_parity")
    p = _prob(d, "64", np.float64)
    L, _ = O.dense_chol(p)
    n = L.shape[0]
    rng = np.random.default_rng(0)
    Lbar = np.tril(np.outer(rng.standard_normal(n), rng.standard_normal(n)))
    A1 = np.tril(O.chol_pullback_dense(L, Lbar))
    P = np.tril(L.T @ Lbar)
    P[np.diag_indices(n)] *= 0.5
    Y = sl.solve_triangular(L, P, trans="T", lower=True)
    S = sl.solve_triangular(L, Y.T, trans="T", lower=True).T
    A2 = np.tril(S + S.T)
    A2[np.diag_indices(n)] = np.diag(S)
    assert relerr(A2, A1) < 1e-13


def test_adjoint_identity_and_fd(golden):
    # test/test_gradients.jl:56-77 (adjoint identity 1e-10) and test/test_ordering.jl FD checks.
    d = golden("generate_parity")
    p = _prob(d, "64", np.float64, with_indices=True)
    N = len(d["xi"])
    rng = np.random.default_rng(9)
    x = rng.standard_normal(N)
    vb = rng.standard_normal(N)
    lhs = float(vb @ O.generate(p, x))
    rhs = float(O.generate_grad_xi(p, vb) @ x)
    assert abs(lhs - rhs) <= 1e-10 * abs(lhs)
    # generate_grad_vals vs central differences of sum(vb .* generate_of_vals(vals)).
    dv = O.generate_grad_vals(p, x, vb)
    for i in (5, 40, 120, 200):
        h = 1e-6 * max(abs(p.vals[i]), 1e-3)
        pp = O.make_problem(p.coords, p.nbrs, p.offsets, p.n0, p.scale, p.bins,
                            p.vals + h * (np.arange(len(p.vals)) == i), p.indices, np.float64)
        pm = O.make_problem(p.coords, p.nbrs, p.offsets, p.n0, p.scale, p.bins,
                            p.vals - h * (np.arange(len(p.vals)) == i), p.indices, np.float64)
        fd = (float(vb @ O.generate(pp, x)) - float(vb @ O.generate(pm, x))) / (2 * h)
        assert np.isclose(dv[i], fd, rtol=1e-4, atol=1e-6), (i, dv[i], fd)


def test_logdet_grad_vs_fd(golden):
    d = golden("small")
    p = _prob(d, "64", np.float64)
    g = O.generate_logdet_grad_vals(p)
    for i in (0, 3, 50, 300):
        h = 1e-7
        e = h * (np.arange(len(p.vals)) == i)
        pp = O.make_problem(p.coords, p.nbrs, p.offsets, p.n0, p.scale, p.bins, p.vals + e,
                            None, np.float64)
        pm = O.make_problem(p.coords, p.nbrs, p.offsets, p.n0, p.scale, p.bins, p.vals - e,
                            None, np.float64)
        fd = (O.generate_logdet(pp) - O.generate_logdet(pm)) / (2 * h)
        assert np.isclose(g[i], fd, rtol=1e-5, atol=1e-4), (i, g[i], fd)
