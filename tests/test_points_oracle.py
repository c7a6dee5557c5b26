"""The host checker's point-position gradients, pinned as the reference pins its own
(test/test_gradients.jl:95-125, 160-201): central finite differences of a continuous-position
forward -- the dense block's and every refined point's covariance rebuilt from the positions
x = scale * coords through the table lookup -- at a few (point, dimension) pairs."""
import numpy as np
import pytest

from oracle import oracle as O

pytestmark = pytest.mark.filterwarnings("ignore::RuntimeWarning")


def _problem(seed=21, N=220, D=3, n0=16, k=6):
    rng = np.random.default_rng(seed)
    pts = rng.standard_normal((N, D))
    bins, vals = O.rbf_kernel(1.0, 0.5, 1e-4, 10.0, 300, jitter=1e-3)
    g = O.build_graph(pts, n0, k)
    p = O.make_problem(g["coords"], g["neighbors"], g["offsets"], g["n0"], g["scale"], bins,
                       vals, g["indices"], np.float64)
    return p, rng


def _cov(p, X, idx):
    """Covariance of the points idx from continuous positions X (N, D)."""
    d = np.linalg.norm(X[idx][:, None, :] - X[idx][None, :, :], axis=-1)
    return O.cov_lookup(d.ravel(), p.bins, p.vals).reshape(d.shape)


def _refined(p, X, per_point):
    s = 0.0
    K = p.nbrs.shape[1]
    for m in range(p.nbrs.shape[0]):
        idx = np.concatenate([p.nbrs[m], [p.n0 + m]])
        L = np.linalg.cholesky(_cov(p, X, idx))
        s += per_point(m, L, K)
    return s


def _fd(f, X, p_, d, h=1e-6):
    Xp = X.copy()
    Xp[p_, d] += h
    Xm = X.copy()
    Xm[p_, d] -= h
    return (f(Xp) - f(Xm)) / (2 * h)


def test_logdet_grad_points_fd():
    p, _ = _problem()
    X = p.scale * p.coords.astype(np.float64)
    n0 = p.n0

    def fwd(X):
        s = np.sum(np.log(np.diag(np.linalg.cholesky(_cov(p, X, np.arange(n0))))))
        return s + _refined(p, X, lambda m, L, K: np.log(L[K, K]))

    gp = O.generate_logdet_grad_points(p)
    assert gp.shape == X.shape
    for (q, d) in ((2, 0), (11, 1), (n0 + 4, 0), (n0 + 59, 2), (n0 + 149, 1)):
        fd = _fd(fwd, X, q, d)
        assert abs(gp[q, d] - fd) <= 2e-3 * abs(fd) + 1e-6, (q, d, gp[q, d], fd)


def test_inv_loss_grad_points_fd():
    p, rng = _problem()
    N = p.coords.shape[0]
    X = p.scale * p.coords.astype(np.float64)
    n0 = p.n0
    data = rng.standard_normal(N)
    dord = data[p.indices]

    def fwd(X):
        Ld = np.linalg.cholesky(_cov(p, X, np.arange(n0)))
        s = 0.5 * np.sum(np.linalg.solve(Ld, dord[:n0]) ** 2)

        def point(m, L, K):
            mv = np.linalg.solve(L[:K, :K].T, L[K, :K])
            xim = (dord[n0 + m] - mv @ dord[p.nbrs[m]]) / L[K, K]
            return 0.5 * xim * xim
        return s + _refined(p, X, point)

    gp = O.generate_inv_loss_grad_points(p, data)
    for (q, d) in ((2, 0), (11, 1), (n0 + 4, 0), (n0 + 59, 2), (n0 + 149, 1)):
        fd = _fd(fwd, X, q, d)
        assert abs(gp[q, d] - fd) <= 2e-3 * abs(fd) + 1e-6, (q, d, gp[q, d], fd)
