"""Covariance tables and the hyperparameter chain rule (src/extras.jl; test/test_extras.jl)."""
import numpy as np
import torch

import graphgp_b200 as gp


def test_make_cov_bins():
    bins = gp.make_cov_bins(1e-4, 1e1, 100)
    assert len(bins) == 100 and bins[0] == 0.0
    assert np.isclose(bins[-1], 10.0, rtol=1e-10) and np.all(np.diff(bins) > 0)


def test_rbf_kernel_vs_fixture(golden):
    # test/test_extras.jl:27-31: the JAX table at rtol 1e-8.
    d = golden("small")
    bins, vals = gp.rbf_kernel(1.0, 0.3, 1e-4, 1e1, 1000, jitter=1e-3)
    assert np.allclose(bins, d["cov_bins64"], rtol=1e-8)
    assert np.allclose(vals, d["cov_vals64"], rtol=1e-8)
    assert np.isclose(vals[0], 1.0 * (1 + 1e-3), rtol=1e-12)
    assert np.all(np.diff(vals[1:]) <= 0) and vals[-1] < 1e-4


def test_matern_kernel():
    for p in (1, 2, 3):
        bins, vals = gp.matern_kernel(p, 1.0, 0.5, 1e-4, 1e1, 200)
        assert len(vals) == 200 and np.all(np.isfinite(vals)) and np.all(vals >= 0)
        assert np.isclose(vals[0], 1.0, rtol=1e-8) and vals[-1] < 1e-2
    _, vj = gp.matern_kernel(1, 2.0, 0.5, 1e-4, 1e1, 50, jitter=0.1)
    assert np.isclose(vj[0], 2.2, rtol=1e-10)
    # nu = 3/2 closed form: (1 + sqrt(3) r / l) exp(-sqrt(3) r / l).
    b, v = gp.matern_kernel(1, 1.0, 0.05, 1e-5, 2.0, 2000)
    x = np.sqrt(3) * b / 0.05
    assert np.allclose(v, (1 + x) * np.exp(-x), rtol=1e-12)


def test_torch_tables_match_numpy():
    b0, v0 = gp.rbf_kernel(1.3, 0.2, 1e-4, 2.0, 300, jitter=1e-5)
    b1, v1 = gp.rbf_kernel(torch.tensor(1.3, dtype=torch.float64),
                           torch.tensor(0.2, dtype=torch.float64), 1e-4, 2.0, 300, jitter=1e-5)
    assert np.allclose(v0, v1.numpy(), rtol=1e-14)
    _, m0 = gp.matern_kernel(2, 0.7, 0.3, 1e-4, 2.0, 300)
    _, m1 = gp.matern_kernel(2, torch.tensor(0.7, dtype=torch.float64),
                             torch.tensor(0.3, dtype=torch.float64), 1e-4, 2.0, 300)
    assert np.allclose(m0, m1.numpy(), rtol=1e-14)


def test_hyperparam_grad_chain_rule():
    # J' g against central differences of g . vals(theta).
    rng = np.random.default_rng(0)
    g = rng.standard_normal(400)
    make = lambda var, sc: gp.rbf_kernel(var, sc, 1e-4, 1e1, 400, jitter=1e-3)  # noqa: E731
    th = np.array([1.2, 0.35])
    gh = gp.hyperparam_grad(g, make, th)
    for i in range(2):
        e = np.zeros(2)
        e[i] = 1e-6
        fd = (g @ make(*(th + e))[1] - g @ make(*(th - e))[1]) / 2e-6
        assert np.isclose(gh[i], fd, rtol=1e-6)
