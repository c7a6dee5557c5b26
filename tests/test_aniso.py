"""The anisotropic covariance (src/aniso.jl): the host checker pinned to the reference's own
checks (test/test_aniso.jl) and fixture (test/reference/aniso_parity.npz, compared at 1e-11 as
test/python_parity_aniso.jl does), and the CUDA path against both."""
from types import SimpleNamespace

import numpy as np
import pytest

from conftest import load_golden, relerr
from oracle import oracle as O


def _ref_aniso(ds, dz, sb, zb, grid):
    """The reference test's bilinear formula (test/test_aniso.jl:10-20)."""
    ns, nz = len(sb), len(zb)

    def fi(d, b, n):
        if d <= b[0]:
            return 0.0
        if d >= b[n - 1]:
            return float(n - 1)
        i = np.searchsorted(b, d, side="right") - 1
        return i + (d - b[i]) / (b[i + 1] - b[i])
    fx, fz = fi(ds, sb, ns), fi(dz, zb, nz)
    i0, j0 = int(np.floor(fx)), int(np.floor(fz))
    i1, j1 = min(i0 + 1, ns - 1), min(j0 + 1, nz - 1)
    tx, tz = fx - i0, fz - j0
    return ((grid[i0, j0] * (1 - tx) + grid[i1, j0] * tx) * (1 - tz)
            + (grid[i0, j1] * (1 - tx) + grid[i1, j1] * tx) * tz)


def _fixture_problem(dt):
    d = load_golden("aniso_parity")
    p = O.make_problem(d["coords"], d["neighbors"], d["offsets"], int(d["n0"]), d["scale"],
                       d["spatial_bins"], d["z_bins"], d["indices"], dt)
    cov = SimpleNamespace(spatial_bins=d["spatial_bins"], z_bins=d["z_bins"], grid=d["grid"],
                          alpha=float(d["alpha"]))
    return d, p, cov


def test_lookup_and_split():
    rng = np.random.default_rng(0xA115)
    sb = np.concatenate([[0.0], np.sort(rng.random(6) * 3)])
    zb = np.concatenate([[0.0], np.sort(rng.random(5) * 2)])
    grid = rng.random((len(sb), len(zb)))
    p = O.make_problem(np.zeros((2, 4), np.uint32), np.zeros((1, 1), np.int64), [1, 2], 1, 1.0,
                       sb, zb, None, np.float64)
    ds = rng.random(500) * 4 - 0.3
    dz = rng.random(500) * 2.5 - 0.2
    with O.anisotropic(p, SimpleNamespace(spatial_bins=sb, z_bins=zb, grid=grid, alpha=1.0)):
        got = O.aniso_lookup(p, ds, dz)
        assert O.aniso_lookup(p, 0.0, 0.0)[0] == grid[0, 0]
    ref = np.array([_ref_aniso(a, b, sb, zb, grid) for a, b in zip(ds, dz)])
    np.testing.assert_allclose(got, ref, rtol=1e-13, atol=1e-14)
    # The assembly splits spatial (first D-1) and radial (last) separations: two pairs at the
    # same 4-D lattice distance 3 get different covariances (test/test_aniso.jl:34-54).
    sbins = np.array([0, 1, 2, 3, 4.0])
    zbins = np.array([0, 0.5, 1, 1.5, 2.0])
    g = np.exp(-sbins[:, None] - 3 * zbins[None, :])
    coords = np.array([[0, 0, 0, 0], [3, 0, 0, 0], [0, 0, 0, 0], [0, 0, 0, 3]], np.uint32)
    q = O.make_problem(coords, np.zeros((0, 1), np.int64), [4], 4, 1.0, sbins, zbins, None,
                       np.float64)
    cov = SimpleNamespace(spatial_bins=sbins, z_bins=zbins, grid=g, alpha=2.0)
    with O.anisotropic(q, cov):
        Kd = O.dense_cov(q)
        assert Kd[0, 1] == O.aniso_lookup(q, 3.0, 0.0)[0]
        assert Kd[0, 3] == O.aniso_lookup(q, 0.0, 1.5)[0]
    assert abs(Kd[0, 1] - Kd[0, 3]) > 1e-3 * abs(Kd[0, 3])


def test_oracle_fixture():
    d, p, cov = _fixture_problem(np.float64)
    with O.anisotropic(p, cov):
        f = O.generate(p, d["xi"])
        xi = O.generate_inv(p, d["values"])
        back = O.generate_inv(p, f)
    assert relerr(f, d["generate_field"]) < 1e-11
    assert relerr(xi, d["generate_inv_xi"]) < 1e-11
    assert relerr(back, d["xi"]) < 1e-9


@pytest.mark.gpu
@pytest.mark.parametrize("dt", [np.float64, np.float32])
def test_aniso_gpu(cuda_device, dt):
    # generate and generate_grad_xi (the per-point factors, the exact-order dense factor and
    # mat-vecs) are the checker's bit for bit; generate_inv's dense layer multiplies by the kept
    # inverse of the factor (not the checker's forward substitution), and the log-determinant is
    # summed in another order, so those two agree to the tolerance, as in the isotropic tests.
    # The reverse sweep runs in its pull form, whose sums follow the serial sweep's order.
    import graphgp_b200 as gp
    tol = 1e-12 if dt == np.float64 else 1e-5
    d, p, cov = _fixture_problem(dt)
    acov = gp.AnisoCov(np.asarray(cov.spatial_bins, dt), np.asarray(cov.z_bins, dt),
                       np.asarray(cov.grid, dt), cov.alpha)
    prob = gp.GraphGPProblem.anisotropic(d["coords"], d["neighbors"], d["offsets"], int(d["n0"]),
                                         dt(d["scale"]), acov, d["indices"], dtype=dt)
    prob.set_reverse_mode(1)
    xi = d["xi"].astype(dt)
    vals = d["values"].astype(dt)
    vb = np.random.default_rng(4).standard_normal(len(xi)).astype(dt)
    f = np.asarray(gp.generate(prob, xi))
    x = np.asarray(gp.generate_inv(prob, vals))
    with O.anisotropic(p, cov):
        fo = O.generate(p, xi)
        xo = O.generate_inv(p, vals)
        lo = O.generate_logdet(p)
        go = O.generate_grad_xi(p, vb)
    assert np.array_equal(f, fo)
    assert relerr(x, xo) < tol
    assert abs(gp.generate_logdet(prob) - lo) <= tol * abs(lo)
    assert np.array_equal(np.asarray(gp.generate_grad_xi(prob, vb)), go)
    if dt == np.float64:
        assert relerr(f, d["generate_field"]) < 1e-11
        assert relerr(x, d["generate_inv_xi"]) < 1e-11
    with pytest.raises(gp.GraphGPError):
        gp.generate_grad_vals(prob, xi, vb)
