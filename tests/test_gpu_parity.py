"""Parity of the CUDA path (libgraphgp_b200.so through its C ABI) with the CPU oracle and with
the reference's golden vectors.

Bars: the forward refine and refine_inv kernels evaluate each point's arithmetic in the oracle's
exact order with IEEE round-to-nearest operations and no contraction, so they are compared BIT
FOR BIT.  Everything that sums in a different order (logdet sums, the dense block through
cuBLAS/cuSOLVER, atomic reverse sweeps and histograms) is compared by norm-relative error:
1e-12 in float64 and 1e-5 in float32, the tolerances of the drop-in target.
"""
import numpy as np
import pytest
import torch

import graphgp_b200 as gp
from conftest import relerr
from graphgp_b200 import _lib
from oracle import oracle as O

pytestmark = pytest.mark.gpu

TOL = {np.float64: 1e-12, np.float32: 1e-5}
FIXTURES = ["small", "medium", "generate_parity"]


def _tag(dt):
    return "64" if dt == np.float64 else "32"


def _pair(d, dt, with_indices=False):
    """(device problem, oracle problem) on the same arrays."""
    tag = _tag(dt) if f"cov_bins{_tag(dt)}" in d else "64"
    bins = d["cov_bins" + tag].astype(dt)
    vals = d["cov_vals" + tag].astype(dt)
    idx = d["indices"] if with_indices and "indices" in d else None
    prob = gp.GraphGPProblem(d["coords"], d["neighbors"], d["offsets"], int(d["n0"]),
                             dt(d["scale"]), bins, vals, idx, dtype=dt)
    orc = O.make_problem(d["coords"], d["neighbors"], d["offsets"], d["n0"], dt(d["scale"]),
                         bins, vals, idx, dt)
    return prob, orc


@pytest.fixture(autouse=True)
def _sweep_mode():
    _lib.lib().gpb2_set_forward_mode(0)
    yield
    _lib.lib().gpb2_set_forward_mode(0)


@pytest.mark.parametrize("dt", [np.float64, np.float32])
@pytest.mark.parametrize("name", FIXTURES)
@pytest.mark.parametrize("mode", [0, 1, 2, 3])
def test_refine_bit_exact(golden, cuda_device, name, dt, mode):
    d = golden(name)
    prob, orc = _pair(d, dt)
    rng = np.random.default_rng(1)
    iv = rng.standard_normal(prob.n0).astype(dt)
    xr = rng.standard_normal(prob.nrefined()).astype(dt)
    _lib.check(_lib.lib().gpb2_set_forward_mode(mode))
    v = gp.refine(prob, iv, xr)
    vo = O.refine(orc, iv, xr)
    assert np.array_equal(v, vo), relerr(v, vo)


@pytest.mark.parametrize("dt", [np.float64, np.float32])
@pytest.mark.parametrize("name", FIXTURES)
def test_refine_inv_bit_exact(golden, cuda_device, name, dt):
    d = golden(name)
    prob, orc = _pair(d, dt)
    vals = np.random.default_rng(2).standard_normal(prob.npoints()).astype(dt)
    assert np.array_equal(gp.refine_inv(prob, vals), O.refine_inv(orc, vals))


@pytest.mark.parametrize("dt", [np.float64, np.float32])
@pytest.mark.parametrize("name", ["small", "medium"])
def test_refine_vs_golden(golden, cuda_device, name, dt):
    # The reference's fixture values (test/test_refine.jl): f64 tight, f32 at its tolerance.
    d = golden(name)
    prob, _ = _pair(d, dt)
    t = _tag(dt)
    v = gp.refine(prob, d["initial_values" + t], d["xi_ref" + t])
    xi = gp.refine_inv(prob, d["values" + t])
    ld = gp.refine_logdet(prob)
    if dt == np.float64:
        assert relerr(v, d["refine_values64"]) < 1e-12
        assert relerr(xi, d["xi64"]) < 1e-12
        assert abs(ld - d["logdet64"]) < 1e-12 * abs(d["logdet64"])
    else:
        assert relerr(v, d["refine_values32"]) < 1e-4
        assert relerr(xi, d["xi32"]) < 1e-3
        assert abs(ld - d["logdet32"]) < 2e-3 * abs(d["logdet32"])


@pytest.mark.parametrize("dt", [np.float64, np.float32])
@pytest.mark.parametrize("name", FIXTURES)
def test_logdet_terms(golden, cuda_device, name, dt):
    d = golden(name)
    prob, orc = _pair(d, dt)
    terms = gp.refine_logdet_terms(prob)
    assert relerr(terms, O.refine_logdet_terms(orc)) < (1e-15 if dt == np.float64 else 1e-7)
    assert abs(gp.refine_logdet(prob) - O.refine_logdet(orc)) <= TOL[dt] * abs(O.refine_logdet(orc))


def test_generate_parity_golden(golden, cuda_device):
    # test/python_parity_generate.jl: generate / generate_inv in ORIGINAL order at 1e-12.
    d = golden("generate_parity")
    prob, orc = _pair(d, np.float64, with_indices=True)
    f = gp.generate(prob, d["xi"])
    assert relerr(f, d["generate_field"]) < 1e-12
    assert relerr(gp.generate_inv(prob, d["values"]), d["generate_inv_xi"]) < 1e-12
    assert relerr(gp.generate_inv(prob, f), d["xi"]) < 1e-10
    assert relerr(f, O.generate(orc, d["xi"])) < 1e-12


@pytest.mark.parametrize("dt", [np.float64, np.float32])
@pytest.mark.parametrize("name", FIXTURES)
def test_generate_ops_vs_oracle(golden, cuda_device, name, dt):
    d = golden(name)
    prob, orc = _pair(d, dt, with_indices=True)
    N = prob.npoints()
    rng = np.random.default_rng(3)
    xi = rng.standard_normal(N).astype(dt)
    vb = rng.standard_normal(N).astype(dt)
    tol = TOL[dt]
    f = gp.generate(prob, xi)
    assert relerr(f, O.generate(orc, xi)) < tol
    assert relerr(gp.generate_inv(prob, f), O.generate_inv(orc, f)) < tol
    lo = O.generate_logdet(orc)
    assert abs(gp.generate_logdet(prob) - lo) <= tol * abs(lo)
    assert relerr(gp.generate_grad_xi(prob, vb), O.generate_grad_xi(orc, vb)) < tol
    assert relerr(gp.generate_grad_vals(prob, xi, vb), O.generate_grad_vals(orc, xi, vb)) < tol


@pytest.mark.parametrize("dt", [np.float64, np.float32])
@pytest.mark.parametrize("name", ["small", "medium"])
def test_vals_gradients(golden, cuda_device, name, dt):
    d = golden(name)
    prob, orc = _pair(d, dt)
    tol = TOL[dt]
    ld_o, g_o = O.refine_logdet_grad_vals(orc)
    g = gp.refine_logdet_grad_vals(prob)
    assert relerr(g, g_o) < tol
    ld, gg = gp.generate_logdet_and_grad_vals(prob)
    assert relerr(gg, O.generate_logdet_grad_vals(orc)) < tol
    assert abs(ld - O.generate_logdet(orc)) <= tol * abs(ld)
    t = _tag(dt)
    loss, gi = gp.refine_inv_loss_grad_vals(prob, d["values" + t])
    loss_o, gi_o = O.refine_inv_loss_grad_vals(orc, d["values" + t])
    assert abs(loss - loss_o) <= tol * abs(loss_o)
    assert relerr(gi, gi_o) < tol
    if dt == np.float64:  # the reference's JAX gradients (test/test_gradients.jl)
        nz = d["grad_logdet_vals64"] != 0
        assert relerr(g[nz], d["grad_logdet_vals64"][nz]) < 1e-12
        nz = d["grad_inv_loss_vals64"] != 0
        assert relerr(gi[nz], d["grad_inv_loss_vals64"][nz]) < 1e-12
        assert abs(loss - d["inv_loss64"]) < 1e-12 * d["inv_loss64"]


def test_generate_inv_loss_dense_part(golden, cuda_device):
    d = golden("small")
    prob, orc = _pair(d, np.float64)
    data = d["values64"]
    loss, g = gp.generate_inv_loss_grad_vals(prob, data)
    # dense part: 0.5*||L^-1 y||^2 and its gradient through K^-1 y (src/dense.jl:244-266).
    L, _ = O.dense_chol(orc)
    z = O.generate_dense_inv(L, data[: prob.n0])
    loss_ref = 0.5 * float(z @ z) + O.refine_inv_loss_grad_vals(orc, data)[0]
    assert abs(loss - loss_ref) <= 1e-12 * abs(loss_ref)
    # FD of the loss w.r.t. a few vals entries (f64 problem).
    for i in (0, 7, 60):
        h = 1e-6
        e = h * (np.arange(prob.nbins()) == i)
        lp = gp.generate_inv_loss_grad_vals(gp.set_vals(prob, prob.vals + e), data)[0]
        lm = gp.generate_inv_loss_grad_vals(gp.set_vals(prob, prob.vals - e), data)[0]
        assert np.isclose(g[i], (lp - lm) / (2 * h), rtol=1e-5, atol=1e-3 * abs(g).max() * 1e-6)


def _config_problem(N, D, n0, k, dt, seed, kernel="rbf"):
    rng = np.random.default_rng(seed)
    pts = rng.standard_normal((N, D))
    if kernel == "rbf":
        bins, vals = gp.rbf_kernel(1.0, 0.3, 1e-4, 10.0, 1000, jitter=1e-5)
    else:
        bins, vals = gp.matern_kernel(1, 1.0, 0.05, 1e-5, 2.0, 2000, jitter=1e-5)
    g = gp.build_graph_arrays(pts, n0, k)
    prob = gp.GraphGPProblem(g["coords"], g["neighbors"], g["offsets"], g["n0"],
                             dt(g["scale"]), bins.astype(dt), vals.astype(dt), g["indices"],
                             dtype=dt)
    orc = O.make_problem(g["coords"], g["neighbors"], g["offsets"], g["n0"], dt(g["scale"]),
                         bins.astype(dt), vals.astype(dt), g["indices"], dt)
    return prob, orc


def test_config1_f64(cuda_device):
    # BASELINE config 1 shape: N=10000, D=2, n0=100, k=10, RBF(1, 0.3, 1e-4..10, 1000 bins,
    # jitter 1e-5), f64; ops generate / generate_inv / generate_logdet.
    prob, orc = _config_problem(10_000, 2, 100, 10, np.float64, 99)
    xi = np.random.default_rng(7).standard_normal(prob.npoints())
    f = gp.generate(prob, xi)
    assert relerr(f, O.generate(orc, xi)) < 1e-12
    assert relerr(gp.generate_inv(prob, f), xi) < 1e-8
    lo = O.generate_logdet(orc)
    assert abs(gp.generate_logdet(prob) - lo) < 1e-12 * abs(lo)


@pytest.mark.parametrize("K,D,kernel", [(8, 2, "rbf"), (8, 3, "rbf"), (16, 3, "matern"),
                                        (6, 3, "rbf"), (4, 2, "rbf"), (12, 2, "rbf")])
def test_supported_shapes_f32(cuda_device, K, D, kernel):
    prob, orc = _config_problem(6000, D, 200, K, np.float32, 11 + K + D, kernel)
    rng = np.random.default_rng(4)
    xi = rng.standard_normal(prob.npoints()).astype(np.float32)
    vb = rng.standard_normal(prob.npoints()).astype(np.float32)
    f = gp.generate(prob, xi)
    assert relerr(f, O.generate(orc, xi)) < 1e-5
    assert relerr(gp.generate_grad_xi(prob, vb), O.generate_grad_xi(orc, vb)) < 1e-5
    assert relerr(gp.generate_grad_vals(prob, xi, vb), O.generate_grad_vals(orc, xi, vb)) < 1e-5
    assert relerr(gp.refine_logdet_grad_vals(prob), O.refine_logdet_grad_vals(orc)[1]) < 1e-5


@pytest.mark.parametrize("dt", [np.float64, np.float32])
def test_dense_jitter_ladder(cuda_device, dt):
    # The config-2 root block (n0 = 1000 spread tree medians, RBF scale 0.3, jitter 1e-5) is
    # indefinite as a matrix of interpolated covariances, so the reference's ladder
    # (src/dense.jl:46-67) must step up to eps = 1e-3.  The device factorisation must take the
    # same step as the oracle and, being exact-order, produce the same field.
    prob, orc = _config_problem(20_000, 2, 1000, 8, dt, 1)
    xi = np.random.default_rng(2).standard_normal(prob.npoints()).astype(dt)
    f = gp.generate(prob, xi)
    _, jit_o = O.dense_chol(orc)
    assert jit_o > 0
    assert np.isclose(prob.dense_jitter(), jit_o, rtol=1e-6)
    assert relerr(f, O.generate(orc, xi)) < TOL[dt]


@pytest.mark.parametrize("dt", [np.float64, np.float32])
@pytest.mark.parametrize("n0,N", [(1000, 20_000), (200, 3000), (37, 1000)])
def test_dense_factor_bit_exact(cuda_device, dt, n0, N):
    # The device's blocked, ladder-speculative Cholesky applies each entry's subtractions in the
    # oracle's order: the factor (and the ladder step) must be identical bit for bit.
    prob, orc = _config_problem(N, 2, n0, 8, dt, 5)
    gp.generate_logdet(prob)
    L_dev = prob.dense_factor()
    L_ora, jit = O.dense_chol(orc)
    assert np.isclose(prob.dense_jitter(), jit, rtol=1e-6)
    assert np.array_equal(L_dev, np.tril(L_ora))


@pytest.mark.parametrize("dt", [np.float64, np.float32])
def test_update_vals_refactors(cuda_device, dt):
    # The handle reuses the dense factor across calls until the table changes; a new table must
    # give exactly what a fresh handle (and the oracle) gives for it, and switching back must
    # reproduce the first result bit for bit.
    prob, _ = _config_problem(3000, 2, 200, 8, dt, 21)
    xi = np.random.default_rng(8).standard_normal(prob.npoints()).astype(dt)
    f1 = gp.generate(prob, xi)
    f1b = gp.generate(prob, xi)  # reuses the factor
    assert np.array_equal(f1, f1b)
    bins_b, vals_b = gp.rbf_kernel(1.3, 0.5, 1e-4, 10.0, 1000, jitter=1e-5)
    assert np.allclose(bins_b.astype(dt), prob.bins)
    prob.update_vals(vals_b.astype(dt))
    f2 = gp.generate(prob, xi)
    L2 = prob.dense_factor()
    fresh = gp.set_vals(prob, vals_b.astype(dt))
    assert np.array_equal(f2, gp.generate(fresh, xi))
    orc_b = O.make_problem(prob.coords, prob.neighbors, prob.offsets, prob.n0, dt(prob.scale),
                           prob.bins, vals_b.astype(dt), prob.indices, dt)
    L_ora, _ = O.dense_chol(orc_b)
    assert np.array_equal(L2, np.tril(L_ora))
    assert relerr(f2, O.generate(orc_b, xi)) < TOL[dt]
    prob.update_vals(gp.rbf_kernel(1.0, 0.3, 1e-4, 10.0, 1000, jitter=1e-5)[1].astype(dt))
    assert np.array_equal(gp.generate(prob, xi), f1)


@pytest.mark.parametrize("dt", [np.float64, np.float32])
def test_prefactor(cuda_device, dt):
    # prefactor() queues a new table's factorisations without waiting; the operations that
    # follow use them (the same results as without it), and a dense block that no jitter step
    # factorises is reported by the next operation -- again by the one after, on the same
    # table -- while a good table afterwards works as before.  (Synchronous calls: the status
    # of each call is what is checked.)
    gp.set_synchronous(True)
    prob, orc = _config_problem(3000, 2, 200, 8, dt, 21)
    rng = np.random.default_rng(8)
    xi = rng.standard_normal(prob.npoints()).astype(dt)
    vb = rng.standard_normal(prob.npoints()).astype(dt)
    f0 = gp.generate(prob, xi)
    g0 = gp.generate_grad_vals(prob, xi, vb)
    good = np.array(prob.vals, copy=True)
    prob.update_vals(good).prefactor()
    assert np.array_equal(gp.generate(prob, xi), f0)
    assert np.array_equal(prob.dense_factor(), np.tril(O.dense_chol(orc)[0]))
    assert relerr(gp.generate_grad_vals(prob, xi, vb), g0) < TOL[dt]
    prob.update_vals(-good).prefactor()  # negative variances: no jitter step helps
    for _ in range(2):
        with pytest.raises(_lib.GraphGPError) as e:
            gp.generate(prob, xi)
        assert e.value.status == _lib.GPB2_ERR_NOT_PD
    prob.update_vals(good)
    assert np.array_equal(gp.generate(prob, xi), f0)


@pytest.fixture
def _async_mode():
    gp.set_synchronous(False)
    yield
    gp.set_synchronous(True)


@pytest.mark.parametrize("dt", [np.float64, np.float32])
def test_asynchronous_calls(cuda_device, dt, _async_mode):
    # With set_synchronous(False) the operations only queue their work; the results are the
    # synchronous ones, and a dense block that no jitter step factorises is reported by
    # check(), not by the operation.
    prob, _ = _config_problem(3000, 2, 200, 8, dt, 21)
    rng = np.random.default_rng(8)
    xi_h = rng.standard_normal(prob.npoints()).astype(dt)
    vb_h = rng.standard_normal(prob.npoints()).astype(dt)
    xi = torch.from_numpy(xi_h).to(prob.device)
    vb = torch.from_numpy(vb_h).to(prob.device)
    good = np.array(prob.vals, copy=True)
    prob.update_vals(good).prefactor()
    f = gp.generate(prob, xi)
    gx = gp.generate_grad_xi(prob, vb)
    gv = gp.generate_grad_vals(prob, xi, vb)
    prob.check()
    gp.set_synchronous(True)
    assert np.array_equal(f.cpu().numpy(), gp.generate(prob, xi_h))
    assert np.array_equal(gx.cpu().numpy(), gp.generate_grad_xi(prob, vb_h)) or \
        relerr(gx.cpu().numpy(), gp.generate_grad_xi(prob, vb_h)) < TOL[dt]
    assert relerr(gv.cpu().numpy(), gp.generate_grad_vals(prob, xi_h, vb_h)) < TOL[dt]
    gp.set_synchronous(False)
    prob.update_vals(-good).prefactor()  # negative variances: no jitter step helps
    gp.generate(prob, xi)                # queued; the status comes with check()
    with pytest.raises(_lib.GraphGPError) as e:
        prob.check()
    assert e.value.status == _lib.GPB2_ERR_NOT_PD
    prob.update_vals(good)
    f2 = gp.generate(prob, xi)
    prob.check()
    assert np.array_equal(f2.cpu().numpy(), f.cpu().numpy())


@pytest.mark.parametrize("dt", [np.float64, np.float32])
def test_inverse_readers_right_after_prefactor(cuda_device, dt, _async_mode):
    # The triangular preparation (row-major copy of L, L^-1) is queued on the dense stream
    # after the prefactor's join; every reader queued straight after it (L^T x, products with
    # L^-1, K^-1) must order itself after it: the results equal those of synchronous calls on
    # a handle whose preparation had long finished.
    prob, _ = _config_problem(3000, 2, 200, 8, dt, 23)
    rng = np.random.default_rng(9)
    v_h = rng.standard_normal(prob.npoints()).astype(dt)
    vb_h = rng.standard_normal(prob.npoints()).astype(dt)
    v = torch.from_numpy(v_h).to(prob.device)
    vb = torch.from_numpy(vb_h).to(prob.device)
    good = np.array(prob.vals, copy=True)
    got = {}
    for name, call in (("inv", lambda: gp.generate_inv(prob, v)),
                       ("gxi", lambda: gp.generate_grad_xi(prob, vb)),
                       ("ldg", lambda: gp.generate_logdet_grad_vals(prob)),
                       ("ilg", lambda: gp.generate_inv_loss_grad_vals(prob, v)[1])):
        prob.update_vals(good).prefactor()
        got[name] = call()
        prob.check()
    gp.set_synchronous(True)
    want = {"inv": gp.generate_inv(prob, v_h), "gxi": gp.generate_grad_xi(prob, vb_h),
            "ldg": gp.generate_logdet_grad_vals(prob),
            "ilg": gp.generate_inv_loss_grad_vals(prob, v_h)[1]}
    assert np.array_equal(got["inv"].cpu().numpy(), want["inv"])
    for k in ("gxi", "ldg", "ilg"):
        g = got[k].cpu().numpy() if hasattr(got[k], "cpu") else got[k]
        assert relerr(g, want[k]) < TOL[dt], k


@pytest.mark.parametrize("dt", [np.float64, np.float32])
def test_grad_vals_repeated_and_after_refactor(cuda_device, dt):
    # Repeated vals-gradients on one handle, before and after the table is re-set (which
    # refactors the dense block and the per-point factors), must agree with each other and with
    # the oracle.
    prob, orc = _config_problem(5000, 2, 200, 8, dt, 33)
    rng = np.random.default_rng(9)
    xi = rng.standard_normal(prob.npoints()).astype(dt)
    vb = rng.standard_normal(prob.npoints()).astype(dt)
    g1 = gp.generate_grad_vals(prob, xi, vb)
    prob.update_vals(prob.vals)                        # same table: everything refactorised
    g2 = gp.generate_grad_vals(prob, xi, vb)
    g3 = gp.generate_grad_vals(prob, xi, vb)          # reuses the factors
    g_o = O.generate_grad_vals(orc, xi, vb)
    # (the reverse sweep's float atomics make repeated f32 gradients differ at ~1e-6)
    assert relerr(g2, g1) < TOL[dt]
    assert relerr(g3, g2) < TOL[dt]
    assert relerr(g2, g_o) < TOL[dt]


@pytest.mark.parametrize("dt", [np.float64, np.float32])
def test_dense_ladder_sequential_launches(cuda_device, dt, monkeypatch):
    # Above the speculation limit the ladder runs one candidate per launch, reusing one slot; the
    # step it settles on and the factor must be the same as the oracle's (the config-2 root block
    # needs eight launches: eps = 0, 1e-9, ..., 1e-3).
    monkeypatch.setenv("GPB2_DENSE_SPEC_MAX", "0")
    prob, orc = _config_problem(20_000, 2, 1000, 8, dt, 1)
    gp.generate_logdet(prob)
    L_ora, jit = O.dense_chol(orc)
    assert jit > 0
    assert np.isclose(prob.dense_jitter(), jit, rtol=1e-6)
    assert np.array_equal(prob.dense_factor(), np.tril(L_ora))


@pytest.mark.parametrize("dt", [np.float64, np.float32])
def test_dense_large_tile_and_ladder_switch(cuda_device, dt, monkeypatch):
    # The large trailing tile (the default above n0 = 2048) gives the oracle's factor bit for bit
    # at n0 = 1000 too; one handle switched between one-candidate-per-launch and speculative
    # ladders (which need different candidate buffers) refactors correctly each time.
    monkeypatch.setenv("GPB2_CHOL_TILE", "128" if dt == np.float32 else "64")
    prob, orc = _config_problem(20_000, 2, 1000, 8, dt, 1)
    L_ora, jit = O.dense_chol(orc)
    for spec in ("0", "4096", "0"):
        monkeypatch.setenv("GPB2_DENSE_SPEC_MAX", spec)
        prob.update_vals(prob.vals)  # same table: the dense block is refactorised
        gp.generate_logdet(prob)
        assert np.isclose(prob.dense_jitter(), jit, rtol=1e-6)
        assert np.array_equal(prob.dense_factor(), np.tril(L_ora))


@pytest.mark.parametrize("dt", [np.float64, np.float32])
def test_dense_whole_gpu_ladder(cuda_device, dt, monkeypatch):
    # The whole-GPU form (one candidate per cooperative launch, every SM on its trailing
    # update; the default above n0 = 2048) forced onto the config-2 root block: eight launches
    # in ladder order, the same step and the same factor bit for bit as the oracle.
    monkeypatch.setenv("GPB2_DENSE_GRID_MIN", "0")
    prob, orc = _config_problem(20_000, 2, 1000, 8, dt, 1)
    gp.generate_logdet(prob)
    L_ora, jit = O.dense_chol(orc)
    assert jit > 0
    assert np.isclose(prob.dense_jitter(), jit, rtol=1e-6)
    assert np.array_equal(prob.dense_factor(), np.tril(L_ora))


@pytest.mark.parametrize("dt", [np.float64, np.float32])
def test_dense_whole_gpu_large(cuda_device, dt):
    # A first layer above the switch (n0 = 3000, D = 3): bit for bit as the oracle.
    prob, orc = _config_problem(60_000, 3, 3000, 8, dt, 21)
    gp.generate_logdet(prob)
    L_ora, jit = O.dense_chol(orc)
    assert np.isclose(prob.dense_jitter(), jit, rtol=1e-6)
    assert np.array_equal(prob.dense_factor(), np.tril(L_ora))


def test_degenerate_duplicates(cuda_device):
    # test/test_degenerate.jl: 30 exact duplicate points must give finite results everywhere.
    rng = np.random.default_rng(0xDEAD)
    n, D, n0, k = 5000, 3, 128, 10
    p = rng.uniform(size=(n, D))
    p[200:230] = p[:30]
    bins = np.linspace(0, 2, 200)
    vals = np.exp(-bins ** 1.5)
    vals[0] *= 1.001
    g = gp.build_graph_arrays(p, n0, k)
    prob = gp.GraphGPProblem(g["coords"], g["neighbors"], g["offsets"], g["n0"], g["scale"],
                             bins, vals, g["indices"])
    orc = O.make_problem(g["coords"], g["neighbors"], g["offsets"], g["n0"], g["scale"], bins,
                         vals, g["indices"], np.float64)
    xi = rng.standard_normal(n)
    f = gp.generate(prob, xi)
    assert np.all(np.isfinite(f))
    assert np.all(np.isfinite(gp.generate_inv(prob, f)))
    assert np.all(np.isfinite(gp.generate_grad_xi(prob, rng.standard_normal(n))))
    assert np.isfinite(gp.generate_logdet(prob))
    assert relerr(f, O.generate(orc, xi)) < 1e-12


def test_torch_tensors_in_and_out(golden, cuda_device):
    d = golden("generate_parity")
    prob, orc = _pair(d, np.float64, with_indices=True)
    xi = torch.from_numpy(d["xi"]).to(cuda_device)
    f = gp.generate(prob, xi)
    assert isinstance(f, torch.Tensor) and f.is_cuda
    assert relerr(f.cpu().numpy(), d["generate_field"]) < 1e-12


def test_autodiff_generate_of_vals(golden, cuda_device):
    d = golden("generate_parity")
    prob, orc = _pair(d, np.float64, with_indices=True)
    vals = torch.from_numpy(prob.vals.copy()).to(cuda_device).requires_grad_(True)
    xi = torch.from_numpy(d["xi"]).to(cuda_device).requires_grad_(True)
    w = torch.from_numpy(np.random.default_rng(5).standard_normal(len(d["xi"]))).to(cuda_device)
    (w * gp.generate_of_vals(prob, vals, xi)).sum().backward()
    wn = w.cpu().numpy()
    assert relerr(vals.grad.cpu().numpy(), O.generate_grad_vals(orc, d["xi"], wn)) < 1e-12
    assert relerr(xi.grad.cpu().numpy(), O.generate_grad_xi(orc, wn)) < 1e-12


def test_invalid_graph_rejected(golden, cuda_device):
    d = golden("small")
    nb = d["neighbors"].copy()
    nb[5, 0] = d["n0"] + 5  # a point that is its own neighbour (not in an earlier batch)
    prob = gp.GraphGPProblem(d["coords"], nb, d["offsets"], int(d["n0"]), d["scale"],
                             d["cov_bins64"], d["cov_vals64"])
    with pytest.raises(gp.GraphInvariantError):
        gp.check_graph(prob)


def test_unsupported_k_rejected(cuda_device):
    rng = np.random.default_rng(1)
    g = gp.build_graph_arrays(rng.standard_normal((500, 2)), 40, 7)
    bins, vals = gp.rbf_kernel(1.0, 0.3, 1e-4, 10.0, 100, jitter=1e-3)
    prob = gp.GraphGPProblem(g["coords"], g["neighbors"], g["offsets"], g["n0"], g["scale"],
                             bins, vals)
    with pytest.raises(gp.UnsupportedError):
        gp.generate_logdet(prob)


def test_large_roundtrip_and_linearity_f32(cuda_device):
    # Size-independent properties at a BASELINE config 2 scale (N = 10^6, D = 2, k = 8, f32):
    # generate_inv(generate(xi)) ~ xi and the adjoint identity <vb, G xi> = <G^T vb, xi>.
    rng = np.random.default_rng(1)
    pts = rng.standard_normal((1_000_000, 2))
    g = gp.build_graph_arrays(pts, 1000, 8)
    bins, vals = gp.rbf_kernel(1.0, 0.3, 1e-4, 10.0, 1000, jitter=1e-5)
    prob = gp.GraphGPProblem(g["coords"], g["neighbors"], g["offsets"], g["n0"],
                             np.float32(g["scale"]), bins.astype(np.float32),
                             vals.astype(np.float32), g["indices"])
    xi = torch.from_numpy(rng.standard_normal(1_000_000).astype(np.float32)).to(cuda_device)
    vb = torch.from_numpy(rng.standard_normal(1_000_000).astype(np.float32)).to(cuda_device)
    f = gp.generate(prob, xi)
    back = gp.generate_inv(prob, f)
    assert relerr(back.cpu().numpy(), xi.cpu().numpy()) < 1e-3
    lhs = float(torch.dot(vb.double(), f.double()))
    rhs = float(torch.dot(gp.generate_grad_xi(prob, vb).double(), xi.double()))
    assert abs(lhs - rhs) <= 1e-4 * abs(lhs)
    dv = gp.generate_grad_vals(prob, xi, vb)
    assert torch.isfinite(dv).all()


@pytest.mark.parametrize("dt", [np.float64, np.float32])
@pytest.mark.parametrize("shift,offset", [("12", 0), (None, 0), (None, 1)])
def test_two_pass_permutation(cuda_device, dt, shift, offset, monkeypatch):
    # The two-pass original <-> library permutation of large fields (forced here on a 3e5-point
    # problem; 4096-value destination blocks give 74 blocks, the default 64 KB ones 19 or 37, the
    # last one partial) gives the direct gather / scatter's results bit for bit -- also from and
    # into caller arrays that are not 16-byte aligned (offset 1: the element-wise form).
    if shift is not None:
        monkeypatch.setenv("GPB2_PERM_BLOCK_SHIFT", shift)
    prob, orc = _config_problem(300_000, 2, 500, 8, dt, 9)
    rng = np.random.default_rng(3)
    n = prob.npoints()
    xi = torch.from_numpy(rng.standard_normal(n + offset).astype(dt)).to(cuda_device)[offset:]
    vb = torch.from_numpy(rng.standard_normal(n + offset).astype(dt)).to(cuda_device)[offset:]
    monkeypatch.setenv("GPB2_PERM_TWO_PASS_MIN", str(1 << 40))
    ref = (gp.generate(prob, xi), gp.generate_inv(prob, xi), gp.generate_grad_xi(prob, vb))
    monkeypatch.setenv("GPB2_PERM_TWO_PASS_MIN", "0")
    got = [torch.empty(n + offset, dtype=xi.dtype, device=cuda_device)[offset:] for _ in range(3)]
    for fn, x, o in (("gpb2_generate", xi, got[0]), ("gpb2_generate_inv", xi, got[1]),
                     ("gpb2_generate_grad_xi", vb, got[2])):
        gp.api._call(fn, prob.handle, gp.api._ptr(x), gp.api._ptr(o), gp.api._stream(prob))
    torch.cuda.synchronize(cuda_device)
    assert torch.equal(got[0], ref[0])
    assert torch.equal(got[1], ref[1])
    # The reverse sweep's atomic sums are not reproducible bit for bit from run to run.
    assert relerr(got[2].cpu().numpy(), ref[2].cpu().numpy()) < TOL[dt]


@pytest.mark.parametrize("dt", [np.float64, np.float32])
def test_library_order(cuda_device, dt, monkeypatch):
    # Inside the handle every depth batch is re-sorted by Morton code.  The maps are a
    # within-batch permutation (identity on the dense block), and every result -- in original
    # order and through the tree-order refine entry points -- is the one the reference's tree
    # order gives, bit for bit where the arithmetic has a fixed order.
    prob, orc = _config_problem(120_000, 3, 700, 8, dt, 13)
    monkeypatch.setenv("GPB2_TREE_ORDER", "1")
    ref = gp.GraphGPProblem(prob.coords, prob.neighbors, prob.offsets, prob.n0, prob.scale,
                            prob.bins, prob.vals, prob.indices, dtype=dt)
    ref.handle
    monkeypatch.delenv("GPB2_TREE_ORDER")
    lt, lo = (t.cpu().numpy() for t in prob.library_order())
    n0 = prob.n0
    assert np.array_equal(lt[:n0], np.arange(n0))
    offs = prob.offsets
    for a, b in zip(offs[:-1], offs[1:]):
        assert np.array_equal(np.sort(lt[a:b]), np.arange(a, b))
    assert np.array_equal(lo, prob.indices[lt])
    assert not np.array_equal(lt, np.arange(len(lt)))  # the order did change
    rng = np.random.default_rng(4)
    xi = rng.standard_normal(prob.npoints()).astype(dt)
    iv = rng.standard_normal(n0).astype(dt)
    xr = rng.standard_normal(prob.nrefined()).astype(dt)
    f = gp.generate(prob, xi)
    assert np.array_equal(f, gp.generate(ref, xi))
    assert np.array_equal(gp.generate_inv(prob, f), gp.generate_inv(ref, f))
    v = gp.refine(prob, iv, xr)
    assert np.array_equal(v, gp.refine(ref, iv, xr))
    assert np.array_equal(v, O.refine(orc, iv, xr))
    assert np.array_equal(gp.refine_inv(prob, v), gp.refine_inv(ref, v))
    assert np.array_equal(gp.refine_logdet_terms(prob), gp.refine_logdet_terms(ref))
    l1, l2 = gp.refine_inv_loss_grad_vals(prob, v), gp.refine_inv_loss_grad_vals(ref, v)
    assert abs(l1[0] - l2[0]) <= TOL[dt] * abs(l2[0]) and relerr(l1[1], l2[1]) < TOL[dt]
    assert abs(gp.generate_logdet(prob) - gp.generate_logdet(ref)) <= \
        TOL[dt] * abs(gp.generate_logdet(ref))


@pytest.mark.parametrize("dt", [np.float64, np.float32])
def test_factor_cache(cuda_device, dt):
    # The vals-gradients that read each point's factor and pair weights from the factor cache
    # agree with the ones that recompute them and with the host checker, before and after a
    # table change (the cache is refilled by the new table's factor pass).  The cached entries
    # are the recomputation's bits; the histogram sums are atomic, hence the tolerance.
    prob, orc = _config_problem(60_000, 3, 300, 8, dt, 17)
    rng = np.random.default_rng(5)
    xi = rng.standard_normal(prob.npoints()).astype(dt)
    vb = rng.standard_normal(prob.npoints()).astype(dt)
    y = gp.generate(prob, xi)

    def grads():
        return (gp.generate_grad_vals(prob, xi, vb), gp.refine_logdet_grad_vals(prob),
                gp.refine_inv_loss_grad_vals(prob, y))

    prob.set_factor_cache(0)
    assert not prob.factor_cache()["valid"]
    ref = grads()
    prob.set_factor_cache(1)
    got = grads()
    info = prob.factor_cache()
    assert info["valid"] and info["mode"] == 1
    assert info["bytes"] == (prob.npoints() - prob.n0) * (45 * dt().itemsize + 36 * (dt().itemsize + 2))
    def flat(r):  # a gradient, or a (scalar, gradient) pair
        parts = r if isinstance(r, tuple) else (r,)
        return np.concatenate([np.atleast_1d(np.asarray(x, dtype=np.float64)) for x in parts])

    for a, b in zip(got, ref):
        assert relerr(flat(a), flat(b)) < TOL[dt]
    assert relerr(np.asarray(got[0]), O.generate_grad_vals(orc, xi, vb)) < TOL[dt]
    # A new table: the factor pass of the next call refills the cache.
    _, vals2 = gp.rbf_kernel(1.3, 0.25, 1e-4, 10.0, 1000, jitter=1e-5)
    prob.update_vals(vals2.astype(dt))
    assert not prob.factor_cache()["valid"]
    got2 = gp.generate_grad_vals(prob, xi, vb)
    assert prob.factor_cache()["valid"]
    orc2 = O.make_problem(orc.coords, orc.nbrs, orc.offsets, orc.n0, orc.scale, orc.bins,
                          vals2.astype(dt), orc.indices, dt)
    assert relerr(np.asarray(got2), O.generate_grad_vals(orc2, xi, vb)) < TOL[dt]
    prob.set_factor_cache(0)
    assert not prob.factor_cache()["valid"]
    assert relerr(np.asarray(gp.generate_grad_vals(prob, xi, vb)), np.asarray(got2)) < TOL[dt]


@pytest.mark.parametrize("dt", [np.float64, np.float32])
def test_reverse_pull_bit_exact(cuda_device, dt):
    # The pull-form reverse sweep adds every point's incoming terms in the serial reference
    # sweep's order (descending tree order of the child, slot order), so generate_grad_xi is the
    # host checker's bit for bit and the same from run to run; the atomic push agrees to the
    # tolerance.  generate_grad_vals (atomic histogram) agrees to the tolerance in both forms.
    prob, orc = _config_problem(80_000, 2, 400, 8, dt, 23)
    rng = np.random.default_rng(8)
    n = prob.npoints()
    xi = rng.standard_normal(n).astype(dt)
    vb = rng.standard_normal(n).astype(dt)
    prob.set_reverse_mode(1)
    g = np.asarray(gp.generate_grad_xi(prob, vb))
    info = prob.reverse_mode()
    assert info["built"] and info["mode"] == 1
    assert info["bytes"] == (n - prob.n0) * 8 * (4 + dt().itemsize) + 4 * (n + 1)
    ref = O.generate_grad_xi(orc, vb)
    assert np.array_equal(g, ref), relerr(g, ref)
    assert np.array_equal(np.asarray(gp.generate_grad_xi(prob, vb)), g)
    dv = np.asarray(gp.generate_grad_vals(prob, xi, vb))
    assert relerr(dv, O.generate_grad_vals(orc, xi, vb)) < TOL[dt]
    prob.set_reverse_mode(0)
    assert not prob.reverse_mode()["built"]
    assert relerr(np.asarray(gp.generate_grad_xi(prob, vb)), ref) < TOL[dt]
    assert relerr(np.asarray(gp.generate_grad_vals(prob, xi, vb)), dv) < TOL[dt]


@pytest.mark.parametrize("dt", [np.float64, np.float32])
def test_points_gradients(cuda_device, dt):
    # Point-position gradients -- refine_ and generate_ forms of the log-determinant's and of
    # the inverse loss's -- against the host checker (itself pinned by finite differences of a
    # continuous-position forward), (N, D) in tree order.  The pairs' terms are added
    # atomically, hence the tolerance.
    prob, orc = _config_problem(30_000, 3, 200, 8, dt, 31)
    rng = np.random.default_rng(9)
    n = prob.npoints()
    data = rng.standard_normal(n).astype(dt)
    vt = data[orc.indices]
    g = np.asarray(gp.refine_logdet_grad_points(prob))
    assert g.shape == (n, 3)
    assert relerr(g, O.refine_logdet_grad_points(orc)) < TOL[dt]
    assert relerr(np.asarray(gp.generate_logdet_grad_points(prob)),
                  O.generate_logdet_grad_points(orc)) < TOL[dt]
    assert relerr(np.asarray(gp.refine_inv_loss_grad_points(prob, vt)),
                  O.refine_inv_loss_grad_points(orc, vt)) < TOL[dt]
    assert relerr(np.asarray(gp.generate_inv_loss_grad_points(prob, data)),
                  O.generate_inv_loss_grad_points(orc, data)) < TOL[dt]
