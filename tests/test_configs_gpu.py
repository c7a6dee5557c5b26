"""Parity of the CUDA path with the oracle on the benchmark configurations' own inputs.

C2 and C3 run at their full sizes (1e6 and 1e7 points); C4 and C5 run their distributions
(blob mixture in the unit cube, uniform in the unit square), first layers (n0 = 5000 and 10^4)
and tables at sizes the host oracle finishes in minutes.  A density-matched C5 window puts the
1e9-point regime in a 1e6-point cloud: the same points per kernel length (uniform in a square
of side sqrt(1e6/1e9)) and the same lattice step relative to the point spacing (16 lattice bits
over the window instead of 21 over the unit square), so the per-point factorisations meet the
near-singular covariances and lattice collisions of the full configuration; the clamp counts
are reported with the errors.  Tolerances are those of the drop-in target: 1e-5 norm-relative
in float32 (test/python_parity_generate.jl:26-36 measures the same way).  The reverse sweep runs
in its pull form (set_reverse_mode(1); automatic only from 2e7 points up, where it is also the
faster form), whose sums follow the serial reference sweep's order: generate_grad_xi is then the
oracle's bit for bit at every configuration.
"""
import numpy as np
import pytest
import torch

import graphgp_b200 as gp
from conftest import report
from graphgp_b200 import configs as CF
from oracle import oracle as O

pytestmark = pytest.mark.gpu

TOL32 = 1e-5


def _problems(c, pts=None, n0=None, lattice_bits=21):
    """(device problem, oracle problem, graph) for configuration c."""
    pts = CF.points(c) if pts is None else pts
    g = gp.build_graph_arrays(pts, c.n0 if n0 is None else n0, c.k, lattice_bits=lattice_bits)
    bins, vals = CF.table(c)
    dt = c.dtype
    prob = gp.GraphGPProblem(g["coords"], g["neighbors"], g["offsets"], g["n0"], dt(g["scale"]),
                             bins, vals, g["indices"], dtype=dt)
    prob.set_reverse_mode(1)
    orc = O.make_problem(g["coords"], g["neighbors"], g["offsets"], g["n0"], dt(g["scale"]),
                         bins, vals, g["indices"], dt)
    return prob, orc, g


def _dev(x, device):
    return torch.from_numpy(np.ascontiguousarray(x)).to(device)


def _clamp_note(orc):
    s = O.clamp_stats(orc)
    return (f"clamped points {s['points_clamped']}, pivots {s['pivots_clamped']}, "
            f"collisions {s['collisions']}, zeroed weights {s['weights_zeroed']}")


def test_c2_full(cuda_device):
    c = CF.get("C2")
    prob, orc, _ = _problems(c)
    xi, vb = CF.xi(c), CF.vbar(c)
    f = gp.generate(prob, _dev(xi, cuda_device)).cpu().numpy()
    assert report("C2", "generate", c.n, f, O.generate(orc, xi)) < TOL32
    xg = gp.generate_grad_xi(prob, _dev(vb, cuda_device)).cpu().numpy()
    assert report("C2", "generate_grad_xi", c.n, xg, O.generate_grad_xi(orc, vb)) < TOL32
    dv = gp.generate_grad_vals(prob, _dev(xi, cuda_device), _dev(vb, cuda_device)).cpu().numpy()
    assert report("C2", "generate_grad_vals", c.n, dv, O.generate_grad_vals(orc, xi, vb)) < TOL32


def test_c3_full(cuda_device):
    c = CF.get("C3")
    prob, orc, _ = _problems(c)
    xi = CF.xi(c)
    f = gp.generate(prob, _dev(xi, cuda_device))
    fo = O.generate(orc, xi)
    assert report("C3", "generate", c.n, f.cpu().numpy(), fo) < TOL32
    back = gp.generate_inv(prob, _dev(fo, cuda_device)).cpu().numpy()
    assert report("C3", "generate_inv", c.n, back, O.generate_inv(orc, fo)) < TOL32
    ld, ldo = gp.generate_logdet(prob), O.generate_logdet(orc)
    assert report("C3", "generate_logdet", c.n, [ld], [ldo]) < TOL32
    dv = gp.refine_logdet_grad_vals(prob)
    dv = dv.cpu().numpy() if isinstance(dv, torch.Tensor) else dv
    assert report("C3", "refine_logdet_grad_vals", c.n, dv,
                  O.refine_logdet_grad_vals(orc)[1]) < TOL32


def test_c4_distribution(cuda_device):
    c = CF.get("C4", 2_000_000)
    prob, orc, _ = _problems(c)
    xi, vb = CF.xi(c), CF.vbar(c)
    note = _clamp_note(orc)
    f = gp.generate(prob, _dev(xi, cuda_device)).cpu().numpy()
    assert report("C4 (2e6)", "generate", c.n, f, O.generate(orc, xi), note) < TOL32
    xg = gp.generate_grad_xi(prob, _dev(vb, cuda_device)).cpu().numpy()
    assert report("C4 (2e6)", "generate_grad_xi", c.n, xg, O.generate_grad_xi(orc, vb)) < TOL32
    assert prob.dense_jitter() == orc._dense_cache[2]


def test_c5_distribution(cuda_device):
    c = CF.get("C5", 2_000_000)
    prob, orc, _ = _problems(c)
    xi, vb = CF.xi(c), CF.vbar(c)
    note = _clamp_note(orc)
    f = gp.generate(prob, _dev(xi, cuda_device)).cpu().numpy()
    assert report("C5 (2e6)", "generate", c.n, f, O.generate(orc, xi), note) < TOL32
    xg = gp.generate_grad_xi(prob, _dev(vb, cuda_device)).cpu().numpy()
    assert report("C5 (2e6)", "generate_grad_xi", c.n, xg, O.generate_grad_xi(orc, vb)) < TOL32
    dv = gp.generate_grad_vals(prob, _dev(xi, cuda_device), _dev(vb, cuda_device)).cpu().numpy()
    assert report("C5 (2e6)", "generate_grad_vals", c.n, dv,
                  O.generate_grad_vals(orc, xi, vb)) < TOL32
    assert prob.dense_jitter() == orc._dense_cache[2]


def test_c5_density_matched_window(cuda_device):
    n = 1_000_000
    c = CF.get("C5", n)
    side = (n / CF.CONFIGS["C5"].n) ** 0.5
    pts = side * np.random.default_rng(c.seed_points).random((n, 2))
    prob, orc, _ = _problems(c, pts=pts, n0=1000, lattice_bits=16)
    xi, vb = CF.xi(c), CF.vbar(c)
    note = _clamp_note(orc)
    tag = "C5 window"
    f = gp.generate(prob, _dev(xi, cuda_device)).cpu().numpy()
    assert report(tag, "generate", n, f, O.generate(orc, xi), note) < TOL32
    xg = gp.generate_grad_xi(prob, _dev(vb, cuda_device)).cpu().numpy()
    assert report(tag, "generate_grad_xi", n, xg, O.generate_grad_xi(orc, vb)) < TOL32
    dv = gp.generate_grad_vals(prob, _dev(xi, cuda_device), _dev(vb, cuda_device)).cpu().numpy()
    assert report(tag, "generate_grad_vals", n, dv, O.generate_grad_vals(orc, xi, vb)) < TOL32
