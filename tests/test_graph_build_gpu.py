"""The device graph builder (gpb2_build_graph_device) against the host restatement and the
reference's fixture: the same coordinates, neighbours, permutation, offsets and scale, byte for
byte, on the configurations' distributions and on sizes that exercise the tree's edge cases
(N just above and below powers of two, tiny N, duplicate points, points on a lattice)."""
import numpy as np
import pytest
import torch

import graphgp_b200 as gp
from graphgp_b200 import configs as CF

pytestmark = pytest.mark.gpu


def _host(g):
    return dict(coords=g["coords"].cpu().numpy().view(np.uint32),
                neighbors=g["neighbors"].cpu().numpy().astype(np.int64),
                indices=g["indices"].cpu().numpy().astype(np.int64),
                offsets=g["offsets"], n0=g["n0"], scale=g["scale"])


def _same(a, b):
    for key in ("coords", "neighbors", "indices", "offsets"):
        assert np.array_equal(np.asarray(a[key]), np.asarray(b[key])), key
    assert a["n0"] == b["n0"]
    assert a["scale"] == b["scale"]


def test_device_build_golden(cuda_device, golden):
    d = golden("generate_parity")
    idx = d["indices"]
    inv = np.empty_like(idx)
    inv[idx] = np.arange(len(idx))
    pts = d["coords"][inv].astype(np.float64)
    g = _host(gp.build_graph_device(pts, int(d["n0"]), d["neighbors"].shape[1]))
    assert np.array_equal(g["indices"], d["indices"])
    assert np.array_equal(g["neighbors"], d["neighbors"])
    assert np.array_equal(g["offsets"], d["offsets"])
    assert np.array_equal(g["coords"], d["coords"])


@pytest.mark.parametrize("N,D,n0,k,dist", [
    (2, 1, 1, 1, "normal"), (3, 2, 1, 2, "normal"), (7, 2, 2, 3, "uniform"),
    (1023, 2, 10, 4, "normal"), (1024, 3, 10, 8, "uniform"), (1025, 3, 17, 8, "normal"),
    (65537, 2, 300, 10, "normal"), (100_000, 4, 64, 6, "normal"), (131071, 3, 1000, 16, "uniform"),
    (50_000, 2, 100, 32, "uniform"), (20000, 5, 200, 8, "normal")])
def test_device_build_matches_host(cuda_device, N, D, n0, k, dist):
    rng = np.random.default_rng(N * 7 + D)
    pts = rng.standard_normal((N, D)) if dist == "normal" else rng.random((N, D))
    _same(_host(gp.build_graph_device(pts, n0, k)), gp.build_graph_arrays(pts, n0, k))


def test_device_build_duplicates_and_lattice(cuda_device):
    # Repeated points (equal keys: ties broken by position) and integer-valued points (equal
    # distances: ties broken by index, and lattice collisions after quantisation).
    rng = np.random.default_rng(9)
    base = rng.integers(0, 50, size=(3000, 2)).astype(np.float64)
    pts = np.concatenate([base, base[:1000], -base[:500]])
    _same(_host(gp.build_graph_device(pts, 64, 8)), gp.build_graph_arrays(pts, 64, 8))
    _same(_host(gp.build_graph_device(pts, 64, 8, lattice_bits=8)),
          gp.build_graph_arrays(pts, 64, 8, lattice_bits=8))


@pytest.mark.parametrize("name,n", [("C2", 1_000_000), ("C3", 1_000_000), ("C4", 2_000_000),
                                    ("C5", 2_000_000)])
def test_device_build_configs(cuda_device, name, n):
    c = CF.get(name, n)
    pts = CF.points(c)
    _same(_host(gp.build_graph_device(pts, c.n0, c.k)), gp.build_graph_arrays(pts, c.n0, c.k))


def test_device_graph_problem(cuda_device):
    # A problem built from the device arrays (permutation checked on the device) gives the same
    # field as one built from the host arrays.
    c = CF.get("C2", 200_000)
    pts = CF.points(c)
    gd = gp.build_graph_device(pts, c.n0, c.k)
    gh = gp.build_graph_arrays(pts, c.n0, c.k)
    bins, vals = CF.table(c)
    pd = gp.GraphGPProblem(gd["coords"], gd["neighbors"], gd["offsets"], gd["n0"],
                           np.float32(gd["scale"]), bins, vals, gd["indices"], dtype=np.float32)
    ph = gp.GraphGPProblem(gh["coords"], gh["neighbors"], gh["offsets"], gh["n0"],
                           np.float32(gh["scale"]), bins, vals, gh["indices"], dtype=np.float32)
    xi = torch.from_numpy(CF.xi(c)).to(cuda_device)
    assert torch.equal(gp.generate(pd, xi), gp.generate(ph, xi))
    bad = gd["indices"].clone()
    bad[0] = bad[1]
    with pytest.raises(ValueError):
        gp.GraphGPProblem(gd["coords"], gd["neighbors"], gd["offsets"], gd["n0"],
                          np.float32(gd["scale"]), bins, vals, bad, dtype=np.float32).handle
