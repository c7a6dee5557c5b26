"""Seeded synthetic inputs of the five benchmark configurations (C1 ... C5).

Each configuration fixes the point distribution, the graph parameters (n0, k), the covariance
table and the input seeds; ``points``, ``table``, ``xi`` and ``vbar`` produce them.  The reference
names Julia ``MersenneTwister`` seeds, whose streams cannot be reproduced outside Julia: here
the same seed numbers feed numpy's ``Generator(PCG64(seed))`` on the host, or torch's Philox
generator when the points are produced on a GPU (``device="cuda"``, for the 1e8 / 1e9-point
configurations whose host generation would take minutes).  Both are deterministic.

Every generator accepts ``n`` to draw a smaller cloud of the same distribution (the parity
tests run the configurations' distributions at sizes the host checker finishes quickly).

C1  F64, N=1e4, D=2, N(0,1) (seed 99), n0=100,  k=10, RBF(1, 0.3, [1e-4, 10], 1000 bins)
C2  F32, N=1e6, D=2, N(0,1) (seed 1),  n0=1000, k=8,  RBF(1, 0.3, [1e-4, 10], 1000 bins)
C3  F32, N=1e7, D=3, U[0,1]^3 (seed 11), n0=2000, k=16, Matern p=1 (nu=1.5), scale 0.05,
    2000 bins over [1e-5, 2]
C4  F32, N=1e8, D=3, 90 % from 1000 Gaussian blobs (sigma 0.01, centres U[0,1]^3) + 10 %
    U[0,1]^3 (seed 21), n0=5000, k=8, RBF(1, 0.02, [1e-6, 2], 1000 bins)
C5  F32, N=1e9, D=2, U[0,1]^2 (seed 31), n0=1e4, k=8, RBF(1, 0.01, [1e-7, 1.5], 1000 bins)
All tables carry jitter 1e-5 on vals[0] (rbf_kernel / matern_kernel, src/extras.jl:26-73).
"""
from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np


@dataclass(frozen=True)
class Config:
    name: str
    n: int
    d: int
    n0: int
    k: int
    dtype: type
    dist: str                 # "normal" | "uniform" | "blobs"
    seed_points: int
    seed_xi: int
    seed_vbar: int | None
    kernel: str               # "rbf" | "matern1"
    variance: float
    scale: float
    r_min: float
    r_max: float
    n_bins: int
    jitter: float = 1e-5
    ops: tuple = field(default_factory=tuple)

    def scaled(self, n: int) -> "Config":
        """The same distribution and graph parameters with n points."""
        from dataclasses import replace
        return replace(self, n=int(n))


CONFIGS = {
    "C1": Config("C1", 10_000, 2, 100, 10, np.float64, "normal", 99, 7, None, "rbf",
                 1.0, 0.3, 1e-4, 10.0, 1000, ops=("generate", "generate_inv", "generate_logdet")),
    "C2": Config("C2", 1_000_000, 2, 1000, 8, np.float32, "normal", 1, 2, 3, "rbf",
                 1.0, 0.3, 1e-4, 10.0, 1000,
                 ops=("generate", "generate_grad_xi", "generate_grad_vals")),
    "C3": Config("C3", 10_000_000, 3, 2000, 16, np.float32, "uniform", 11, 12, None, "matern1",
                 1.0, 0.05, 1e-5, 2.0, 2000,
                 ops=("generate", "generate_inv", "generate_logdet", "refine_logdet_grad_vals")),
    "C4": Config("C4", 100_000_000, 3, 5000, 8, np.float32, "blobs", 21, 22, 23, "rbf",
                 1.0, 0.02, 1e-6, 2.0, 1000, ops=("generate", "generate_grad_xi")),
    "C5": Config("C5", 1_000_000_000, 2, 10_000, 8, np.float32, "uniform", 31, 32, 33, "rbf",
                 1.0, 0.01, 1e-7, 1.5, 1000,
                 ops=("generate", "generate_grad_xi", "generate_grad_vals")),
}

# Blob mixture of C4: 1000 isotropic Gaussian blobs, sigma 0.01, centres U[0,1]^3, 90 % of the
# points; the other 10 % uniform on the cube.
BLOBS = 1000
BLOB_SIGMA = 0.01
BLOB_FRACTION = 0.9


def get(name: str, n: int | None = None) -> Config:
    c = CONFIGS[name.upper()]
    return c if n is None else c.scaled(n)


def _points_numpy(c: Config) -> np.ndarray:
    rng = np.random.default_rng(c.seed_points)
    if c.dist == "normal":
        return rng.standard_normal((c.n, c.d))
    if c.dist == "uniform":
        return rng.random((c.n, c.d))
    if c.dist == "blobs":
        centres = rng.random((BLOBS, c.d))
        n_blob = int(round(BLOB_FRACTION * c.n))
        which = rng.integers(0, BLOBS, size=n_blob)
        pts = np.empty((c.n, c.d))
        pts[:n_blob] = centres[which] + BLOB_SIGMA * rng.standard_normal((n_blob, c.d))
        pts[n_blob:] = rng.random((c.n - n_blob, c.d))
        return pts
    raise ValueError(f"unknown distribution {c.dist!r}")


def _points_torch(c: Config, device):
    import torch
    g = torch.Generator(device=device)
    g.manual_seed(c.seed_points)
    f64 = torch.float64
    if c.dist == "normal":
        return torch.randn((c.n, c.d), generator=g, device=device, dtype=f64)
    if c.dist == "uniform":
        return torch.rand((c.n, c.d), generator=g, device=device, dtype=f64)
    if c.dist == "blobs":
        centres = torch.rand((BLOBS, c.d), generator=g, device=device, dtype=f64)
        n_blob = int(round(BLOB_FRACTION * c.n))
        which = torch.randint(0, BLOBS, (n_blob,), generator=g, device=device)
        pts = torch.empty((c.n, c.d), device=device, dtype=f64)
        pts[:n_blob] = centres[which]
        pts[:n_blob] += BLOB_SIGMA * torch.randn((n_blob, c.d), generator=g, device=device,
                                                 dtype=f64)
        pts[n_blob:] = torch.rand((c.n - n_blob, c.d), generator=g, device=device, dtype=f64)
        return pts
    raise ValueError(f"unknown distribution {c.dist!r}")


def points(c: Config, device=None):
    """(n, d) float64 points of the configuration: a numpy array (host generation, PCG64) when
    ``device`` is None, else a torch tensor generated on that device (Philox)."""
    if device is None:
        return _points_numpy(c)
    return _points_torch(c, device)


def table(c: Config):
    """(bins float64, vals in the configuration's dtype): the covariance table."""
    from .extras import matern_kernel, rbf_kernel
    if c.kernel == "rbf":
        bins, vals = rbf_kernel(c.variance, c.scale, c.r_min, c.r_max, c.n_bins,
                                jitter=c.jitter)
    elif c.kernel == "matern1":
        bins, vals = matern_kernel(1, c.variance, c.scale, c.r_min, c.r_max, c.n_bins,
                                   jitter=c.jitter)
    else:
        raise ValueError(f"unknown kernel {c.kernel!r}")
    return bins.astype(c.dtype), np.asarray(vals).astype(c.dtype)


def _normal(seed: int, n: int, dtype, device=None):
    if device is None:
        return np.random.default_rng(seed).standard_normal(n).astype(dtype)
    import torch
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    tdt = torch.float32 if np.dtype(dtype) == np.float32 else torch.float64
    return torch.randn(n, generator=g, device=device, dtype=tdt)


def xi(c: Config, device=None):
    """Latent white noise xi ~ N(0, 1), n entries in the configuration's dtype."""
    return _normal(c.seed_xi, c.n, c.dtype, device)


def vbar(c: Config, device=None):
    """Upstream cotangent on the generated values ~ N(0, 1) (C2: seed 3; the other
    configurations name none, and use seed_xi + 1)."""
    seed = c.seed_vbar if c.seed_vbar is not None else c.seed_xi + 1
    return _normal(seed, c.n, c.dtype, device)


def describe(c: Config) -> str:
    tab = (f"RBF(var {c.variance:g}, scale {c.scale:g}, [{c.r_min:g}, {c.r_max:g}], "
           f"{c.n_bins} bins, jitter {c.jitter:g})" if c.kernel == "rbf" else
           f"Matern p=1 (var {c.variance:g}, scale {c.scale:g}, [{c.r_min:g}, {c.r_max:g}], "
           f"{c.n_bins} bins, jitter {c.jitter:g})")
    return (f"{c.name}: N={c.n:.0e} D={c.d} {c.dist}(seed {c.seed_points}) n0={c.n0} k={c.k} "
            f"{tab} {np.dtype(c.dtype).name}")
