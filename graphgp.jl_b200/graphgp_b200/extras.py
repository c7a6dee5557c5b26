"""Covariance tables and the hyperparameter chain rule (src/extras.jl).

These run once per table on the host (nbins values) and produce the ``bins``/``vals`` inputs of
the refine path.  ``rbf_kernel`` and ``matern_kernel`` accept float or torch scalars; with torch
scalars the table is differentiable, which is what ``hyperparam_grad`` uses (the reference uses
a ForwardDiff Jacobian, src/extras.jl:86-92).
"""
from __future__ import annotations

import math

import numpy as np
import torch


def make_cov_bins(r_min: float, r_max: float, n_bins: int) -> np.ndarray:
    """``[0; 10 .^ range(log10(r_min), log10(r_max), n_bins - 1)]`` (src/extras.jl:14-17)."""
    inner = 10.0 ** np.linspace(math.log10(float(r_min)), math.log10(float(r_max)), n_bins - 1)
    return np.concatenate([[0.0], inner])


def _is_torch(*xs) -> bool:
    return any(isinstance(x, torch.Tensor) for x in xs)


def rbf_kernel(variance, scale, r_min, r_max, n_bins: int, jitter=0.0, dtype=np.float64):
    """RBF table: ``vals[i] = variance * exp(-1/2 * (bins[i]/scale)^2)``, ``vals[0] *= 1 +
    jitter`` (src/extras.jl:26-38).  Returns (bins float64, vals)."""
    bins = make_cov_bins(r_min, r_max, n_bins)
    if _is_torch(variance, scale):
        r = torch.as_tensor(bins, dtype=torch.float64)
        v = variance * torch.exp(-0.5 * (r / scale) ** 2)
        v = torch.cat([v[:1] * (1 + jitter), v[1:]])
        return bins, v
    r = bins.astype(dtype)
    v = (np.asarray(variance, dtype) * np.exp(np.asarray(-0.5, dtype) * (r / np.asarray(scale, dtype)) ** 2)).astype(dtype)
    v[0] = v[0] * (1 + np.asarray(jitter, dtype))
    return bins, v


def _matern_coeffs(p: int):
    return [math.exp(math.lgamma(p + 1.0) + math.lgamma(p + i + 1.0) - math.lgamma(i + 1.0)
                     - math.lgamma(p - i + 1.0) - math.lgamma(2 * p + 1.0)) for i in range(p + 1)]


def matern_kernel(p: int, variance, cutoff, r_min, r_max, n_bins: int, jitter=0.0,
                  dtype=np.float64):
    """Matern table with nu = p + 1/2 (src/extras.jl:57-73): ``variance * exp(-x) *
    polyval(c, 2x)`` with ``x = sqrt(2p+1) * r / cutoff`` and
    ``c_i = exp(lgamma(p+1) + lgamma(p+i+1) - lgamma(i+1) - lgamma(p-i+1) - lgamma(2p+1))``."""
    bins = make_cov_bins(r_min, r_max, n_bins)
    coeffs = _matern_coeffs(int(p))
    s = math.sqrt(float(2 * p + 1))
    if _is_torch(variance, cutoff):
        r = torch.as_tensor(bins, dtype=torch.float64)
        x = s * r / cutoff
        z = 2 * x
        acc = torch.full_like(z, coeffs[0])
        for c in coeffs[1:]:
            acc = acc * z + c
        v = variance * torch.exp(-x) * acc
        return bins, torch.cat([v[:1] * (1 + jitter), v[1:]])
    r = bins.astype(dtype)
    x = dtype(s) * r / np.asarray(cutoff, dtype)
    z = 2 * x
    acc = np.full_like(z, coeffs[0])
    for c in coeffs[1:]:
        acc = acc * z + dtype(c)
    v = (np.asarray(variance, dtype) * np.exp(-x) * acc).astype(dtype)
    v[0] = v[0] * (1 + np.asarray(jitter, dtype))
    return bins, v


def hyperparam_grad(grad_cov_vals, make_kernel, hyperparams):
    """``J' * grad_cov_vals`` with J = d(vals)/d(hyperparams) (src/extras.jl:86-92).

    ``make_kernel(*hyperparams) -> (bins, vals)`` must accept torch scalars (``rbf_kernel`` and
    ``matern_kernel`` do); the Jacobian is taken with torch autograd in float64."""
    hp = torch.as_tensor(np.asarray(hyperparams, dtype=np.float64))
    g = torch.as_tensor(np.asarray(
        grad_cov_vals.detach().cpu().numpy() if isinstance(grad_cov_vals, torch.Tensor)
        else grad_cov_vals, dtype=np.float64))

    def f(h):
        return torch.as_tensor(make_kernel(*h)[1], dtype=torch.float64)

    J = torch.autograd.functional.jacobian(f, hp)
    return (J.T @ g).numpy()


class AnisoCov:
    """Anisotropic covariance K(d_spatial, d_z) (src/types.jl:15-20): a 2-D table
    ``grid[i, j] = K(spatial_bins[i], z_bins[j])`` bilinear in the fractional bin indices;
    points carry the radial coordinate last (alpha * z), the first D - 1 spatial."""

    def __init__(self, spatial_bins, z_bins, grid, alpha):
        self.spatial_bins = spatial_bins
        self.z_bins = z_bins
        self.grid = grid
        self.alpha = float(alpha)


def build_anisotropic_covariance(spatial_bins, z_bins, grid, alpha, jitter=0.0, dtype=None):
    """``build_anisotropic_covariance`` (src/aniso.jl:20-39): grid (ns, nz), increasing axes
    starting at 0; ``grid[0, 0]`` inflated by ``1 + jitter`` (in the grid's type)."""
    g = np.array(grid, dtype=dtype if dtype is not None else np.asarray(grid).dtype, copy=True)
    if g.shape != (len(spatial_bins), len(z_bins)):
        raise ValueError("grid must be (len(spatial_bins), len(z_bins))")
    t = g.dtype.type
    g[0, 0] = g[0, 0] * (t(1) + t(jitter))
    return AnisoCov(np.asarray(spatial_bins, g.dtype), np.asarray(z_bins, g.dtype), g,
                    alpha)
