"""graphgp_b200 -- GraphGP.jl's refine path on B200, behind the reference's API.

The Vecchia per-point refine operations and their analytic adjoints run in libgraphgp_b200.so
(hand-written sm_100a kernels behind a C ABI, include/graphgp_b200.h); this package is the host
mirror of the GraphGP.jl interface over that library.
"""
from . import _lib
from ._lib import (GraphGPError, GraphInvariantError, NotPositiveDefiniteError,
                   UnsupportedError)
from .api import (check_graph, generate, generate_grad_vals, generate_grad_xi, generate_inv,
                  generate_inv_loss_grad_points, generate_inv_loss_grad_vals, generate_logdet,
                  generate_logdet_and_grad_vals, generate_logdet_grad_points,
                  generate_logdet_grad_vals, refine, refine_, refine_inv, refine_inv_,
                  refine_inv_loss_grad_points, refine_inv_loss_grad_vals, refine_logdet,
                  refine_logdet_grad_points, refine_logdet_grad_vals,
                  refine_logdet_grad_vals_noalloc, refine_logdet_terms, set_synchronous)
from .autodiff import generate_of_vals, generate_t, inv_quadratic_loss_of_vals, logdet_of_vals
from .extras import (AnisoCov, build_anisotropic_covariance, hyperparam_grad, make_cov_bins,
                     matern_kernel, rbf_kernel)
from .graph import build_graph, build_graph_arrays, build_graph_device, cached_graph
from .problem import GraphGPProblem, set_vals, to_backend

__all__ = [
    "GraphGPProblem", "to_backend", "set_vals", "build_graph", "build_graph_arrays",
    "build_graph_device",
    "cached_graph", "check_graph", "generate", "generate_inv", "generate_logdet",
    "generate_grad_xi", "generate_grad_vals", "refine", "refine_", "refine_inv", "refine_inv_",
    "refine_logdet", "refine_logdet_terms", "refine_logdet_grad_vals",
    "refine_logdet_grad_vals_noalloc",
    "generate_logdet_grad_vals", "generate_logdet_and_grad_vals", "refine_inv_loss_grad_vals",
    "generate_inv_loss_grad_vals", "logdet_of_vals", "inv_quadratic_loss_of_vals",
    "generate_of_vals", "generate_t", "make_cov_bins", "rbf_kernel", "matern_kernel",
    "hyperparam_grad", "GraphGPError", "GraphInvariantError", "UnsupportedError",
    "NotPositiveDefiniteError", "set_synchronous",
]


def library_path() -> str:
    return _lib.lib_path()
