"""The GraphGP.jl operations on the B200 path (names, argument meaning and order as in
src/GraphGP.jl:27-57).

Arrays in and out: a torch CUDA tensor in gives a torch tensor out (on the problem's device,
ordered on torch's current stream); a numpy array in gives a numpy array out (copied to the
device, computed, copied back).  Functions without an array argument return the kind the
problem was built from.  Every call goes through libgraphgp_b200.so; nothing is computed on the
host.

Orders follow the reference: ``generate``/``generate_inv``/``generate_grad_xi``/
``generate_grad_vals`` take and return ORIGINAL point order (the problem's ``indices``
permutation is applied on the device); the ``refine*`` family works in tree order.
"""
from __future__ import annotations

import ctypes as C

import numpy as np
import torch

from . import _lib
from .problem import GraphGPProblem

__all__ = [
    "refine", "refine_", "refine_inv", "refine_inv_", "refine_logdet", "refine_logdet_terms",
    "generate", "generate_inv", "generate_logdet", "generate_grad_xi", "generate_grad_vals",
    "refine_logdet_grad_vals", "generate_logdet_grad_vals", "generate_logdet_and_grad_vals",
    "refine_inv_loss_grad_vals", "generate_inv_loss_grad_vals", "check_graph",
]


def _stream(prob: GraphGPProblem) -> C.c_void_p:
    return C.c_void_p(torch.cuda.current_stream(prob.device).cuda_stream)


def _ptr(t: torch.Tensor) -> C.c_void_p:
    return C.c_void_p(t.data_ptr())


def _vec(prob: GraphGPProblem, x, n: int, name: str):
    """Device copy of a length-n vector in the problem's dtype; returns (tensor, was_host)."""
    if isinstance(x, torch.Tensor):
        t = x.detach().to(device=prob.device, dtype=prob.torch_dtype).contiguous()
        host = False
    else:
        a = np.ascontiguousarray(x, dtype=prob.dtype)
        t = torch.from_numpy(a).to(prob.device, non_blocking=False)
        host = True
    if t.ndim != 1 or t.shape[0] != n:
        raise ValueError(f"{name} must have length {n} (got shape {tuple(t.shape)})")
    return t, host


def _empty(prob: GraphGPProblem, n: int) -> torch.Tensor:
    return torch.empty(n, dtype=prob.torch_dtype, device=prob.device)


def _ret(t: torch.Tensor, host: bool):
    return t.cpu().numpy() if host else t


def _call(fn: str, *args) -> None:
    _lib.check(getattr(_lib.lib(), fn)(*args), fn)


# ---------------------------------------------------------------------------------------------
# Refine layer (tree order): src/api.jl
# ---------------------------------------------------------------------------------------------

def refine_(values, prob: GraphGPProblem, xi):
    """``refine!`` (src/api.jl:113-141): fills values[n0:] in place; values is a CUDA tensor."""
    if not isinstance(values, torch.Tensor) or not values.is_cuda or \
            values.dtype != prob.torch_dtype or not values.is_contiguous():
        raise TypeError("refine_ needs a contiguous CUDA tensor of the problem's dtype; "
                        "use refine() for host arrays")
    xr, _ = _vec(prob, xi, prob.nrefined(), "xi")
    _call("gpb2_refine", prob.handle, _ptr(values), _ptr(xr), _stream(prob))
    return values


def refine(prob: GraphGPProblem, initial_values, xi):
    """``refine(prob, initial_values, xi)`` (src/api.jl:176-182): values (N), tree order."""
    iv, host = _vec(prob, initial_values, prob.n0, "initial_values")
    values = torch.zeros(prob.npoints(), dtype=prob.torch_dtype, device=prob.device)
    values[: prob.n0] = iv
    refine_(values, prob, xi)
    return _ret(values, host)


def refine_inv_(xi_out, prob: GraphGPProblem, values):
    """``refine_inv!`` (src/api.jl:66-97)."""
    v, _ = _vec(prob, values, prob.npoints(), "values")
    _call("gpb2_refine_inv", prob.handle, _ptr(v), _ptr(xi_out), _stream(prob))
    return xi_out


def refine_inv(prob: GraphGPProblem, values):
    """``refine_inv(prob, values)`` (src/api.jl:99-103): xi of the refined points (M)."""
    v, host = _vec(prob, values, prob.npoints(), "values")
    xi = _empty(prob, prob.nrefined())
    _call("gpb2_refine_inv", prob.handle, _ptr(v), _ptr(xi), _stream(prob))
    return _ret(xi, host)


def refine_logdet_terms(prob: GraphGPProblem):
    """Per-point log(std) (src/api.jl:30-57)."""
    terms = _empty(prob, prob.nrefined())
    _call("gpb2_refine_logdet_terms", prob.handle, _ptr(terms), _stream(prob))
    return _ret(terms, prob.host_arrays)


def refine_logdet(prob: GraphGPProblem) -> float:
    """``refine_logdet`` (src/api.jl:24-28); the sum is accumulated in double."""
    out = C.c_double()
    _call("gpb2_refine_logdet", prob.handle, C.byref(out), _stream(prob))
    return out.value


# ---------------------------------------------------------------------------------------------
# Orchestration (original order): src/orchestrate.jl
# ---------------------------------------------------------------------------------------------

def generate(prob: GraphGPProblem, xi):
    """``generate(prob, xi)`` (src/orchestrate.jl:19-42)."""
    x, host = _vec(prob, xi, prob.npoints(), "xi")
    out = _empty(prob, prob.npoints())
    _call("gpb2_generate", prob.handle, _ptr(x), _ptr(out), _stream(prob))
    return _ret(out, host)


def generate_inv(prob: GraphGPProblem, values):
    """``generate_inv(prob, values)`` (src/orchestrate.jl:53-81)."""
    v, host = _vec(prob, values, prob.npoints(), "values")
    out = _empty(prob, prob.npoints())
    _call("gpb2_generate_inv", prob.handle, _ptr(v), _ptr(out), _stream(prob))
    return _ret(out, host)


def generate_logdet(prob: GraphGPProblem) -> float:
    """``generate_logdet(prob)`` (src/orchestrate.jl:89-97)."""
    out = C.c_double()
    _call("gpb2_generate_logdet", prob.handle, C.byref(out), _stream(prob))
    return out.value


# ---------------------------------------------------------------------------------------------
# Adjoints: src/grad.jl, src/grad_generate_vals.jl
# ---------------------------------------------------------------------------------------------

def generate_grad_xi(prob: GraphGPProblem, vbar):
    """VJP of ``generate`` w.r.t. xi (src/grad.jl:392-506); original order in and out."""
    vb, host = _vec(prob, vbar, prob.npoints(), "vbar")
    out = _empty(prob, prob.npoints())
    _call("gpb2_generate_grad_xi", prob.handle, _ptr(vb), _ptr(out), _stream(prob))
    return _ret(out, host)


def generate_grad_vals(prob: GraphGPProblem, xi, vbar):
    """VJP of ``generate`` w.r.t. the covariance values (src/grad_generate_vals.jl:111-282)."""
    x, host = _vec(prob, xi, prob.npoints(), "xi")
    vb, _ = _vec(prob, vbar, prob.npoints(), "vbar")
    out = _empty(prob, prob.nbins())
    _call("gpb2_generate_grad_vals", prob.handle, _ptr(x), _ptr(vb), _ptr(out), _stream(prob))
    return _ret(out, host)


def refine_logdet_grad_vals(prob: GraphGPProblem):
    """d(refine_logdet)/d(vals) (src/grad.jl:96-119)."""
    out = _empty(prob, prob.nbins())
    _call("gpb2_refine_logdet_grad_vals", prob.handle, _ptr(out), None, _stream(prob))
    return _ret(out, prob.host_arrays)


def refine_logdet_grad_vals_noalloc(prob: GraphGPProblem, out: torch.Tensor | None = None):
    """refine_logdet_grad_vals computed without any device allocation inside the library call
    (a fixed per-device accumulator; nbins <= 4096, overlapping calls on one device race).
    ``out``: optional caller-owned device tensor of nbins entries in the problem's dtype."""
    if out is None:
        out = _empty(prob, prob.nbins())
    elif (not isinstance(out, torch.Tensor) or out.device != prob.device
          or out.dtype != prob.torch_dtype or out.numel() != prob.nbins()
          or not out.is_contiguous()):
        raise ValueError("out must be a contiguous device tensor of nbins entries in the "
                         "problem's dtype on the problem's device")
    _call("gpb2_refine_logdet_grad_vals_noalloc", prob.handle, _ptr(out), None, _stream(prob))
    return _ret(out, prob.host_arrays)


def generate_logdet_grad_vals(prob: GraphGPProblem):
    """d(generate_logdet)/d(vals) (src/grad.jl:149-154)."""
    out = _empty(prob, prob.nbins())
    _call("gpb2_generate_logdet_grad_vals", prob.handle, _ptr(out), None, _stream(prob))
    return _ret(out, prob.host_arrays)


def generate_logdet_and_grad_vals(prob: GraphGPProblem):
    """(generate_logdet, its vals-gradient) in one pass (src/grad.jl:680-715)."""
    out = _empty(prob, prob.nbins())
    ld = C.c_double()
    _call("gpb2_generate_logdet_grad_vals", prob.handle, _ptr(out), C.byref(ld), _stream(prob))
    return ld.value, _ret(out, prob.host_arrays)


def refine_inv_loss_grad_vals(prob: GraphGPProblem, values):
    """(0.5*||refine_inv||^2, its vals-gradient) (src/grad.jl:643-678); values in tree order."""
    v, host = _vec(prob, values, prob.npoints(), "values")
    out = _empty(prob, prob.nbins())
    loss = C.c_double()
    _call("gpb2_refine_inv_loss_grad_vals", prob.handle, _ptr(v), _ptr(out), C.byref(loss),
          _stream(prob))
    return loss.value, _ret(out, host)


def generate_inv_loss_grad_vals(prob: GraphGPProblem, data):
    """(0.5*||generate_inv(data)||^2, its vals-gradient) (src/grad.jl:514-526); original order."""
    d, host = _vec(prob, data, prob.npoints(), "data")
    out = _empty(prob, prob.nbins())
    loss = C.c_double()
    _call("gpb2_generate_inv_loss_grad_vals", prob.handle, _ptr(d), _ptr(out), C.byref(loss),
          _stream(prob))
    return loss.value, _ret(out, host)


# ---------------------------------------------------------------------------------------------
# Point-position gradients: src/grad.jl:168-377 -- (N, D) in tree order (Julia's (D, N))
# ---------------------------------------------------------------------------------------------

def _points_out(prob: GraphGPProblem) -> torch.Tensor:
    return torch.empty((prob.npoints(), prob.ndims_space()), dtype=prob.torch_dtype,
                       device=prob.device)


def refine_logdet_grad_points(prob: GraphGPProblem):
    """``refine_logdet_grad_points(prob)`` (src/grad.jl:168-233)."""
    out = _points_out(prob)
    _call("gpb2_refine_logdet_grad_points", prob.handle, _ptr(out), _stream(prob))
    return _ret(out, prob.host_arrays)


def generate_logdet_grad_points(prob: GraphGPProblem):
    """``generate_logdet_grad_points(prob)`` (src/grad.jl:234-247): refinement + dense block."""
    out = _points_out(prob)
    _call("gpb2_generate_logdet_grad_points", prob.handle, _ptr(out), _stream(prob))
    return _ret(out, prob.host_arrays)


def refine_inv_loss_grad_points(prob: GraphGPProblem, values):
    """``refine_inv_loss_grad_points(prob, values)`` (src/grad.jl:259-358); values in tree
    order."""
    v, host = _vec(prob, values, prob.npoints(), "values")
    out = _points_out(prob)
    _call("gpb2_refine_inv_loss_grad_points", prob.handle, _ptr(v), _ptr(out), _stream(prob))
    return _ret(out, host)


def generate_inv_loss_grad_points(prob: GraphGPProblem, data):
    """``generate_inv_loss_grad_points(prob, data)`` (src/grad.jl:360-377); data in the
    original order."""
    d, host = _vec(prob, data, prob.npoints(), "data")
    out = _points_out(prob)
    _call("gpb2_generate_inv_loss_grad_points", prob.handle, _ptr(d), _ptr(out), _stream(prob))
    return _ret(out, host)


def set_synchronous(on: bool) -> None:
    """Process-wide call mode.  True (the default): every operation waits for its work and
    raises its numerical status (NotPositiveDefiniteError, barrier timeouts).  False: operations
    on device tensors return once their work is queued, as CUDA launches do; `prob.check()`
    waits and raises the status.  Operations that return host values still wait for them."""
    _lib.check(_lib.lib().gpb2_set_synchronous(1 if on else 0), "set_synchronous")


def check_graph(prob: GraphGPProblem) -> None:
    """Validate the graph invariants (src/graph_build.jl:20-57): offsets start at n0 and end at
    N, are non-decreasing, and every neighbour lies in an earlier depth batch.  The check runs
    on the device when the problem is uploaded; a violation raises GraphInvariantError (a
    ValueError, as the reference's ArgumentError)."""
    prob.handle  # noqa: B018  (upload validates)
