"""gpb2_refine_logdet_grad_vals_noalloc against gpb2_refine_logdet_grad_vals.

The no-allocation entry point accumulates in a fixed per-device array instead of the handle's
scratch.  Two calls in a row must each match the allocating entry point (the second call proves
the array is cleared between calls), and tables larger than the array must be refused.  This
file is collected last so it also runs after every other GPU test has used the device.
"""
import ctypes as C

import numpy as np
import pytest

import graphgp_b200 as gp
from graphgp_b200 import _lib
from conftest import relerr

pytestmark = pytest.mark.gpu

TOL = {np.float64: 1e-12, np.float32: 1e-5}


def _problem(dt, nbins=1000, seed=3):
    rng = np.random.default_rng(seed)
    pts = rng.standard_normal((20_000, 2))
    bins, vals = gp.rbf_kernel(1.0, 0.3, 1e-4, 10.0, nbins, jitter=1e-5)
    g = gp.build_graph_arrays(pts, 200, 8)
    return gp.GraphGPProblem(g["coords"], g["neighbors"], g["offsets"], g["n0"],
                             dt(g["scale"]), bins.astype(dt), vals.astype(dt), g["indices"],
                             dtype=dt)


@pytest.mark.parametrize("dt", [np.float64, np.float32])
def test_noalloc_matches_allocating_entry_point(cuda_device, dt):
    prob = _problem(dt)
    ref = gp.refine_logdet_grad_vals(prob)
    assert np.all(np.isfinite(ref)) and np.any(ref != 0)
    for _ in range(2):
        got = gp.refine_logdet_grad_vals_noalloc(prob)
        assert relerr(got, ref) < TOL[dt]


@pytest.mark.parametrize("dt", [np.float64, np.float32])
def test_noalloc_logdet_and_caller_buffer(cuda_device, dt):
    import torch
    prob = _problem(dt, seed=4)
    ref = gp.refine_logdet_grad_vals(prob)
    ld_ref = gp.refine_logdet(prob)
    out = torch.empty(prob.nbins(), dtype=prob.torch_dtype, device=prob.device)
    stream = C.c_void_p(torch.cuda.current_stream(prob.device).cuda_stream)
    for _ in range(2):
        ld = C.c_double(0.0)
        st = _lib.lib().gpb2_refine_logdet_grad_vals_noalloc(
            prob.handle, C.c_void_p(out.data_ptr()), C.byref(ld), stream)
        _lib.check(st, "noalloc")
        assert relerr(out.cpu().numpy(), ref) < TOL[dt]
        assert abs(ld.value - ld_ref) <= 1e-9 * abs(ld_ref)


def test_noalloc_rejects_oversize_table(cuda_device):
    prob = _problem(np.float32, nbins=5000, seed=5)
    with pytest.raises(gp.GraphGPError, match="4096"):
        gp.refine_logdet_grad_vals_noalloc(prob)
    # the allocating entry point still serves it
    assert np.all(np.isfinite(gp.refine_logdet_grad_vals(prob)))


def test_noalloc_fresh_handle_allocates_nothing(cuda_device):
    # A handle whose first operation is the no-allocation call (no scratch exists yet) gives the
    # allocating entry point's result, and the device's free memory is the same before and after
    # the call.  The library's module is loaded on the device by an earlier call first (module
    # loading reserves the fixed array itself, once per device).
    import torch
    gp.refine_logdet_grad_vals_noalloc(_problem(np.float32, seed=6))
    prob = _problem(np.float32, seed=7)
    ref = gp.refine_logdet_grad_vals(_problem(np.float32, seed=7))
    out = torch.empty(prob.nbins(), dtype=prob.torch_dtype, device=prob.device)
    h = prob.handle
    stream = C.c_void_p(torch.cuda.current_stream(prob.device).cuda_stream)
    torch.cuda.synchronize(cuda_device)
    free0 = torch.cuda.mem_get_info(cuda_device)[0]
    st = _lib.lib().gpb2_refine_logdet_grad_vals_noalloc(h, C.c_void_p(out.data_ptr()), None,
                                                         stream)
    torch.cuda.synchronize(cuda_device)
    free1 = torch.cuda.mem_get_info(cuda_device)[0]
    _lib.check(st, "noalloc")
    assert free1 == free0
    assert relerr(out.cpu().numpy(), ref) < TOL[np.float32]
