"""ctypes binding of libgraphgp_b200.so (the C ABI declared in include/graphgp_b200.h).

The library is loaded from ``$GRAPHGP_B200_LIB`` when set, else from the package tree
(``graphgp.jl_b200/libgraphgp_b200.so``), mirroring the ``GRAPHGP_CUDA_LIB`` lookup of the
reference's CUDA extension (ext/GraphGPCUDAExt.jl:15-24).  A missing library is an error: there
is no CPU fallback for the refine path.
"""
from __future__ import annotations

import ctypes as C
import os
import threading

_PKG_ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
DEFAULT_LIB = os.path.join(_PKG_ROOT, "libgraphgp_b200.so")

GPB2_OK = 0
GPB2_ERR_INVALID_ARG = 1
GPB2_ERR_UNSUPPORTED_K = 2
GPB2_ERR_UNSUPPORTED_D = 3
GPB2_ERR_OOM = 4
GPB2_ERR_CUDA = 5
GPB2_ERR_NCCL = 6
GPB2_ERR_TIMEOUT = 7
GPB2_ERR_GRAPH = 8
GPB2_ERR_NOT_PD = 9
GPB2_ERR_UNSUPPORTED_TABLE = 10
GPB2_ERR_NO_DEVICE = 11

GPB2_F32 = 0
GPB2_F64 = 1


class GraphGPError(RuntimeError):
    """A non-zero status from libgraphgp_b200.so (the reference turns rc != 0 into `error()`,
    ext/GraphGPCUDAExt.jl:47,61)."""

    def __init__(self, status: int, message: str):
        super().__init__(f"[gpb2 status {status}] {message}")
        self.status = status


class GraphInvariantError(GraphGPError, ValueError):
    """check_graph invariant violated (src/graph_build.jl:20-57 raises ArgumentError)."""


class UnsupportedError(GraphGPError, NotImplementedError):
    """No compiled kernel set for this (K, D) or an unsupported covariance table."""


class NotPositiveDefiniteError(GraphGPError):
    """Dense block not PD even with 1e-2 jitter (src/dense.jl:65-66)."""


_STATUS_CLASS = {
    GPB2_ERR_INVALID_ARG: lambda s, m: _ValueGraphGPError(s, m),
    GPB2_ERR_GRAPH: GraphInvariantError,
    GPB2_ERR_UNSUPPORTED_K: UnsupportedError,
    GPB2_ERR_UNSUPPORTED_D: UnsupportedError,
    GPB2_ERR_UNSUPPORTED_TABLE: UnsupportedError,
    GPB2_ERR_NOT_PD: NotPositiveDefiniteError,
}


class _ValueGraphGPError(GraphGPError, ValueError):
    pass


P = C.c_void_p
I64 = C.c_int64
I32 = C.c_int
PI64 = C.POINTER(C.c_int64)
PD = C.POINTER(C.c_double)

# name -> (restype, argtypes)
_SIGNATURES = {
    "gpb2_version": (I32, []),
    "gpb2_last_error": (C.c_char_p, []),
    "gpb2_problem_create": (I32, [C.POINTER(P), I32, I32, P, I64, I64, P, I32, I32, I64, PI64,
                                  I64, I64, C.c_double, P, P, I64, PI64, I32, P]),
    "gpb2_problem_create_dev": (I32, [C.POINTER(P), I32, I32, P, I64, I64, P, I32, I32, I64,
                                      PI64, I64, I64, C.c_double, P, P, I64, P, I32, I32, P]),
    "gpb2_problem_order": (I32, [P, P, P, P]),
    "gpb2_problem_set_vals": (I32, [P, P, P]),
    "gpb2_problem_prefactor": (I32, [P, P]),
    "gpb2_problem_info": (I32, [P, PI64, PI64, PI64, PI64, PI64]),
    "gpb2_problem_set_factor_cache": (I32, [P, I32]),
    "gpb2_problem_set_aniso": (I32, [P, P, I64, P, I64, P, C.c_double, P]),
    "gpb2_problem_set_reverse_mode": (I32, [P, I32]),
    "gpb2_problem_reverse_mode": (I32, [P, C.POINTER(I32), C.POINTER(I32), PI64]),
    "gpb2_problem_factor_cache": (I32, [P, C.POINTER(I32), C.POINTER(I32), PI64]),
    "gpb2_problem_destroy": (I32, [P]),
    "gpb2_problem_dense_jitter": (I32, [P, PD]),
    "gpb2_problem_dense_factor": (I32, [P, P, P]),
    "gpb2_profile_enable": (I32, [I32]),
    "gpb2_profile_reset": (I32, []),
    "gpb2_profile_report": (I32, [C.c_char_p, I64]),
    "gpb2_launch_count": (I64, []),
    "gpb2_set_forward_mode": (I32, [I32]),
    "gpb2_set_overlap": (I32, [I32]),
    "gpb2_set_synchronous": (I32, [I32]),
    "gpb2_problem_check": (I32, [P, P]),
    "gpb2_refine": (I32, [P, P, P, P]),
    "gpb2_refine_inv": (I32, [P, P, P, P]),
    "gpb2_refine_range": (I32, [P, P, P, I64, I64, P]),
    "gpb2_refine_reverse_range": (I32, [P, P, P, I64, I64, P]),
    "gpb2_dense_apply": (I32, [P, I32, P, P, P]),
    "gpb2_refine_logdet_terms": (I32, [P, P, P]),
    "gpb2_refine_logdet": (I32, [P, PD, P]),
    "gpb2_refine_logdet_grad_vals": (I32, [P, P, PD, P]),
    "gpb2_refine_logdet_grad_vals_noalloc": (I32, [P, P, PD, P]),
    "gpb2_refine_inv_loss_grad_vals": (I32, [P, P, P, PD, P]),
    "gpb2_generate": (I32, [P, P, P, P]),
    "gpb2_generate_inv": (I32, [P, P, P, P]),
    "gpb2_generate_logdet": (I32, [P, PD, P]),
    "gpb2_generate_grad_xi": (I32, [P, P, P, P]),
    "gpb2_generate_grad_vals": (I32, [P, P, P, P, P]),
    "gpb2_generate_logdet_grad_vals": (I32, [P, P, PD, P]),
    "gpb2_generate_inv_loss_grad_vals": (I32, [P, P, P, PD, P]),
    "gpb2_refine_logdet_grad_points": (I32, [P, P, P]),
    "gpb2_generate_logdet_grad_points": (I32, [P, P, P]),
    "gpb2_refine_inv_loss_grad_points": (I32, [P, P, P, P]),
    "gpb2_generate_inv_loss_grad_points": (I32, [P, P, P, P]),
    "gpb2_build_graph": (I32, [P, I64, I64, I64, I64, I64, I64, I64, C.POINTER(P)]),
    "gpb2_graph_n_offsets": (I64, [P]),
    "gpb2_graph_n0": (I64, [P]),
    "gpb2_graph_export": (I32, [P, P, P, P, P, PD]),
    "gpb2_graph_free": (None, [P]),
    "gpb2_comm_unique_id": (I32, [P]),
    "gpb2_comm_create": (I32, [C.POINTER(P), I32, I32, P, I32, C.c_double]),
    "gpb2_comm_set_min_shard": (I32, [P, I64]),
    "gpb2_comm_info": (I32, [P, C.POINTER(I32), C.POINTER(I32)]),
    "gpb2_comm_destroy": (I32, [P]),
    "gpb2_generate_sharded": (I32, [P, P, P, P, P]),
    "gpb2_generate_grad_xi_sharded": (I32, [P, P, P, P, P]),
    "gpb2_generate_grad_vals_sharded": (I32, [P, P, P, P, P, P]),
    "gpb2_generate_logdet_sharded": (I32, [P, P, PD, P]),
    "gpb2_generate_logdet_grad_vals_sharded": (I32, [P, P, P, PD, P]),
    "gpb2_generate_inv_loss_grad_vals_sharded": (I32, [P, P, P, P, PD, P]),
    "gpb2_shard_plan": (I32, [PI64, I64, I32, I32, I64, PI64, PI64, PI64, PI64,
                              C.POINTER(I32), PI64]),
    "gpb2_build_graph_device": (I32, [P, I64, I64, I64, I64, I64, I64, I32, P, C.POINTER(P)]),
    "gpb2_dgraph_n_offsets": (I64, [P]),
    "gpb2_dgraph_n0": (I64, [P]),
    "gpb2_dgraph_export": (I32, [P, P, P, P, PI64, PD, P]),
    "gpb2_dgraph_free": (None, [P]),
}

_lib = None
_lock = threading.Lock()


def lib_path() -> str:
    return os.environ.get("GRAPHGP_B200_LIB", DEFAULT_LIB)


def lib():
    """The loaded library; raises if it is missing (build it with `make -C graphgp.jl_b200`)."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            path = lib_path()
            if not os.path.isfile(path):
                raise ImportError(
                    f"libgraphgp_b200.so not found at {path}: build it with "
                    "`make -C graphgp.jl_b200 -j` (or set GRAPHGP_B200_LIB)")
            L = C.CDLL(path)
            for name, (res, args) in _SIGNATURES.items():
                f = getattr(L, name)
                f.restype = res
                f.argtypes = args
            _lib = L
    return _lib


def last_error() -> str:
    msg = lib().gpb2_last_error()
    return msg.decode() if msg else ""


def check(status: int, what: str = "") -> None:
    if status == GPB2_OK:
        return
    msg = last_error()
    cls = _STATUS_CLASS.get(status, GraphGPError)
    raise cls(status, f"{what}: {msg}" if what else msg)


def profile_report() -> dict:
    """{kernel kind: (launches, total_ms)} of the launches recorded since the last reset."""
    buf = C.create_string_buffer(1 << 16)
    check(lib().gpb2_profile_report(buf, len(buf)), "gpb2_profile_report")
    out = {}
    for line in buf.value.decode().splitlines():
        name, cnt, ms = line.split()
        out[name] = (int(cnt), float(ms))
    return out


def exported_symbols():
    """Names of every entry point this binding expects (the declarations of graphgp_b200.h)."""
    return list(_SIGNATURES)
