"""The C ABI: libgraphgp_b200.so loads (no GPU needed to load it) and exports every entry point
include/graphgp_b200.h declares, with the Python binding's signature table in step."""
import ctypes as C
import os
import re

import pytest

import graphgp_b200 as gp
from graphgp_b200 import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "graphgp_b200.h")


def declared_symbols():
    src = open(HEADER).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(gpb2_\w+)\s*\(", src)))


def test_header_declares_the_path():
    names = declared_symbols()
    for must in ("gpb2_generate", "gpb2_generate_inv", "gpb2_generate_logdet",
                 "gpb2_generate_grad_xi", "gpb2_generate_grad_vals",
                 "gpb2_refine_logdet_grad_vals", "gpb2_refine", "gpb2_refine_inv",
                 "gpb2_problem_create", "gpb2_build_graph"):
        assert must in names


def test_library_loads_and_exports_every_symbol():
    L = C.CDLL(_lib.lib_path())
    missing = [n for n in declared_symbols() if not hasattr(L, n)]
    assert not missing, missing


def test_binding_table_matches_header():
    assert sorted(_lib.exported_symbols()) == declared_symbols()


def test_version_and_error_plumbing():
    L = _lib.lib()
    assert L.gpb2_version() == 1
    # A host-only call with bad arguments sets the thread's error message and returns a status.
    g = C.c_void_p()
    st = L.gpb2_build_graph(None, 10, 2, 1, 2, 4, 21, 1, C.byref(g))
    assert st == _lib.GPB2_ERR_INVALID_ARG
    assert "gpb2_build_graph" in _lib.last_error()
    with pytest.raises(ValueError):
        _lib.check(st, "probe")


def test_forward_mode_setter_validates():
    L = _lib.lib()
    assert L.gpb2_set_forward_mode(7) == _lib.GPB2_ERR_INVALID_ARG
    assert L.gpb2_set_forward_mode(0) == _lib.GPB2_OK


def test_no_oracle_in_product_path():
    # The product package must not reach into the oracle (test infrastructure only).
    pkg = os.path.dirname(gp.__file__)
    for fn in os.listdir(pkg):
        if fn.endswith(".py"):
            txt = open(os.path.join(pkg, fn)).read()
            assert "oracle" not in txt.replace("oracle (test", ""), fn
