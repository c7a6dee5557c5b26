"""Test configuration: the `gpu` marker, import paths, shared fixtures.

CPU tests (`-m "not gpu"`) pin the oracle to the reference's golden vectors, check the graph
builder byte for byte, and check that libgraphgp_b200.so loads and exports every declared entry
point.  GPU tests (`-m gpu`) are the parity tests proper: the CUDA path, called through the C
ABI, against the oracle on the same inputs.
"""
import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "graphgp.jl_b200")
GOLDEN = os.path.join(ROOT, "tests", "golden")
for p in (ROOT, PKG):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


def relerr(a, b) -> float:
    """Norm-relative error ||a - b|| / ||b|| (test/python_parity_generate.jl:26)."""
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-300))


def load_golden(name: str):
    with np.load(os.path.join(GOLDEN, f"{name}.npz")) as d:
        return {k: d[k] for k in d.files}


@pytest.fixture(scope="session")
def golden():
    return load_golden


@pytest.fixture(scope="session")
def cuda_device():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return torch.device("cuda", 0)


# Parity figures recorded by the tests (config, operation, size, norm-relative error, max-abs
# error, note) and printed at the end of the run, so that a run's log carries the measured
# errors next to the pass/fail status.
PARITY = []


def report(config: str, op: str, n: int, a, b, note: str = "") -> float:
    """Record the error of `a` against the reference values `b` and return the norm-relative
    error."""
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    rel = relerr(a, b)
    mx = float(np.max(np.abs(a - b))) if a.size else 0.0
    PARITY.append((config, op, int(n), rel, mx, note))
    return rel


def pytest_terminal_summary(terminalreporter, exitstatus, config):
    if not PARITY:
        return
    tr = terminalreporter
    tr.write_sep("-", "parity against the oracle (norm-relative error, max-abs error)")
    for cfg, op, n, rel, mx, note in PARITY:
        tr.write_line(f"{cfg:<14} {op:<26} n={n:<11} rel={rel:.2e} maxabs={mx:.2e} {note}")
