"""The C ABI from C: a program that includes only include/graphgp_b200.h, linked against
libgraphgp_b200.so, run on the host entry points (CPU suite) and on a problem end to end
(GPU suite, compared with the reference's generate_parity fixture)."""
import os
import subprocess

import numpy as np
import pytest

from conftest import ROOT, relerr
from oracle import oracle as O

SRC = os.path.join(ROOT, "tests", "c", "abi_generate.c")
LIBDIR = os.path.join(ROOT, "graphgp.jl_b200")
CUDA = "/usr/local/cuda"


def _build(tmp_path, with_cuda):
    exe = str(tmp_path / ("abi_gpu" if with_cuda else "abi_host"))
    cmd = ["gcc", "-std=c11", "-O1", "-Wall", "-Wextra", "-Werror", "-I",
           os.path.join(ROOT, "include"), SRC, "-o", exe, "-L", LIBDIR, "-lgraphgp_b200",
           f"-Wl,-rpath,{LIBDIR}"]
    if with_cuda:
        cmd[2:2] = ["-DWITH_CUDA", "-I", os.path.join(CUDA, "include")]
        cmd += ["-L", os.path.join(CUDA, "lib64"), "-lcudart", f"-Wl,-rpath,{CUDA}/lib64"]
    subprocess.run(cmd, check=True)
    return exe


def test_c_program_host_entry_points(tmp_path):
    exe = _build(tmp_path, with_cuda=False)
    r = subprocess.run([exe, "host"], capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    assert "host ok" in r.stdout


@pytest.mark.gpu
def test_c_program_generate(tmp_path, golden, cuda_device):
    d = golden("generate_parity")
    n, dd = d["coords"].shape
    k = d["neighbors"].shape[1]
    (tmp_path / "meta.txt").write_text(
        f"{n} {dd} {k} {int(d['n0'])} {len(d['offsets'])} {len(d['cov_bins64'])} "
        f"{float(d['scale'])!r}\n")
    np.ascontiguousarray(d["coords"], np.uint32).tofile(tmp_path / "coords.u32")
    np.ascontiguousarray(d["neighbors"], np.int64).tofile(tmp_path / "nbrs.i64")
    np.ascontiguousarray(d["offsets"], np.int64).tofile(tmp_path / "offsets.i64")
    np.ascontiguousarray(d["indices"], np.int64).tofile(tmp_path / "indices.i64")
    np.ascontiguousarray(d["cov_bins64"], np.float64).tofile(tmp_path / "bins.f64")
    np.ascontiguousarray(d["cov_vals64"], np.float64).tofile(tmp_path / "vals.f64")
    np.ascontiguousarray(d["xi"], np.float64).tofile(tmp_path / "xi.f64")
    exe = _build(tmp_path, with_cuda=True)
    r = subprocess.run([exe, "gpu", str(tmp_path)], capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    out = np.fromfile(tmp_path / "out.f64", np.float64)
    assert relerr(out[:n], d["generate_field"]) < 1e-12
    orc = O.make_problem(d["coords"], d["neighbors"], d["offsets"], d["n0"], d["scale"],
                         d["cov_bins64"], d["cov_vals64"], d["indices"], np.float64)
    ld = O.generate_logdet(orc)
    assert abs(out[n] - ld) < 1e-12 * abs(ld)
