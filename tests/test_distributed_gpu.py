"""Level-sharded generate / generate_grad_xi on 2 GPUs over NCCL (skipped with fewer GPUs):
the sharded forward must equal the single-GPU generate bit for bit, the reverse must match
the single-GPU generate_grad_xi within tolerance."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, dt_name, q):
    import datetime
    import torch.distributed as dist
    from _dist_common import gp
    from graphgp_b200.distributed import ShardedGenerate
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev,
                            timeout=datetime.timedelta(seconds=120))
    try:
        dt = np.dtype(dt_name).type
        rng = np.random.default_rng(3)
        pts = rng.standard_normal((200_000, 2))
        bins, vals = gp.rbf_kernel(1.0, 0.3, 1e-4, 10.0, 1000, jitter=1e-5)
        g = gp.build_graph_arrays(pts, 500, 8)
        prob = gp.GraphGPProblem(g["coords"], g["neighbors"], g["offsets"], g["n0"],
                                 dt(g["scale"]), bins.astype(dt), vals.astype(dt), g["indices"],
                                 dtype=dt, device=dev)
        sg = ShardedGenerate(prob, min_shard=1024)
        xi = torch.from_numpy(rng.standard_normal(prob.npoints()).astype(dt)).to(dev)
        vb = torch.from_numpy(rng.standard_normal(prob.npoints()).astype(dt)).to(dev)
        f = sg.generate(xi)
        xg = sg.generate_grad_xi(vb)
        f1 = gp.generate(prob, xi)
        xg1 = gp.generate_grad_xi(prob, vb)
        torch.cuda.synchronize(dev)
        same = bool(torch.equal(f, f1))
        err = float((xg - xg1).norm() / xg1.norm())
        q.put((rank, same, err, sum(b.sharded for b in sg.batches)))
        dist.barrier()
        prob.release()
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("dt_name", ["float32", "float64"])
def test_level_sharded_two_gpus(dt_name):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, dt_name, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=600) for _ in range(world)]
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    tol = 1e-12 if dt_name == "float64" else 1e-5
    for rank, same, err, sharded in res:
        assert sharded > 0
        assert same, f"rank {rank}: sharded generate differs from the single-GPU path"
        assert err < tol, f"rank {rank}: grad_xi relerr {err}"


def _lib_worker(rank, world, port, dt_name, q):
    """The library's level-sharded operations (NCCL inside libgraphgp_b200.so) against the
    single-GPU operations on the same problem."""
    import datetime
    import torch.distributed as dist
    from _dist_common import gp
    from graphgp_b200 import configs as CF
    from graphgp_b200.distributed import Comm, LevelSharded, distribute
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=120))
    comm = None
    try:
        dt = np.dtype(dt_name).type
        c = CF.get("C4", 300_000)
        g = gp.build_graph_device(CF.points(c), c.n0, c.k, device=dev)
        bins, vals = CF.table(c)
        prob = gp.GraphGPProblem(g["coords"], g["neighbors"], g["offsets"], g["n0"],
                                 dt(g["scale"]), bins.astype(dt), vals.astype(dt), g["indices"],
                                 dtype=dt, device=dev)
        comm = Comm(device=dev, min_shard=4096, timeout_s=120)
        ls = LevelSharded(prob, comm)
        rng = np.random.default_rng(5)
        xi = torch.from_numpy(rng.standard_normal(prob.npoints()).astype(dt)).to(dev)
        vb = torch.from_numpy(rng.standard_normal(prob.npoints()).astype(dt)).to(dev)
        f, xg, dv = ls.generate(xi), ls.generate_grad_xi(vb), ls.generate_grad_vals(xi, vb)
        d = distribute(prob, comm)
        ld, dl = d.generate_logdet_and_grad_vals()
        loss, dil = d.generate_inv_loss_grad_vals(f)
        f1, xg1, dv1 = gp.generate(prob, xi), gp.generate_grad_xi(prob, vb), \
            gp.generate_grad_vals(prob, xi, vb)
        ld1, dl1 = gp.generate_logdet_and_grad_vals(prob)
        loss1, dil1 = gp.generate_inv_loss_grad_vals(prob, f1)
        torch.cuda.synchronize(dev)

        def rel(a, b):
            return float((a.double() - b.double()).norm() / b.double().norm())
        q.put((rank, bool(torch.equal(f, f1)), rel(xg, xg1), rel(dv, dv1), abs(ld - ld1) / abs(ld1),
               rel(dl, dl1), abs(loss - loss1) / abs(loss1), rel(dil, dil1)))
        dist.barrier()
        prob.release()
    finally:
        if comm is not None:
            comm.close()
        dist.destroy_process_group()


@pytest.mark.parametrize("dt_name", ["float32", "float64"])
def test_library_level_sharded_two_gpus(dt_name):
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_lib_worker, args=(r, world, port, dt_name, q))
             for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=600) for _ in range(world)]
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    tol = 1e-12 if dt_name == "float64" else 1e-5
    for rank, same, *errs in res:
        assert same, f"rank {rank}: sharded generate differs from the single-GPU path"
        assert all(e < tol for e in errs), f"rank {rank}: {errs}"


def test_library_sharded_one_rank(cuda_device):
    # One rank: the same calls through the library communicator (the collectives run over a
    # single rank) give the single-GPU results.
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    p = ctx.Process(target=_lib_worker, args=(0, 1, _free_port(), "float32", q))
    p.start()
    rank, same, *errs = q.get(timeout=600)
    p.join(timeout=120)
    assert p.exitcode == 0
    assert same and all(e < 1e-5 for e in errs), errs
