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
