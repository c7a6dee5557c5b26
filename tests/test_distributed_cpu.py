"""Level-sharded generate / generate_grad_xi: the orchestration (batch split, in-place
gathers, cotangent reductions, slack) run as 2 and 3 gloo ranks on CPU, with the per-batch work
done by a numpy restatement of the oracle's arithmetic.  The sharded forward must reproduce the
oracle's field bit for bit; the reverse must match within the f32/f64 tolerances."""
import os
import socket

import numpy as np
import pytest
import torch.multiprocessing as mp

from _dist_common import O, NumpyOps, gp, small_problem


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, dt_name, min_shard, q):
    import torch
    import torch.distributed as dist
    from graphgp_b200.distributed import ShardedGenerate
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        dt = np.dtype(dt_name).type
        args = small_problem(dt)
        prob = gp.GraphGPProblem(*args, dtype=dt)
        orc = O.make_problem(*args, dt)
        sg = ShardedGenerate(prob, ops=NumpyOps(orc, dt), device="cpu", min_shard=min_shard)
        rng = np.random.default_rng(5)
        xi = rng.standard_normal(prob.npoints()).astype(dt)
        vb = rng.standard_normal(prob.npoints()).astype(dt)
        f = sg.generate(torch.from_numpy(xi)).numpy()
        xg = sg.generate_grad_xi(torch.from_numpy(vb)).numpy()
        sharded = (sum(b.sharded for b in sg.batches), sum(not b.sharded for b in sg.batches))
        q.put((rank, f, xg, sharded, O.generate(orc, xi), O.generate_grad_xi(orc, vb)))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,dt_name,min_shard", [(2, "float64", 8), (3, "float32", 8),
                                                      (2, "float32", 150)])
def test_level_sharded_orchestration(world, dt_name, min_shard):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, dt_name, min_shard, q))
             for r in range(world)]
    for p in procs:
        p.start()
    res = [q.get(timeout=300) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    tol = 1e-12 if dt_name == "float64" else 1e-5
    for rank, f, xg, sharded, f_ref, xg_ref in res:
        assert sharded[0] > 0 and (min_shard < 100 or sharded[1] > 0)
        assert np.array_equal(f, f_ref), f"rank {rank}: sharded forward differs from the oracle"
        err = np.linalg.norm(xg - xg_ref) / np.linalg.norm(xg_ref)
        assert err < tol, f"rank {rank}: grad_xi relerr {err}"


def test_plan_batches_covers_every_point():
    from graphgp_b200.distributed import plan_batches
    offs = [10, 11, 50, 51, 400, 1000]
    for world in (1, 2, 3, 8):
        batches, slack = plan_batches(offs, world, min_shard=4)
        seen = np.zeros(1000, int)
        for b in batches:
            if b.sharded:
                for r in range(world):
                    a, e = b.mine(r)
                    seen[a:e] += 1
                assert b.lo + world * b.chunk <= 1000 + slack
            else:
                seen[b.lo:b.hi] += 1
        assert np.all(seen[10:] == 1)
