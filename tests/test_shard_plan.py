"""The library's sharding plan (gpb2_shard_plan, host only) against the plan of the Python
orchestration, and its invariants: every refined point is computed in the forward sweep by the
ranks that need it and its cotangent is scattered by exactly one rank."""
import numpy as np
import pytest

from graphgp_b200.distributed import library_plan, plan_batches


@pytest.mark.parametrize("world", [1, 2, 3, 4, 8])
@pytest.mark.parametrize("min_shard", [1, 7, 1000])
def test_plan_matches_python(world, min_shard):
    rng = np.random.default_rng(world * 100 + min_shard)
    sizes = np.concatenate([[500], rng.integers(0, 3000, size=40), [0, 1, 2, 5]])
    offs = np.cumsum(sizes)
    py, py_slack = plan_batches(offs, world, min_shard)
    n = int(offs[-1])
    owners = np.zeros(n, np.int64)
    for rank in range(world):
        lib, slack = library_plan(offs, world, rank, min_shard)
        assert slack == py_slack
        assert len(lib) == len(py)
        for (fwd, own, sh), b in zip(lib, py):
            assert sh == b.sharded
            assert fwd == b.mine(rank)
            c = b.chunk if b.sharded else -(-(b.hi - b.lo) // world)
            a = min(b.hi, b.lo + rank * c)
            assert own == (a, min(b.hi, a + c))
            owners[own[0]:own[1]] += 1
            assert fwd[0] <= own[0] and own[1] <= fwd[1]
    assert np.all(owners[int(offs[0]):] == 1)
