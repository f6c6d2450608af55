"""
Rank shares of the data-parallel workload (mlip.sharded_workload): every
system of the global pool goes to exactly one rank, with its own positions
and species; per-rank atom counts differ by less than one system; one rank
gets the whole pool, the same batch as the unsharded workload.
"""

from __future__ import annotations

import pytest
import torch

from create_graph_b200 import mlip


@pytest.mark.parametrize("world", [1, 2, 3, 8])
def test_shares_partition_the_pool(world):
    sizes = mlip.workload_sizes("allscaip_85m", seed=1000, atoms_target=world * 2048)
    pos, species, sys_ptr = mlip.synthetic_systems(sizes, mlip.ALLSCAIP_85M.n_species, seed=1000)
    pool = {tuple(pos[sys_ptr[b]:sys_ptr[b + 1]].flatten().tolist()): b for b in range(len(sizes))}
    seen, totals = [], []
    for rank in range(world):
        s, p, sp, ptr = mlip.sharded_workload("allscaip_85m", rank, world, 2048)
        assert ptr[-1] == p.shape[0] == sp.shape[0] == sum(s)
        totals.append(sum(s))
        for b in range(len(s)):
            key = tuple(p[ptr[b]:ptr[b + 1]].flatten().tolist())
            g = pool[key]
            assert s[b] == sizes[g]
            assert torch.equal(sp[ptr[b]:ptr[b + 1]], species[sys_ptr[g]:sys_ptr[g + 1]])
            seen.append(g)
    assert sorted(seen) == list(range(len(sizes)))
    assert max(totals) - min(totals) < max(sizes)


def test_one_rank_gets_the_unsharded_batch():
    s, p, sp, ptr = mlip.sharded_workload("allscaip_85m", 0, 1, 8192)
    sizes = mlip.workload_sizes("allscaip_85m", seed=1000, atoms_target=8192)
    pos, species, sys_ptr = mlip.synthetic_systems(sizes, mlip.ALLSCAIP_85M.n_species, seed=1000)
    assert s == sizes and torch.equal(p, pos) and torch.equal(sp, species) and torch.equal(ptr, sys_ptr)
