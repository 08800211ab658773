"""CPU tests of the ZeRO-style shard plan, including a world_size-2 gloo run of the gather step."""
import os

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from coat_b200.sharded import GROUP, ShardPlan


def llama2_7b_numels():
    H, I, V, L = 4096, 11008, 32000, 32
    per_layer = [H * H] * 4 + [I * H, I * H, H * I, H, H]
    return [V * H] + per_layer * L + [H, V * H]


def test_llama2_7b_inventory():
    n = llama2_7b_numels()
    assert len(n) == 291 and sum(n) == 6_738_415_616


@pytest.mark.parametrize("world", [1, 2, 3, 4, 8])
def test_plan_covers_every_group_once(world):
    numels = [128 * 5, 77, 128 * 3 + 1, 4096, 1, 128 * 128, 300]
    plan = ShardPlan(numels, world)
    seen = [np.zeros(n, dtype=np.int32) for n in numels]
    for r in range(world):
        off = 0
        for pc in plan.pieces(r):
            assert pc.start % GROUP == 0 and pc.offset % GROUP == 0 and pc.offset == off
            assert pc.stop == numels[pc.tensor] or pc.stop % GROUP == 0
            seen[pc.tensor][pc.start:pc.stop] += 1
            off += (pc.numel + GROUP - 1) // GROUP * GROUP
            assert plan.owner_of(pc.tensor, pc.start) == r and plan.owner_of(pc.tensor, pc.stop - 1) == r
        assert off <= plan.shard_numel
    assert all((s == 1).all() for s in seen)
    sizes = np.diff(plan.rank_group_lo)
    assert sizes.max() - sizes.min() <= 1


def test_llama_plan_is_balanced_at_8():
    plan = ShardPlan(llama2_7b_numels(), 8)
    assert plan.total_groups == 6_738_415_616 // 128
    assert plan.total_groups % 8 == 0 and plan.shard_numel * 8 == 6_738_415_616


def _gather_worker(rank, world, port, numels):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        plan = ShardPlan(numels, world)
        n = plan.shard_numel
        gathered = torch.zeros(world * n, dtype=torch.bfloat16)
        mine = gathered[rank * n:(rank + 1) * n]
        # each rank fills its pieces with (tensor index + 1)
        for pc in plan.pieces(rank):
            mine[pc.offset:pc.offset + pc.numel] = pc.tensor + 1
        dist.all_gather_into_tensor(gathered, mine.clone())
        for r in range(world):
            for pc in plan.pieces(r):
                seg = gathered[r * n + pc.offset: r * n + pc.offset + pc.numel]
                assert (seg == pc.tensor + 1).all()
    finally:
        dist.destroy_process_group()


def test_gather_of_bf16_slices_world2_gloo():
    numels = [128 * 5, 77, 128 * 3 + 1, 4096, 1, 128 * 9]
    port = 29500 + os.getpid() % 2000
    mp.spawn(_gather_worker, args=(2, port, numels), nprocs=2, join=True)
