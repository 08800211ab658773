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


@pytest.mark.parametrize("world,buckets", [(1, 1), (2, 3), (3, 8), (8, 4), (2, 1000)])
def test_bucket_pieces_cover_every_element_once(world, buckets):
    numels = [128 * 5, 77, 128 * 3 + 1, 4096, 1, 128 * 128, 300]
    plan = ShardPlan(numels, world)
    bounds = plan.bucket_bounds(buckets) * GROUP
    assert bounds[0] == 0 and bounds[-1] == plan.shard_numel and (np.diff(bounds) > 0).all()
    seen = [np.zeros(n, dtype=np.int32) for n in numels]
    slots = np.zeros(world * plan.shard_numel, dtype=np.int32)
    for r in range(world):
        per_bucket = plan.bucket_pieces(r, buckets)
        assert len(per_bucket) == len(bounds) - 1
        for b, pcs in enumerate(per_bucket):
            for pc in pcs:
                assert pc.numel > 0 and pc.start % GROUP == 0 and pc.offset % GROUP == 0
                assert bounds[b] <= pc.offset and pc.offset + pc.numel <= bounds[b + 1]
                seen[pc.tensor][pc.start:pc.stop] += 1
                o = plan.gathered_offset(r, pc.offset, buckets)
                # a piece is contiguous in the gathered buffer and lies in its rank's slot of bucket b
                size = int(bounds[b + 1] - bounds[b])
                lo = int(bounds[b]) * world + r * size
                assert lo <= o and o + pc.numel <= lo + size
                slots[o:o + pc.numel] += 1
    assert all((s == 1).all() for s in seen)
    assert slots.max() == 1 and slots.sum() == sum(numels)


def _bucketed_gather_worker(rank, world, port, numels, buckets):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        plan = ShardPlan(numels, world)
        bounds = plan.bucket_bounds(buckets) * GROUP
        gathered = torch.zeros(world * plan.shard_numel, dtype=torch.bfloat16)
        for pcs in plan.bucket_pieces(rank, buckets):
            for pc in pcs:
                o = plan.gathered_offset(rank, pc.offset, buckets)
                gathered[o:o + pc.numel] = torch.arange(pc.start, pc.stop).to(torch.bfloat16) + pc.tensor
        for b in range(len(bounds) - 1):
            lo, hi = int(bounds[b]), int(bounds[b + 1])
            whole = gathered[lo * world: hi * world]
            mine = whole[rank * (hi - lo):(rank + 1) * (hi - lo)]
            dist.all_gather_into_tensor(whole, mine.clone())
        for r in range(world):
            for pcs in plan.bucket_pieces(r, buckets):
                for pc in pcs:
                    o = plan.gathered_offset(r, pc.offset, buckets)
                    want = torch.arange(pc.start, pc.stop).to(torch.bfloat16) + pc.tensor
                    assert torch.equal(gathered[o:o + pc.numel], want)
    finally:
        dist.destroy_process_group()


def test_bucketed_gather_world2_gloo():
    numels = [128 * 5, 77, 128 * 3 + 1, 4096, 1, 128 * 9]
    port = 31500 + os.getpid() % 2000
    mp.spawn(_bucketed_gather_worker, args=(2, port, numels, 3), nprocs=2, join=True)


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


class _FakePeerBuffer:
    """Stand-in for the CUDA IPC buffer: records what the set-up did to it."""

    def __init__(self, rank, fail_create=False, fail_open=False):
        if fail_create:
            raise RuntimeError("out of memory (injected)")
        self.handle = f"handle-of-{rank}".encode()
        self.fail_open = fail_open
        self.peers, self.closed, self.freed = {}, False, False

    def open_peer(self, rank, handle):
        if self.fail_open:
            raise RuntimeError(f"cannot map the buffer of rank {rank} (injected)")
        assert handle == f"handle-of-{rank}".encode()
        self.peers[rank] = 1000 + rank

    def close(self):
        self.closed = True

    def free(self):
        self.freed = True


def _peer_setup_worker(rank, world, port, failing_rank, how):
    from coat_b200.sharded import exchange_peer_buffers
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        made = []

        def make():
            buf = _FakePeerBuffer(rank, fail_create=(how == "create" and rank == failing_rank),
                                  fail_open=(how == "open" and rank == failing_rank))
            made.append(buf)
            return buf

        if failing_rank is None:
            buf = exchange_peer_buffers(make, rank, world)
            assert sorted(buf.peers) == [r for r in range(world) if r != rank] and not buf.closed
        else:
            try:
                exchange_peer_buffers(make, rank, world)
            except RuntimeError as e:
                # EVERY rank raises, and the message names the rank that failed
                assert f"rank {failing_rank}" in str(e) and "injected" in str(e), str(e)
            else:
                raise AssertionError(f"rank {rank} did not see the failure of rank {failing_rank}")
            assert all(b.closed and b.freed for b in made)
        dist.barrier()   # no rank is stuck in a collective of the set-up
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("failing_rank,how", [(None, ""), (1, "open"), (0, "create")])
def test_peer_buffer_setup_failure_reaches_every_rank_world2_gloo(failing_rank, how):
    port = 33500 + os.getpid() % 2000 + (0 if failing_rank is None else 1 + failing_rank)
    mp.spawn(_peer_setup_worker, args=(2, port, failing_rank, how), nprocs=2, join=True)


def _verify_worker(rank, world, port, corrupt_rank):
    """bench.verify_gathered on two gloo ranks: consistent buffers -> True on every rank; one wrong element in ONE
    rank's copy of a peer's slot -> False on every rank."""
    import types
    import bench
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        plan = ShardPlan([128 * 5, 77, 128 * 3 + 1, 4096], world)
        n = plan.shard_numel
        bounds = plan.bucket_bounds(2)
        gen = torch.Generator().manual_seed(5)
        shards = [torch.randn(n, generator=gen) for _ in range(world)]        # every rank can rebuild every shard
        gathered = torch.zeros(world * n, dtype=torch.bfloat16)
        bucket_all = []
        for b in range(len(bounds) - 1):
            lo, hi = int(bounds[b]) * GROUP, int(bounds[b + 1]) * GROUP
            whole = gathered[lo * world: hi * world]
            for r in range(world):
                whole[r * (hi - lo):(r + 1) * (hi - lo)] = shards[r][lo:hi].to(torch.bfloat16)
            bucket_all.append(whole)
        if rank == corrupt_rank:
            gathered[3] += 1.0   # element 3 of rank 0's slot in bucket 0, as seen by `corrupt_rank` only
        opt = types.SimpleNamespace(device=torch.device("cpu"), world_size=world, rank=rank, n_buckets=len(bounds) - 1,
                                    bounds=bounds, param=shards[rank], _bucket_all=bucket_all)
        ok = bench.verify_gathered(opt, torch, dist)
        assert ok == (corrupt_rank is None), (rank, ok)
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("corrupt_rank", [None, 1])
def test_gather_verification_of_the_benchmark_world2_gloo(corrupt_rank):
    port = 35500 + os.getpid() % 2000 + (0 if corrupt_rank is None else 7)
    mp.spawn(_verify_worker, args=(2, port, corrupt_rank), nprocs=2, join=True)


@pytest.mark.parametrize("world", [2, 3, 4, 8])
@pytest.mark.parametrize("exchange,k", [("p2p", None), ("copy", None), ("hybrid", None), ("hybrid", 1), ("hybrid", 3)])
def test_exchange_routes_cover_every_pair_once(world, exchange, k):
    """Every ordered pair (sender, receiver) is served by exactly one transport, and under "hybrid" every rank
    receives from as many DMA engines as it feeds."""
    from coat_b200.sharded import exchange_routes
    served = {}
    copies_into = {r: 0 for r in range(world)}
    for rank in range(world):
        copy_ranks, store_ranks = exchange_routes(rank, world, exchange, k)
        assert rank not in copy_ranks and rank not in store_ranks
        assert not set(copy_ranks) & set(store_ranks)
        for r in copy_ranks + store_ranks:
            assert (rank, r) not in served
            served[(rank, r)] = True
        for r in copy_ranks:
            copies_into[r] += 1
        if exchange == "p2p":
            assert not copy_ranks
        if exchange == "copy":
            assert not store_ranks
    assert len(served) == world * (world - 1)
    assert len(set(copies_into.values())) == 1   # the engines' traffic is spread evenly over the receivers


def test_exchange_routes_without_peer_transport():
    from coat_b200.sharded import exchange_routes
    assert exchange_routes(1, 4, "nccl") == ([], [])
    assert exchange_routes(0, 1, "none") == ([], [])
