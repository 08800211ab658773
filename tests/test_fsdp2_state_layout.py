"""CoatAdamW on DTensor parameters (FSDP2 / `fully_shard`): the layout of the optimizer state, on two gloo ranks on
the CPU (the step itself needs the CUDA kernels: tests/test_fsdp2_gpu.py).

The reference leaves FSDP2 as future work (README "To-Do List") and shards nothing itself; what it fixes is the
state of ONE tensor: E4M3 moments of the parameter's shape and one fp32 scale / exponent / sqrt(max*min) per 128
consecutive elements of the flattened tensor (coat/optimizer/fp8_adamw.py:117-140).  Under dimension-0 sharding with
rows that are whole groups, every rank's groups are groups of the flattened full tensor, so the sharded state is the
unsharded state cut along rows: that is what these tests pin."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from torch.distributed.device_mesh import init_device_mesh
        from torch.distributed.tensor import DTensor, Replicate, Shard, distribute_tensor

        from coat_b200.optimizer.fp8_adamw import CoatAdamW, _group_state_layout, local_tensor
        from coat_b200.utils._fp8_quantization_config import QuantizationConfig
        mesh = init_device_mesh("cpu", (world,))
        torch.manual_seed(0)
        full = {"w": torch.randn(6, 256), "norm": torch.randn(512), "odd": torch.randn(5, 96), "rep": torch.randn(300),
                "short": torch.randn(200)}
        params = {k: torch.nn.Parameter(distribute_tensor(v, mesh, [Replicate()] if k == "rep" else [Shard(0)]))
                  for k, v in full.items()}
        opt = CoatAdamW(list(params.values()), qargs=QuantizationConfig(first_order_expansion="true",
                                                                        second_order_expansion="true"))
        res = {}
        for name, p in params.items():
            st = opt._init_state(p, True, False)
            lay = _group_state_layout(p, 128)
            res[name + "/layout"] = None if lay is None else tuple(lay[0])
            res[name + "/moment_is_dtensor"] = isinstance(st["exp_avg"], DTensor) and st["exp_avg"].shape == p.shape
            res[name + "/moment_local"] = tuple(local_tensor(st["exp_avg"]).shape)
            res[name + "/moment_dtype"] = str(st["exp_avg"].dtype)
            res[name + "/scale_is_dtensor"] = isinstance(st["scale_exp_avg"], DTensor)
            res[name + "/scale_local"] = local_tensor(st["scale_exp_avg"]).numel()
            res[name + "/expected_local_groups"] = -(-local_tensor(p).numel() // 128)
            if isinstance(st["expand_exp_avg"], DTensor):
                # write this rank's id into its local groups: the full tensor must show the ranks row block by row block
                local_tensor(st["expand_exp_avg"]).fill_(float(rank + 1))
                res[name + "/full"] = st["expand_exp_avg"].full_tensor().flatten().tolist()
        if rank == 0:
            out.put(res)
    finally:
        dist.destroy_process_group()


def test_state_layout_on_two_gloo_ranks():
    ctx = mp.get_context("spawn")
    out = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, out)) for r in range(2)]
    for p in procs:
        p.start()
    res = out.get(timeout=120)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    # [6, 256] over 2 ranks: 3 rows each, 2 groups per row: the group vector is a [6, 2] matrix sharded by rows
    assert res["w/layout"] == (6, 2) and res["w/moment_is_dtensor"] and res["w/scale_is_dtensor"]
    assert res["w/moment_local"] == (3, 256) and res["w/moment_dtype"] == "torch.float8_e4m3fn"
    assert res["w/scale_local"] == res["w/expected_local_groups"] == 6
    assert res["w/full"] == [1.0] * 6 + [2.0] * 6
    # a [512] vector: 256 elements = 2 groups per rank
    assert res["norm/layout"] == (4,) and res["norm/scale_is_dtensor"] and res["norm/full"] == [1.0, 1.0, 2.0, 2.0]
    # rows of 96 elements are not whole groups: the groups of a shard are not groups of the full tensor -> rank-local
    assert res["odd/layout"] is None and not res["odd/scale_is_dtensor"] and res["odd/moment_is_dtensor"]
    assert res["odd/scale_local"] == res["odd/expected_local_groups"] == 3      # 3 rows x 96 = 288 elements
    # replicated: the local tensor is the full tensor
    assert res["rep/layout"] == (3,) and res["rep/scale_is_dtensor"] and res["rep/scale_local"] == 3
    # [200] over 2 ranks: chunks of 100 elements are not whole groups
    assert res["short/layout"] is None and res["short/scale_local"] == 1


def test_plain_tensors_are_untouched():
    from coat_b200.optimizer.fp8_adamw import CoatAdamW, local_tensor
    p = torch.nn.Parameter(torch.randn(4, 128))
    assert local_tensor(p) is p
    opt = CoatAdamW([p])
    st = opt._init_state(p, True, False)
    assert type(st["exp_avg"]) is torch.Tensor and st["scale_exp_avg"].shape == (4,)
