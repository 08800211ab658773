"""CoatAdamW under FSDP2 (`torch.distributed.fsdp.fully_shard`): parameters, gradients and optimizer state are DTensors,
the fused kernel steps every rank's local shard.  Checked against the same model trained unsharded with the same
optimizer: with rows that are whole groups of 128 the local groups are the groups of the full tensors, so parameters,
FP8 moments, scales, exponents and sqrt(max*min) must be IDENTICAL bit for bit to the unsharded run (every rank sees
the same batch, so the averaged gradient equals the single-process gradient exactly), and a state dict saved from the
sharded optimizer must continue to the same bits.  World size 1 runs everywhere (one NCCL rank: the DTensor plumbing);
world size 2 needs two GPUs."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


class _Net(torch.nn.Module):
    def __init__(self):
        super().__init__()
        self.a = torch.nn.Linear(256, 512, bias=False)
        self.norm = torch.nn.LayerNorm(512)          # weight and bias of 512: 1-D parameters
        self.b = torch.nn.Linear(512, 256, bias=False)

    def forward(self, x):
        return self.b(self.norm(torch.nn.functional.silu(self.a(x))))


def _worker(rank, world, port, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=torch.device("cuda", rank))
    try:
        from torch.distributed.device_mesh import init_device_mesh
        from torch.distributed.fsdp import fully_shard
        from torch.distributed.tensor import DTensor

        from coat_b200.optimizer.fp8_adamw import CoatAdamW, local_tensor
        from coat_b200.utils._fp8_quantization_config import QuantizationConfig
        qargs = QuantizationConfig(first_order_expansion="true", second_order_expansion="true")
        torch.manual_seed(0)
        plain = _Net().cuda()
        sharded = _Net().cuda()
        sharded.load_state_dict(plain.state_dict())
        mesh = init_device_mesh("cuda", (world,))
        fully_shard(sharded, mesh=mesh)
        kw = dict(lr=1e-3, betas=(0.9, 0.95), weight_decay=0.1, qargs=qargs)
        opt_plain, opt_sharded = CoatAdamW(plain.parameters(), **kw), CoatAdamW(sharded.parameters(), **kw)
        gen = torch.Generator(device="cuda").manual_seed(1)
        batches = [torch.randn(64, 256, generator=gen, device="cuda") for _ in range(6)]

        def train(model, opt, xs):
            for x in xs:
                opt.zero_grad(set_to_none=True)
                model(x).square().mean().backward()
                opt.step()

        train(plain, opt_plain, batches[:3])
        train(sharded, opt_sharded, batches[:3])
        problems = []

        def compare(tag):
            for (n, p), (_, q) in zip(plain.named_parameters(), sharded.named_parameters()):
                if not isinstance(q, DTensor):
                    problems.append(f"{tag}: {n} is not a DTensor")
                    continue
                if not torch.equal(q.full_tensor(), p):
                    problems.append(f"{tag}: parameter {n} differs")
                sp, sq = opt_plain.state[p], opt_sharded.state[q]
                for k, v in sp.items():
                    w = sq[k]
                    if k == "step":
                        ok = float(v) == float(w)
                    else:
                        if not isinstance(w, DTensor):
                            problems.append(f"{tag}: state {k} of {n} is rank-local")
                            continue
                        full = w.full_tensor()
                        ok = torch.equal(full.reshape(-1).view(torch.uint8), v.reshape(-1).view(torch.uint8))
                    if not ok:
                        problems.append(f"{tag}: state {k} of {n} differs")

        compare("after 3 steps")
        # save from the sharded optimizer, load into a fresh one, continue: same bits as the uninterrupted plain run
        saved = opt_sharded.state_dict()
        opt_sharded = CoatAdamW(sharded.parameters(), **kw)
        opt_sharded.load_state_dict(saved)
        for q in sharded.parameters():
            st = opt_sharded.state[q]
            if st["exp_avg"].dtype != torch.float8_e4m3fn or local_tensor(st["exp_avg"]).device.type != "cuda":
                problems.append("loaded state changed dtype or device")
        train(plain, opt_plain, batches[3:])
        train(sharded, opt_sharded, batches[3:])
        compare("after reload and 3 more steps")
        if rank == 0:
            out.put(problems)
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [1, 2])
def test_fsdp2_training_equals_unsharded_training_bit_for_bit(world):
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    ctx = mp.get_context("spawn")
    out = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, out)) for r in range(world)]
    for p in procs:
        p.start()
    try:
        problems = out.get(timeout=300)
    finally:
        for p in procs:
            p.join(timeout=120)
    assert all(p.exitcode == 0 for p in procs)
    assert problems == [], problems
