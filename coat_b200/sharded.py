"""ZeRO-style sharding of the fused FP8 AdamW step across the GPUs of one node.

The step has no exchange at all: every 128-element group is independent.  The flat list of
groups of all parameter tensors is cut into `world_size` contiguous ranges; a cut never falls
inside a group (boundaries are multiples of 128 elements from each tensor's start), so every
code, scale and exponent is identical to the single-GPU run.  Each rank keeps its slice of the
fp32 master weights, gradients, E4M3 moments and per-group vectors, runs ONE persistent kernel
over its slice, which also emits the bf16 copy of the updated weights, and the only collective
is the all-gather of those bf16 slices (NCCL over NVLink; `gloo` in the CPU tests of the plan).

The reference has no counterpart: it leaves data parallelism to the host framework's FSDP
(examples/ToolBench/scripts/train_toolllama_fp8.sh:28-29), whose arbitrary shard boundaries
change the grouping.
"""
from dataclasses import dataclass
from typing import List, Sequence

import numpy as np
import torch

GROUP = 128


@dataclass
class Piece:
    tensor: int   # index into the list of parameter tensors
    start: int    # first element of the tensor that this rank owns (multiple of 128)
    stop: int     # one past the last element
    offset: int   # element offset of the piece inside the rank's flat shard (multiple of 128)

    @property
    def numel(self):
        return self.stop - self.start


class ShardPlan:
    """Which elements of which tensor each rank owns."""

    def __init__(self, numels: Sequence[int], world_size: int):
        if world_size < 1:
            raise ValueError("world_size must be >= 1")
        self.numels = [int(n) for n in numels]
        self.world_size = world_size
        groups = [(n + GROUP - 1) // GROUP for n in self.numels]
        self.group_prefix = np.concatenate([[0], np.cumsum(groups)]).astype(np.int64)
        self.total_groups = int(self.group_prefix[-1])
        base, rem = divmod(self.total_groups, world_size)
        sizes = [base + (1 if r < rem else 0) for r in range(world_size)]
        self.rank_group_lo = np.concatenate([[0], np.cumsum(sizes)]).astype(np.int64)
        # every rank's flat shard has the same capacity so that one all-gather moves them
        self.shard_groups = max(sizes) if sizes else 0
        self.shard_numel = self.shard_groups * GROUP

    def pieces(self, rank: int) -> List[Piece]:
        lo, hi = int(self.rank_group_lo[rank]), int(self.rank_group_lo[rank + 1])
        out = []
        offset = 0
        t = int(np.searchsorted(self.group_prefix, lo, side="right") - 1)
        g = lo
        while g < hi and t < len(self.numels):
            t_lo, t_hi = int(self.group_prefix[t]), int(self.group_prefix[t + 1])
            if t_hi <= g:
                t += 1
                continue
            take_hi = min(hi, t_hi)
            start = (g - t_lo) * GROUP
            stop = min((take_hi - t_lo) * GROUP, self.numels[t])
            out.append(Piece(t, start, stop, offset))
            offset += (take_hi - g) * GROUP
            g = take_hi
        return out

    def owner_of(self, tensor: int, element: int) -> int:
        g = int(self.group_prefix[tensor]) + element // GROUP
        return int(np.searchsorted(self.rank_group_lo, g, side="right") - 1)


class ShardedCoatAdamW:
    """One rank's slice of the optimizer: flat buffers, one fused launch, one all-gather.

    `process_group=None` with world_size 1 skips the collective.  Gradients are written by the
    caller into `self.grad` (already reduce-scattered, as under ZeRO); the updated bf16 weights of
    ALL ranks appear in `self.gathered` after step()."""

    def __init__(self, numels, rank=0, world_size=1, device="cuda", lr=1e-3, betas=(0.9, 0.999), eps=1e-8,
                 weight_decay=1e-2, expand_min=16, use_expansion=True, process_group=None, flags=0):
        from . import _lib
        self._lib = _lib
        self.plan = ShardPlan(numels, world_size)
        self.rank, self.world_size = rank, world_size
        self.device = torch.device(device)
        self.hyper = dict(lr=lr, betas=betas, eps=eps, weight_decay=weight_decay, expand_min=expand_min)
        self.use_expansion = use_expansion
        self.process_group = process_group
        self.flags = flags
        self.step_count = 0
        self.my_pieces = self.plan.pieces(rank)
        n, g = self.plan.shard_numel, self.plan.shard_groups
        dev = self.device
        self.param = torch.zeros(n, dtype=torch.float32, device=dev)
        self.grad = torch.zeros(n, dtype=torch.float32, device=dev)
        self.exp_avg = torch.zeros(n, dtype=torch.uint8, device=dev)
        self.exp_avg_sq = torch.zeros(n, dtype=torch.uint8, device=dev)
        self.scale_exp_avg = torch.zeros(g, dtype=torch.float32, device=dev)
        self.scale_exp_avg_sq = torch.zeros(g, dtype=torch.float32, device=dev)
        self.expand_exp_avg = torch.ones(g, dtype=torch.float32, device=dev)
        self.expand_exp_avg_sq = torch.ones(g, dtype=torch.float32, device=dev)
        self.sqrt_minmax_exp_avg = torch.ones(g, dtype=torch.float32, device=dev)
        self.sqrt_minmax_exp_avg_sq = torch.ones(g, dtype=torch.float32, device=dev)
        # all ranks' bf16 slices, rank-major; this rank's kernel writes straight into its own slot
        self.gathered = torch.zeros(world_size * n, dtype=torch.bfloat16, device=dev)
        self.bf16_shard = self.gathered[rank * n:(rank + 1) * n]
        self._build_table()

    def _build_table(self):
        L = self._lib
        rows = np.zeros(len(self.my_pieces), dtype=[(k, np.uint64) for k in
                        ("p", "g", "m", "v", "s_m", "k_m", "r_m", "s_v", "k_v", "r_v", "bf16_out")]
                        + [("numel", np.int64)])
        prefix = np.zeros(len(self.my_pieces) + 1, dtype=np.int64)
        for i, pc in enumerate(self.my_pieces):
            o, go = pc.offset, pc.offset // GROUP
            r = rows[i]
            r["p"] = self.param.data_ptr() + 4 * o
            r["g"] = self.grad.data_ptr() + 4 * o
            r["m"] = self.exp_avg.data_ptr() + o
            r["v"] = self.exp_avg_sq.data_ptr() + o
            r["s_m"] = self.scale_exp_avg.data_ptr() + 4 * go
            r["s_v"] = self.scale_exp_avg_sq.data_ptr() + 4 * go
            r["k_m"] = self.expand_exp_avg.data_ptr() + 4 * go
            r["k_v"] = self.expand_exp_avg_sq.data_ptr() + 4 * go
            r["r_m"] = self.sqrt_minmax_exp_avg.data_ptr() + 4 * go
            r["r_v"] = self.sqrt_minmax_exp_avg_sq.data_ptr() + 4 * go
            r["bf16_out"] = self.bf16_shard.data_ptr() + 2 * o
            r["numel"] = pc.numel
            prefix[i + 1] = prefix[i] + (pc.numel + GROUP - 1) // GROUP
        self._table = torch.from_numpy(rows.view(np.uint8).reshape(-1).copy()).to(self.device)
        self._prefix = torch.from_numpy(prefix).to(self.device)
        self._total_groups = int(prefix[-1])
        assert L.CoatAdamwTensor  # the row layout above mirrors this ctypes structure

    def local_step(self):
        """The fused kernel over this rank's slice (no communication)."""
        L = self._lib
        self.step_count += 1
        h = self.hyper
        if not self.my_pieces:
            return
        with torch.cuda.device(self.device):
            rc = L.lib().coat_fp8_adamw_multi_step(
                self._table.data_ptr(), self._prefix.data_ptr(), len(self.my_pieces), self._total_groups,
                int(self.use_expansion), h["betas"][0], h["betas"][1], h["lr"], h["weight_decay"], h["eps"],
                self.step_count, GROUP, h["expand_min"], L.F32, self.flags, L.stream_ptr(self.device))
        L.check(rc, "fp8_adamw_multi_step")

    def gather(self):
        """All-gather of the bf16 slices, in place in `self.gathered`."""
        if self.world_size == 1:
            return
        import torch.distributed as dist
        dist.all_gather_into_tensor(self.gathered, self.bf16_shard, group=self.process_group)

    def step(self):
        self.local_step()
        self.gather()

    def weight_views(self, shapes):
        """bf16 views of the full parameter tensors inside `self.gathered`, for tensors that are not
        split across ranks (a split tensor is returned as the list of its pieces' views)."""
        n = self.plan.shard_numel
        out = [[] for _ in shapes]
        for r in range(self.world_size):
            for pc in self.plan.pieces(r):
                out[pc.tensor].append(self.gathered[r * n + pc.offset: r * n + pc.offset + pc.numel])
        return [v[0].view(shapes[i]) if len(v) == 1 else v for i, v in enumerate(out)]
