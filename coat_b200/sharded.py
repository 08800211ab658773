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

    def bucket_bounds(self, n_buckets: int) -> np.ndarray:
        """Cuts of a rank's shard (in groups, the same for every rank) into `n_buckets` near-equal
        ranges: bucket b of every rank is gathered by one collective while bucket b+1 is stepped."""
        n_buckets = max(1, min(int(n_buckets), max(self.shard_groups, 1)))
        base, rem = divmod(self.shard_groups, n_buckets)
        sizes = [base + (1 if b < rem else 0) for b in range(n_buckets)]
        return np.concatenate([[0], np.cumsum(sizes)]).astype(np.int64)

    def bucket_pieces(self, rank: int, n_buckets: int) -> List[List[Piece]]:
        """pieces(rank) cut at the bucket bounds; `offset` stays relative to the rank's shard."""
        bounds = self.bucket_bounds(n_buckets) * GROUP
        out = [[] for _ in range(len(bounds) - 1)]
        for pc in self.pieces(rank):
            span = (pc.numel + GROUP - 1) // GROUP * GROUP
            lo = pc.offset
            while lo < pc.offset + span:
                b = int(np.searchsorted(bounds, lo, side="right") - 1)
                hi = min(pc.offset + span, int(bounds[b + 1]))
                start = pc.start + (lo - pc.offset)
                out[b].append(Piece(pc.tensor, start, min(pc.stop, pc.start + (hi - pc.offset)), lo))
                lo = hi
        return out

    def gathered_offset(self, rank: int, offset: int, n_buckets: int) -> int:
        """Element offset, inside the bucket-major buffer of all ranks' bf16 weights (bucket b holds
        world_size slots of that bucket's size, rank-major), of shard-local element `offset` of `rank`."""
        bounds = self.bucket_bounds(n_buckets) * GROUP
        b = int(np.searchsorted(bounds, offset, side="right") - 1)
        size = int(bounds[b + 1] - bounds[b])
        return int(bounds[b]) * self.world_size + rank * size + (offset - int(bounds[b]))

    def owner_of(self, tensor: int, element: int) -> int:
        g = int(self.group_prefix[tensor]) + element // GROUP
        return int(np.searchsorted(self.rank_group_lo, g, side="right") - 1)


class _PeerBuffer:
    """A device buffer from coat_peer_buffer_create, exposed to torch through the CUDA array interface."""

    def __init__(self, lib_module, nbytes, device):
        import ctypes
        self._L = lib_module
        self.device = device
        self.nbytes = int(nbytes)
        ptr = ctypes.c_void_p()
        handle = ctypes.create_string_buffer(lib_module.PEER_HANDLE_BYTES)
        with torch.cuda.device(device):
            lib_module.check(lib_module.lib().coat_peer_buffer_create(self.nbytes, ctypes.byref(ptr), handle),
                             "peer_buffer_create")
        self.ptr = int(ptr.value)
        self.handle = handle.raw
        self.peers = {}   # rank -> mapped base address of that rank's buffer
        self.__cuda_array_interface__ = {"shape": (self.nbytes,), "typestr": "|u1", "data": (self.ptr, False),
                                         "version": 3, "strides": None}

    def open_peer(self, rank, handle):
        import ctypes
        ptr = ctypes.c_void_p()
        with torch.cuda.device(self.device):
            self._L.check(self._L.lib().coat_peer_buffer_open(handle, ctypes.byref(ptr)), "peer_buffer_open")
        self.peers[rank] = int(ptr.value)

    def close(self):
        for r, p in list(self.peers.items()):
            self._L.lib().coat_peer_buffer_close(p)
            del self.peers[r]

    def free(self):
        if self.ptr:
            self._L.lib().coat_peer_buffer_free(self.ptr)
            self.ptr = 0


def exchange_peer_buffers(make_buffer, rank, world_size, process_group=None):
    """Create this rank's peer-mappable buffer with `make_buffer()`, swap handles over the process group and
    map every peer's buffer (`buf.open_peer(rank, handle)`).  Returns the buffer.

    A failure on ANY rank (allocation, or mapping one peer) is raised on EVERY rank, as a RuntimeError that
    names the ranks that failed: the status travels with two object collectives that every rank takes part
    in whatever happened to it, so no rank is left waiting in a collective for one that has already raised.
    Callers may therefore fall back (e.g. to an NCCL exchange) on all ranks alike.  On failure whatever was
    mapped is unmapped and, after a barrier, the rank's own buffer is freed."""
    import torch.distributed as dist
    err, buf = None, None
    try:
        buf = make_buffer()
    except Exception as e:   # reported to every rank below
        err = f"rank {rank}: {e}"
    everyone = [None] * world_size
    dist.all_gather_object(everyone, (err, buf.handle if buf is not None else None), group=process_group)
    if not any(e for e, _ in everyone):
        try:
            for r in range(world_size):
                if r != rank:
                    buf.open_peer(r, everyone[r][1])
        except Exception as e:
            err = f"rank {rank}: {e}"
    # second collective: every rank has mapped (or failed to map) every buffer before anyone steps
    status = [None] * world_size
    dist.all_gather_object(status, err, group=process_group)
    failed = [e for e in status if e]
    if failed:
        if buf is not None:
            buf.close()
            dist.barrier(group=process_group)   # nobody maps this buffer any more
            buf.free()
        else:
            dist.barrier(group=process_group)
        raise RuntimeError("peer buffers could not be set up: " + "; ".join(failed))
    return buf


def exchange_routes(rank, world_size, exchange, copy_peers=None):
    """(ranks this rank's DMA engines copy its slice to, ranks its step kernel stores its slice to) for an exchange
    kind.  "copy": every peer by the engines; "p2p": every peer by the kernel; "hybrid": the next `copy_peers` ranks
    (about a third of the peers when None) by the engines, so that every rank also RECEIVES from exactly that many
    engines, and the rest by the kernel; "nccl" / "none": neither (NCCL moves the slices, or nobody does)."""
    n_peers = world_size - 1
    if exchange == "copy":
        k = n_peers
    elif exchange == "hybrid":
        k = copy_peers if copy_peers is not None else max(1, round(0.35 * n_peers))
        k = min(max(int(k), 0), n_peers)
    else:
        k = 0
    copy_ranks = [(rank + 1 + i) % world_size for i in range(k)]
    if exchange in ("p2p", "hybrid"):
        store_ranks = [r for r in range(world_size) if r != rank and r not in copy_ranks]
    else:
        store_ranks = []
    return copy_ranks, store_ranks


class ShardedCoatAdamW:
    """One rank's slice of the optimizer: flat buffers and one of two ways to get every rank's bf16
    weights everywhere.

    exchange="p2p" (the default with more than two ranks): ONE kernel per step does both the update and
    the exchange; it stores its bf16 slice into every peer's copy of `self.gathered` over NVLink while
    it computes (coat_fp8_adamw_multi_step_bcast), and a one-element all-reduce after it is the
    barrier that tells every rank that all slices have landed.
    exchange="nccl": one launch per bucket and one NCCL all-gather per bucket on a side stream, so
    that the gather of bucket b runs under the step of bucket b+1.
    exchange="hybrid": buckets as in "copy", but only `copy_peers` of the peers (about a third) are served by the DMA
    engines; the bucket's kernel is the fused one and stores to the others (measured equal to "p2p" at four ranks:
    what bounds the exchange there is the rate at which a GPU takes in writes from all peers at once, not the sender).
    exchange="copy" (the default with two ranks): one launch per bucket of the plain step kernel (full occupancy, no staging of the bf16 weights in
    shared memory); behind an event after bucket b's kernel, side streams (one per peer) push the bucket's bf16 slice
    into every peer's copy of `self.gathered` with asynchronous peer copies (DMA engines, no SMs) while bucket b+1 is
    stepped; the same one-element all-reduce closes the step.

    With world_size 1 there is one bucket and no exchange.  Gradients are written by the caller
    into `self.grad` (already reduce-scattered, as under ZeRO); the updated bf16 weights of ALL ranks
    appear in `self.gathered` (bucket-major, see ShardPlan.gathered_offset) after step().  No rank may
    start step k+1 while another still reads the weights of step k from `self.gathered`; in training
    the gradient reduce-scatter between the two provides that order."""

    def __init__(self, numels, rank=0, world_size=1, device="cuda", lr=1e-3, betas=(0.9, 0.999), eps=1e-8,
                 weight_decay=1e-2, expand_min=16, use_expansion=True, process_group=None, flags=0,
                 n_buckets=None, exchange=None, copy_peers=None):
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
        if exchange is None:
            # two ranks: the DMA engines hide the whole exchange under the plain kernel (21.0 ms against 26.2 ms for the
            # fused kernel on the Llama-2-7B set); more ranks: the engines sustain only 350-380 GB/s into several peers
            # (28.7 ms against 17.6 ms at four ranks, 31.0 against 18.8 ms at eight), the fused kernel's stores 570-630
            exchange = "none" if world_size == 1 else ("copy" if world_size == 2 else "p2p")
        if exchange not in ("none", "p2p", "nccl", "copy", "hybrid") or (exchange == "none") != (world_size == 1):
            raise ValueError(f"exchange={exchange!r} does not fit world_size={world_size}")
        if exchange in ("p2p", "hybrid") and world_size - 1 > _lib.MAX_PEERS:
            raise ValueError(f"the p2p exchange serves at most {_lib.MAX_PEERS + 1} ranks")
        self.exchange = exchange
        if n_buckets is None:
            # (copy exchange at two ranks, ms per step of the Llama-2-7B set: 4 buckets 23.1, 8: 21.6, 16: 21.0, 32: 20.9)
            n_buckets = 16 if exchange == "copy" else (8 if exchange in ("nccl", "hybrid") else 1)
        self.bounds = self.plan.bucket_bounds(n_buckets)
        self.n_buckets = len(self.bounds) - 1
        self.my_buckets = self.plan.bucket_pieces(rank, self.n_buckets)
        self.my_pieces = [pc for b in self.my_buckets for pc in b]
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
        # all ranks' bf16 slices, bucket-major; this rank's kernel writes straight into its own slots
        self._peer_buffer = None
        self._peer_deltas = None
        self._n_store_peers = None   # how many entries of _peer_deltas the kernel stores to (None: all of them)
        # which peers receive this rank's slice from the DMA engines and which from the kernel's stores
        self._copy_ranks, self._store_ranks = exchange_routes(rank, world_size, exchange, copy_peers)
        if exchange in ("p2p", "copy", "hybrid"):
            self._setup_peer_buffer(world_size * n * 2)
        else:
            self.gathered = torch.zeros(world_size * n, dtype=torch.bfloat16, device=dev)
        self._bucket_all, self._bucket_mine = [], []
        for b in range(self.n_buckets):
            lo, hi = int(self.bounds[b]) * GROUP, int(self.bounds[b + 1]) * GROUP
            whole = self.gathered[lo * world_size: hi * world_size]
            self._bucket_all.append(whole)
            self._bucket_mine.append(whole[rank * (hi - lo):(rank + 1) * (hi - lo)])
        self._comm = torch.cuda.Stream(device=dev) if exchange == "nccl" else None
        self._copy_streams = [torch.cuda.Stream(device=dev) for _ in self._copy_ranks]
        self._events = [torch.cuda.Event() for _ in range(self.n_buckets)] if (self._comm or self._copy_streams) else []
        self._table_cache = {}
        self.set_grad_buffer(self.grad)

    def _setup_peer_buffer(self, nbytes):
        """Allocate this rank's gathered-weights buffer so that peers can map it, swap handles and map every
        peer's buffer (exchange_peer_buffers: a failure on any rank is raised on every rank)."""
        import ctypes
        buf = exchange_peer_buffers(lambda: _PeerBuffer(self._lib, nbytes, self.device), self.rank, self.world_size,
                                    self.process_group)
        self._peer_buffer = buf
        self.gathered = torch.as_tensor(buf, device=self.device).view(torch.bfloat16)
        deltas = [buf.peers[r] - buf.ptr for r in self._store_ranks]
        self._peer_deltas = (ctypes.c_int64 * max(1, len(deltas)))(*deltas)
        self._n_store_peers = len(deltas)
        self._flag = torch.zeros(1, dtype=torch.float32, device=self.device)

    def close(self):
        """Unmap the peers' buffers and free this rank's (collective: every rank calls it)."""
        if self._peer_buffer is not None:
            import torch.distributed as dist
            torch.cuda.synchronize(self.device)
            self._peer_buffer.close()
            dist.barrier(group=self.process_group)   # nobody maps this buffer any more
            del self.gathered, self._bucket_all, self._bucket_mine
            self._peer_buffer.free()
            self._peer_buffer = None

    def set_grad_buffer(self, grad):
        """Point the step at another flat gradient buffer of the shard's size (the device-side tensor
        tables are built once per buffer and reused)."""
        if grad.numel() != self.plan.shard_numel or grad.dtype != torch.float32:
            raise ValueError("gradient buffer must be fp32 with the shard's number of elements")
        self.grad = grad
        key = grad.data_ptr()
        if key not in self._table_cache:
            self._table_cache[key] = [self._build_table(pcs) for pcs in self.my_buckets]
        self._tables = self._table_cache[key]

    def _build_table(self, pieces):
        L = self._lib
        rows = np.zeros(len(pieces), dtype=[(k, np.uint64) for k in
                        ("p", "g", "m", "v", "s_m", "k_m", "r_m", "s_v", "k_v", "r_v", "bf16_out")]
                        + [("numel", np.int64)])
        prefix = np.zeros(len(pieces) + 1, dtype=np.int64)
        for i, pc in enumerate(pieces):
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
            r["bf16_out"] = self.gathered.data_ptr() + 2 * self.plan.gathered_offset(self.rank, o, self.n_buckets)
            r["numel"] = pc.numel
            prefix[i + 1] = prefix[i] + (pc.numel + GROUP - 1) // GROUP
        assert L.CoatAdamwTensor  # the row layout above mirrors this ctypes structure
        return (torch.from_numpy(rows.view(np.uint8).reshape(-1).copy()).to(self.device),
                torch.from_numpy(prefix).to(self.device), len(pieces), int(prefix[-1]))

    def _launch_bucket(self, b, bcast=False):
        L = self._lib
        h = self.hyper
        table, prefix, n_pieces, n_groups = self._tables[b]
        if n_pieces == 0:
            return
        with torch.cuda.device(self.device):
            if bcast:
                rc = L.lib().coat_fp8_adamw_multi_step_bcast(
                    table.data_ptr(), prefix.data_ptr(), n_pieces, n_groups,
                    int(self.use_expansion), h["betas"][0], h["betas"][1], h["lr"], h["weight_decay"], h["eps"],
                    self.step_count, GROUP, h["expand_min"], L.F32, self.flags, self._peer_deltas,
                    len(self._peer_deltas) if self._n_store_peers is None else self._n_store_peers,
                    L.stream_ptr(self.device))
            else:
                rc = L.lib().coat_fp8_adamw_multi_step(
                    table.data_ptr(), prefix.data_ptr(), n_pieces, n_groups,
                    int(self.use_expansion), h["betas"][0], h["betas"][1], h["lr"], h["weight_decay"], h["eps"],
                    self.step_count, GROUP, h["expand_min"], L.F32, self.flags, L.stream_ptr(self.device))
        L.check(rc, "fp8_adamw_multi_step")

    def local_step(self):
        """The fused kernel over this rank's slice (no communication)."""
        self.step_count += 1
        for b in range(self.n_buckets):
            self._launch_bucket(b)

    def gather(self):
        """All-gather of the bf16 slices, in place in `self.gathered`."""
        if self.world_size == 1:
            return
        import torch.distributed as dist
        if self.exchange in ("p2p", "copy", "hybrid"):
            raise RuntimeError(f"exchange='{self.exchange}' has no separate gather: step() does both")
        for b in range(self.n_buckets):
            dist.all_gather_into_tensor(self._bucket_all[b], self._bucket_mine[b], group=self.process_group)

    def step(self):
        """Step and gather, pipelined by bucket: the collective of bucket b is queued on a side stream
        behind an event recorded after bucket b's kernel, and runs while bucket b+1 is stepped."""
        import torch.distributed as dist
        if self.exchange == "p2p":
            self.step_count += 1
            for b in range(self.n_buckets):
                self._launch_bucket(b, bcast=True)
            # stream-ordered barrier: it completes on a rank only after every rank's kernel has
            dist.all_reduce(self._flag, group=self.process_group)
            return
        if self.exchange in ("copy", "hybrid"):
            compute = torch.cuda.current_stream(self.device)
            for st in self._copy_streams:
                st.wait_stream(compute)   # readers of the previous step's gathered weights are done
            self.step_count += 1
            base = self._peer_buffer.ptr
            for b in range(self.n_buckets):
                # the kernel's own stores serve `_store_ranks` (none of them: the plain kernel at full occupancy)
                self._launch_bucket(b, bcast=bool(self._n_store_peers))
                self._events[b].record(compute)
                mine = self._bucket_mine[b]
                nbytes = mine.numel() * 2
                if nbytes == 0:
                    continue
                offset = mine.data_ptr() - base
                for peer, st in zip(self._copy_ranks, self._copy_streams):
                    st.wait_event(self._events[b])
                    self._lib.check(self._lib.lib().coat_peer_copy_async(
                        self._peer_buffer.peers[peer] + offset, mine.data_ptr(), nbytes, st.cuda_stream), "peer_copy_async")
            for st in self._copy_streams:
                compute.wait_stream(st)
            dist.all_reduce(self._flag, group=self.process_group)   # every rank's stores and copies have landed everywhere
            return
        if self.world_size == 1 or self._comm is None:
            self.local_step()
            self.gather()
            return
        compute = torch.cuda.current_stream(self.device)
        self._comm.wait_stream(compute)   # readers of the previous step's gathered weights are done
        self.step_count += 1
        for b in range(self.n_buckets):
            self._launch_bucket(b)
            self._events[b].record(compute)
            with torch.cuda.stream(self._comm):
                self._comm.wait_event(self._events[b])
                dist.all_gather_into_tensor(self._bucket_all[b], self._bucket_mine[b], group=self.process_group)
        compute.wait_stream(self._comm)

    def weight_views(self, shapes):
        """bf16 views of the full parameter tensors inside `self.gathered`: one view for a tensor that
        lies in one bucket of one rank, else the list of its pieces' views in element order."""
        out = [[] for _ in shapes]
        for r in range(self.world_size):
            for pcs in self.plan.bucket_pieces(r, self.n_buckets):
                for pc in pcs:
                    o = self.plan.gathered_offset(r, pc.offset, self.n_buckets)
                    out[pc.tensor].append((pc.start, self.gathered[o:o + pc.numel]))
        views = [[v for _, v in sorted(lst, key=lambda t: t[0])] for lst in out]
        return [v[0].view(shapes[i]) if len(v) == 1 else v for i, v in enumerate(views)]
