"""CoatAdamW: AdamW whose moments live in FP8 (E4M3, groups of 128, optional Dynamic
Range Expansion), stepping through the fused sm_100a kernel.

Drop-in for coat/optimizer/fp8_adamw.py: same constructor (:37-48), same per-parameter
state keys, shapes and dtypes (:117-140), state dicts load without casting the
quantized state (:158-262), and the same functional entry points `Coatadamw` /
`_single_tensor_Coatadamw` (:345-515).  What differs is below the API: instead of one
launch per tensor of a 1-element-per-thread kernel, all tensors of a parameter group
that share a step count go to ONE persistent launch that walks a device-side table of
tensors (`multi_tensor=True`, the default; the per-tensor loop remains available).
"""
from collections import defaultdict
from copy import deepcopy
from itertools import chain
from typing import List, Optional, Tuple, Union

import numpy as np
import torch
from torch import Tensor
from torch.optim.optimizer import Optimizer

from .. import _lib
from ..utils._fp8_quantization_config import QuantizationConfig
from . import qoptim_cuda

convert_str_to_fp8 = {"E4M3": torch.float8_e4m3fn, "E5M2": torch.float8_e5m2}

_STATE_DTYPES = (torch.float8_e4m3fn, torch.float8_e5m2, torch.float32)

_TABLE_DTYPE = np.dtype([(n, np.uint64) for n in
                         ("p", "g", "m", "v", "s_m", "k_m", "r_m", "s_v", "k_v", "r_v", "bf16_out")]
                        + [("numel", np.int64)])


def _dtensor_type():
    try:
        from torch.distributed.tensor import DTensor
    except Exception:   # a torch without the distributed tensor package
        return None
    return DTensor


def local_tensor(t):
    """The tensor the kernels see: a DTensor's local shard (FSDP2 / `fully_shard` parameters, their gradients and the
    optimizer state kept as DTensors), anything else as it is."""
    DTensor = _dtensor_type()
    if DTensor is not None and isinstance(t, DTensor):
        return t._local_tensor
    return t


def _group_state_layout(p, group_size):
    """For a DTensor parameter: (global shape, placements) under which a per-group vector of the LOCAL shard is itself a
    shard of one global tensor, or None when the groups of the local shards do not line up with the groups of the
    flattened full tensor.  They line up when the parameter is sharded along dimension 0 only (what `fully_shard` does)
    and every row holds a whole number of groups: then rank r's groups are rows of the [rows, row_numel / group_size]
    matrix of group values, sharded along dimension 0 exactly like the parameter, and a checkpoint of the sharded state
    is a checkpoint of the unsharded state cut along rows, whatever the world size.  One-dimensional parameters qualify
    when every rank's chunk (ceil(n / world) elements, the last one shorter) is a multiple of the group size."""
    from torch.distributed.tensor import Replicate, Shard
    placements = tuple(p.placements)
    sharded = [pl for pl in placements if not isinstance(pl, Replicate)]
    if not sharded:   # replicated everywhere: the local tensor is the full tensor
        return (-(-p.numel() // group_size),), placements
    if len(sharded) != 1 or not isinstance(sharded[0], Shard) or sharded[0].dim != 0 or p.dim() == 0:
        return None
    row = p.numel() // p.shape[0] if p.shape[0] else 0
    if p.dim() >= 2 and row % group_size == 0 and row > 0:
        return (p.shape[0], row // group_size), placements
    if p.dim() == 1:
        world = 1
        for pl, size in zip(placements, p.device_mesh.shape):
            if isinstance(pl, Shard):
                world = size
        chunk = -(-p.shape[0] // world)
        if chunk % group_size == 0:
            return (-(-p.shape[0] // group_size),), placements
    return None


class CoatAdamW(Optimizer):
    def __init__(
        self,
        params,
        lr: float = 1e-3,
        betas: Tuple[float, float] = (0.9, 0.999),
        eps: float = 1e-8,
        weight_decay: float = 1e-2,
        amsgrad: bool = False,
        qargs: QuantizationConfig = None,
        *,
        fused: Optional[bool] = None,
        multi_tensor: bool = True,
    ):
        if qargs is None:
            qargs = QuantizationConfig()
        self.qargs = qargs
        assert self.qargs.first_order_expansion == self.qargs.second_order_expansion, (
            "We expect the first order and second order momentum to use dynamic range expansion at the same time."
        )
        if not 0.0 <= lr:
            raise ValueError(f"Invalid learning rate: {lr}")
        if not 0.0 <= eps:
            raise ValueError(f"Invalid epsilon value: {eps}")
        if not 0.0 <= betas[0] < 1.0:
            raise ValueError(f"Invalid beta parameter at index 0: {betas[0]}")
        if not 0.0 <= betas[1] < 1.0:
            raise ValueError(f"Invalid beta parameter at index 1: {betas[1]}")
        if not 0.0 <= weight_decay:
            raise ValueError(f"Invalid weight_decay value: {weight_decay}")
        defaults = dict(lr=lr, betas=betas, eps=eps, weight_decay=weight_decay, amsgrad=amsgrad, fused=fused)
        super().__init__(params, defaults)
        self.multi_tensor = multi_tensor
        self._tables = {}
        self._bf16_copies = {}

    def attach_bf16_weights(self, pairs):
        """Mixed-precision training: `pairs` = iterable of (fp32 parameter of this optimizer, bf16 tensor of the
        same number of elements).  From now on each step also writes the updated weights, rounded to bf16, into
        the bf16 tensor, inside the same kernel (no separate cast pass).  An extension: the reference leaves the
        cast to the surrounding framework."""
        for master, copy in pairs:
            master = local_tensor(master)   # a DTensor parameter: the copy mirrors this rank's shard
            if copy.dtype != torch.bfloat16 or copy.numel() != master.numel() or not copy.is_contiguous() \
                    or copy.device != master.device:
                raise ValueError("a bf16 copy must be a contiguous bfloat16 tensor of the parameter's size and device")
            self._bf16_copies[id(master)] = copy
        self._tables = {}

    # ---- (de)serialisation -------------------------------------------------------------
    def __setstate__(self, state):
        super().__setstate__(state)
        self.__dict__.setdefault("multi_tensor", True)
        self.__dict__["_tables"] = {}
        self.__dict__.setdefault("_bf16_copies", {})
        for group in self.param_groups:
            group.setdefault("amsgrad", False)
            group.setdefault("fused", None)
            for p in group["params"]:
                p_state = self.state.get(p, [])
                if len(p_state) != 0 and not torch.is_tensor(p_state["step"]):
                    p_state["step"] = torch.tensor(float(p_state["step"]), dtype=torch.float32)

    @torch._disable_dynamo
    def load_state_dict(self, state_dict) -> None:
        """Like Optimizer.load_state_dict, except that state tensors are moved to the
        parameter's device WITHOUT a dtype cast (the stock implementation would cast the
        FP8 codes to the parameter dtype); coat/optimizer/fp8_adamw.py:158-262."""
        state_dict = state_dict.copy()
        for pre_hook in self._optimizer_load_state_dict_pre_hooks.values():
            hook_result = pre_hook(self, state_dict)
            if hook_result is not None:
                state_dict = hook_result

        groups = self.param_groups
        saved_groups = deepcopy(state_dict["param_groups"])
        if len(groups) != len(saved_groups):
            raise ValueError("loaded state dict has a different number of parameter groups")
        if any(len(g["params"]) != len(s["params"]) for g, s in zip(groups, saved_groups)):
            raise ValueError("loaded state dict contains a parameter group that doesn't match the size of "
                             "optimizer's group")
        id_map = dict(zip(chain.from_iterable(g["params"] for g in saved_groups),
                          chain.from_iterable(g["params"] for g in groups)))

        def move(param, value, key=None):
            if isinstance(value, torch.Tensor):
                return self._process_value_according_to_param_policy(
                    param, value, None, state_dict["param_groups"], key)
            if isinstance(value, dict):
                return {k: move(param, v, k) for k, v in value.items()}
            if isinstance(value, (list, tuple)):
                return type(value)(move(param, v) for v in value)
            return value

        state = defaultdict(dict)
        for k, v in state_dict["state"].items():
            if k in id_map:
                state[id_map[k]] = move(id_map[k], v)
            else:
                state[k] = v

        def update_group(group, new_group):
            new_group["params"] = group["params"]
            return new_group

        param_groups = [update_group(g, ng) for g, ng in zip(groups, saved_groups)]
        self.__setstate__({"state": state, "param_groups": param_groups})
        for post_hook in self._optimizer_load_state_dict_post_hooks.values():
            post_hook(self)

    @staticmethod
    def _process_value_according_to_param_policy(param, value, param_id, param_groups, key=None):
        if key == "step":
            return value  # stays a CPU scalar tensor
        assert value.dtype in _STATE_DTYPES, f"unexpected optimizer state dtype {value.dtype}"
        return value.to(device=param.device)  # do not cast optimizer states

    # Flags handed to the kernels of the one-launch path (0: guarded fast arithmetic; _lib.ADAMW_EXACT_POW: the exact
    # routines everywhere, bit-identical weights too).  A non-zero value also sends single tensors through that path.
    kernel_flags = 0

    # ---- state ---------------------------------------------------------------------------
    def _use_expansion(self):
        # Only these two spellings switch the expansion on (coat/optimizer/fp8_adamw.py:293);
        # e.g. "expand" leaves it off.
        return self.qargs.first_order_expansion.lower() in ["expansion", "true"]

    def _init_state(self, p, use_expansion, amsgrad):
        state = self.state[p]
        if len(state) != 0:
            return state
        if p.dtype != torch.float32:
            # The reference allocates the per-group vectors with dtype=p.dtype but its kernel
            # reads them as float32, so fp32 master parameters are the only working case there.
            raise RuntimeError(
                f"CoatAdamW needs float32 (master) parameters, got {p.dtype}: the per-group scale / "
                "exponent vectors are float32 by contract")
        if amsgrad:
            raise RuntimeError("CoatAdamW does not support amsgrad")
        q = self.qargs
        state["step"] = torch.tensor(0.0)
        lp = local_tensor(p)
        if lp is not p:
            return self._init_sharded_state(state, p, lp, use_expansion)
        groups = (p.numel() + q.qgroup_size - 1) // q.qgroup_size
        vec = dict(device=p.device, dtype=p.dtype)
        state["exp_avg"] = torch.zeros_like(p, dtype=convert_str_to_fp8[q.first_order_bit],
                                            memory_format=torch.preserve_format)
        state["scale_exp_avg"] = torch.zeros(groups, **vec)
        if use_expansion:
            state["expand_exp_avg"] = torch.ones(groups, **vec)
            state["sqrt_minmax_exp_avg"] = torch.ones(groups, **vec)
        state["exp_avg_sq"] = torch.zeros_like(p, dtype=convert_str_to_fp8[q.second_order_bit],
                                               memory_format=torch.preserve_format)
        state["scale_exp_avg_sq"] = torch.zeros(groups, **vec)
        if use_expansion:
            state["expand_exp_avg_sq"] = torch.ones(groups, **vec)
            state["sqrt_minmax_exp_avg_sq"] = torch.ones(groups, **vec)
        return state

    def _init_sharded_state(self, state, p, lp, use_expansion):
        """State of a DTensor parameter (FSDP2): every rank quantises its local shard in groups of 128 counted from the
        start of the shard.  The moments are DTensors laid out like the parameter; the per-group vectors are DTensors
        too wherever the local groups are the groups of the full tensor (_group_state_layout), so that
        torch.distributed.checkpoint and get_optimizer_state_dict see one global state; otherwise they stay plain
        rank-local tensors (training works, the state of that parameter is then specific to the world size)."""
        from torch.distributed.tensor import DTensor
        q = self.qargs
        mesh, placements = p.device_mesh, tuple(p.placements)
        layout = _group_state_layout(p, q.qgroup_size)
        groups = (lp.numel() + q.qgroup_size - 1) // q.qgroup_size
        vec = dict(device=lp.device, dtype=lp.dtype)

        def like_param(dtype):
            local = torch.zeros_like(lp, dtype=dtype, memory_format=torch.contiguous_format)
            return DTensor.from_local(local, mesh, placements, run_check=False, shape=p.shape, stride=p.stride())

        def per_group(fill):
            local = torch.full((groups,), fill, **vec)
            if layout is None:
                return local
            shape, pls = layout
            local = local.view((-1,) + tuple(shape[1:]))
            stride = tuple(torch.empty(shape, device="meta").stride())
            return DTensor.from_local(local, mesh, pls, run_check=False, shape=torch.Size(shape), stride=stride)

        state["exp_avg"] = like_param(convert_str_to_fp8[q.first_order_bit])
        state["scale_exp_avg"] = per_group(0.0)
        if use_expansion:
            state["expand_exp_avg"] = per_group(1.0)
            state["sqrt_minmax_exp_avg"] = per_group(1.0)
        state["exp_avg_sq"] = like_param(convert_str_to_fp8[q.second_order_bit])
        state["scale_exp_avg_sq"] = per_group(0.0)
        if use_expansion:
            state["expand_exp_avg_sq"] = per_group(1.0)
            state["sqrt_minmax_exp_avg_sq"] = per_group(1.0)
        return state

    # ---- step ------------------------------------------------------------------------------
    def _health_check(self):
        # torch renamed this hook; accept either name.
        for name in ("_cuda_graph_capture_health_check", "_accelerator_graph_capture_health_check"):
            fn = getattr(self, name, None)
            if fn is not None:
                fn()
                return

    @torch.no_grad()
    def step(self, closure=None):
        """Perform a single optimization step."""
        self._health_check()
        loss = None
        if closure is not None:
            with torch.enable_grad():
                loss = closure()

        use_expansion = self._use_expansion()
        for gi, group in enumerate(self.param_groups):
            # (a rank whose shard of an unevenly divided parameter is empty has nothing to step)
            params = [p for p in group["params"] if p.grad is not None and local_tensor(p).numel() > 0]
            if not params:
                continue
            for p in params:
                if p.grad.is_sparse:
                    raise RuntimeError("AdamW does not support sparse gradients")
            states = [self._init_state(p, use_expansion, group["amsgrad"]) for p in params]
            beta1, beta2 = group["betas"]
            hyper = dict(beta1=beta1, beta2=beta2, lr=group["lr"], weight_decay=group["weight_decay"],
                         eps=group["eps"], qgroup_size=self.qargs.qgroup_size, expand_min=self.qargs.expand_min)
            if (self.multi_tensor and len(params) > 1) or self.kernel_flags:
                self._multi_tensor_step(gi, params, states, use_expansion, **hyper)
            else:
                key = (lambda s, k: [local_tensor(st[k]) for st in s])
                exp = use_expansion
                Coatadamw(
                    self.qargs, [local_tensor(p) for p in params], [local_tensor(p.grad) for p in params],
                    key(states, "exp_avg"), key(states, "scale_exp_avg"),
                    key(states, "expand_exp_avg") if exp else [], key(states, "sqrt_minmax_exp_avg") if exp else [],
                    key(states, "exp_avg_sq"), key(states, "scale_exp_avg_sq"),
                    key(states, "expand_exp_avg_sq") if exp else [], key(states, "sqrt_minmax_exp_avg_sq") if exp else [],
                    [], key(states, "step"), amsgrad=group["amsgrad"], use_expansion=exp, **hyper,
                    fused=group["fused"], grad_scale=getattr(self, "grad_scale", None),
                    found_inf=getattr(self, "found_inf", None))
                for p in params:   # the per-tensor entry points keep the reference's signature: cast afterwards
                    copy = self._bf16_copies.get(id(local_tensor(p)))
                    if copy is not None:
                        copy.view(-1).copy_(local_tensor(p).detach().view(-1))
        return loss

    def _multi_tensor_step(self, gi, params, states, use_expansion, *, beta1, beta2, lr, weight_decay, eps,
                           qgroup_size, expand_min):
        """One persistent launch per (device, step value) bucket of this parameter group."""
        if qgroup_size != 128:
            raise RuntimeError("Only Support 128 per-group quantization currently")
        buckets = defaultdict(list)
        grads = [local_tensor(p.grad) for p in params]
        params = [local_tensor(p) for p in params]   # DTensor parameters: the kernels step the local shards
        states = [{k: local_tensor(v) for k, v in st.items()} for st in states]
        for i, (p, st) in enumerate(zip(params, states)):
            st["step"] += 1
            buckets[(p.device, int(st["step"].item()))].append(i)
        for (device, step), idxs in buckets.items():
            key = (gi, device, tuple(id(params[i]) for i in idxs), use_expansion)
            entry = self._tables.get(key)
            if entry is None:
                host = np.zeros(len(idxs), dtype=_TABLE_DTYPE)
                prefix = np.zeros(len(idxs) + 1, dtype=np.int64)
                for row, i in enumerate(idxs):
                    p, st = params[i], states[i]
                    for t in (st["scale_exp_avg"], st["scale_exp_avg_sq"]):
                        if t.dtype != torch.float32:
                            raise RuntimeError(f"expected scalar type Float but found {t.dtype}")
                    r = host[row]
                    r["p"] = _lib.dev_ptr(p, "param")
                    r["m"] = _lib.dev_ptr(st["exp_avg"])
                    r["v"] = _lib.dev_ptr(st["exp_avg_sq"])
                    r["s_m"] = _lib.dev_ptr(st["scale_exp_avg"])
                    r["s_v"] = _lib.dev_ptr(st["scale_exp_avg_sq"])
                    if use_expansion:
                        r["k_m"] = _lib.dev_ptr(st["expand_exp_avg"])
                        r["r_m"] = _lib.dev_ptr(st["sqrt_minmax_exp_avg"])
                        r["k_v"] = _lib.dev_ptr(st["expand_exp_avg_sq"])
                        r["r_v"] = _lib.dev_ptr(st["sqrt_minmax_exp_avg_sq"])
                    copy = self._bf16_copies.get(id(p))
                    if copy is not None:
                        r["bf16_out"] = _lib.dev_ptr(copy)
                    r["numel"] = p.numel()
                    prefix[row + 1] = prefix[row] + (p.numel() + 127) // 128
                pinned = torch.from_numpy(host.view(np.uint8).reshape(-1)).pin_memory()
                entry = dict(host=pinned, rows=pinned.numpy().view(_TABLE_DTYPE),
                             dev=torch.empty(pinned.numel(), dtype=torch.uint8, device=device),
                             prefix=torch.from_numpy(prefix).to(device), total=int(prefix[-1]))
                self._tables[key] = entry
            rows = entry["rows"]
            changed = []
            for row, i in enumerate(idxs):
                g = grads[i]
                if g.dtype != params[i].dtype or not g.is_contiguous():
                    raise RuntimeError("gradients must be contiguous and match the parameter dtype")
                gp, pp = g.data_ptr(), params[i].data_ptr()
                if rows[row]["g"] != gp or rows[row]["p"] != pp:
                    changed.append((row, gp, pp))
            if changed:
                # The pinned table is the source of an asynchronous copy: it may be rewritten only once the copy
                # queued by an earlier step has read it (the host can run a step ahead of the GPU, and with
                # zero_grad(set_to_none=True) gradients come back at new addresses).  Unchanged pointers need no copy.
                if entry.get("copied") is not None:
                    entry["copied"].synchronize()
                for row, gp, pp in changed:
                    rows[row]["g"] = gp
                    rows[row]["p"] = pp
                with torch.cuda.device(device):
                    entry["dev"].copy_(entry["host"], non_blocking=True)
                    entry["copied"] = torch.cuda.Event()
                    entry["copied"].record(torch.cuda.current_stream(device))
            with torch.cuda.device(device):
                rc = _lib.lib().coat_fp8_adamw_multi_step(
                    entry["dev"].data_ptr(), entry["prefix"].data_ptr(), len(idxs), entry["total"],
                    int(use_expansion), beta1, beta2, lr, weight_decay, eps, step, qgroup_size, expand_min,
                    _lib.F32, int(self.kernel_flags), _lib.stream_ptr(device))
            _lib.check(rc, "fp8_adamw_multi_step")


def Coatadamw(
    qargs,
    params: List[Tensor],
    grads: List[Tensor],
    exp_avgs: List[Tensor],
    scale_exp_avgs: List[Tensor],
    expand_exp_avgs: List[Tensor],
    sqrt_minmax_exp_avgs: List[Tensor],
    exp_avg_sqs: List[Tensor],
    scale_exp_avg_sqs: List[Tensor],
    expand_exp_avg_sqs: List[Tensor],
    sqrt_minmax_exp_avg_sqs: List[Tensor],
    max_exp_avg_sqs: List[Tensor],
    state_steps: List[Tensor],
    fused: Optional[bool] = None,
    grad_scale: Optional[Tensor] = None,
    found_inf: Optional[Tensor] = None,
    *,
    amsgrad: bool,
    use_expansion: bool,
    beta1: float,
    beta2: float,
    lr: Union[float, Tensor],
    weight_decay: float,
    eps: float,
    qgroup_size: int,
    expand_min: int,
):
    """Functional form (coat/optimizer/fp8_adamw.py:345-409): one kernel launch per tensor."""
    if not all(isinstance(t, torch.Tensor) for t in state_steps):
        raise RuntimeError("API has changed, `state_steps` argument must contain a list of singleton tensors")
    _single_tensor_Coatadamw(
        qargs, params, grads, exp_avgs, scale_exp_avgs, expand_exp_avgs, sqrt_minmax_exp_avgs, exp_avg_sqs,
        scale_exp_avg_sqs, expand_exp_avg_sqs, sqrt_minmax_exp_avg_sqs, max_exp_avg_sqs, state_steps,
        grad_scale, found_inf, amsgrad=amsgrad, use_expansion=use_expansion, beta1=beta1, beta2=beta2, lr=lr,
        weight_decay=weight_decay, eps=eps, qgroup_size=qgroup_size, expand_min=expand_min)


def _single_tensor_Coatadamw(
    qargs, params, grads, exp_avgs, scale_exp_avgs, expand_exp_avgs, sqrt_minmax_exp_avgs, exp_avg_sqs,
    scale_exp_avg_sqs, expand_exp_avg_sqs, sqrt_minmax_exp_avg_sqs, max_exp_avg_sqs, state_steps,
    grad_scale, found_inf, *, amsgrad, use_expansion, beta1, beta2, lr, weight_decay, eps, qgroup_size,
    expand_min,
):
    """coat/optimizer/fp8_adamw.py:419-515."""
    assert grad_scale is None and found_inf is None
    for i, param in enumerate(params):
        step_t = state_steps[i]
        step_t += 1
        step = int(step_t.item())
        if use_expansion:
            qoptim_cuda.fp8_adamw_expand_step(
                param, grads[i], exp_avgs[i], scale_exp_avgs[i], expand_exp_avgs[i], sqrt_minmax_exp_avgs[i],
                exp_avg_sqs[i], scale_exp_avg_sqs[i], expand_exp_avg_sqs[i], sqrt_minmax_exp_avg_sqs[i],
                beta1, beta2, float(lr), weight_decay, eps, step, qgroup_size, expand_min)
        else:
            qoptim_cuda.fp8_adamw_step(
                param, grads[i], exp_avgs[i], scale_exp_avgs[i], exp_avg_sqs[i], scale_exp_avg_sqs[i],
                beta1, beta2, float(lr), weight_decay, eps, step, qgroup_size)
