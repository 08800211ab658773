"""Access to the staged reference (TEST / BASELINE INFRASTRUCTURE ONLY): the reference's compiled optimizer extension
and its Triton operator layer, as oracle/build_ref.py put them into oracle/_ref/.  Used by the tests (as the
checker) and by bench.py's "reference on this GPU" baseline figures; never by the product package."""
import importlib
import os
import sys

REF_DIR = os.path.join(os.path.dirname(os.path.abspath(__file__)), "_ref")
_PKG = "coat_ref.activation.real_quantization"
_loaded = {}


def load_ref_qoptim():
    """The reference's `qoptim_cuda` module built into oracle/_ref, or None."""
    so = os.path.join(REF_DIR, "qoptim_cuda.so")
    if not os.path.exists(so):
        return None
    import torch  # noqa: F401  (the extension links against torch)
    if REF_DIR not in sys.path:
        sys.path.insert(0, REF_DIR)
    try:
        return importlib.import_module("qoptim_cuda")
    except Exception:
        return None


def _one_config(obj, seen):
    """Walk a Triton kernel wrapper chain (Heuristics -> Autotuner -> JITFunction) and keep ONE of the
    autotuner's own candidate configurations, so that nothing is benchmarked: every candidate computes
    the same values (the kernels reduce with max only, tile by tile), the choice only affects speed.
    The smallest tile of the list is kept (least register pressure, quickest to compile)."""
    from triton.runtime.autotuner import Autotuner
    while obj is not None and id(obj) not in seen:
        seen.add(id(obj))
        if isinstance(obj, Autotuner) and len(obj.configs) > 1:
            def area(c):
                kw = c.kwargs
                return kw.get("BLOCK_M", 1) * kw.get("BLOCK_N", 1), c.num_warps, c.num_stages
            obj.configs = [min(obj.configs, key=area)]
        obj = getattr(obj, "fn", None)


def load_ref_triton(one_config=True):
    """The reference's operator layer (its Triton kernels and python wrappers) as staged into
    oracle/_ref/coat_ref/, or None when it has not been staged.  GPU only.  one_config=True (the parity tests)
    restricts every autotuned kernel to one of its own candidate configurations; one_config=False (timing) leaves
    the reference's autotuning as it is.  The first call in a process decides."""
    if "mod" in _loaded:
        return _loaded["mod"]
    pkg = os.path.join(REF_DIR, "coat_ref", "activation", "real_quantization")
    if not os.path.isdir(pkg):
        return None
    if REF_DIR not in sys.path:
        sys.path.insert(0, REF_DIR)
    mod = importlib.import_module(_PKG)
    if one_config:
        seen = set()
        for name in sorted(os.listdir(pkg)):
            if not name.endswith(".py") or name == "__init__.py":
                continue
            try:
                sub = importlib.import_module(f"{_PKG}.{name[:-3]}")
            except Exception:
                continue
            for val in list(vars(sub).values()):
                for k in (val.values() if isinstance(val, dict) else (val,)):
                    if hasattr(k, "fn"):
                        _one_config(k, seen)
    _loaded["mod"] = mod
    return mod


def ref_module(name, one_config=True):
    """A submodule of the staged reference package, e.g. ref_module('_quantize_transpose')."""
    if load_ref_triton(one_config) is None:
        return None
    return importlib.import_module(f"{_PKG}.{name}")


def load_ref_optimizer():
    """The reference's own `CoatAdamW` class and `QuantizationConfig` (coat/optimizer/fp8_adamw.py,
    coat/utils/_fp8_quantization_config.py, staged unmodified) on top of its compiled extension, or None.
    The reference's step() calls `Optimizer._cuda_graph_capture_health_check`, which current torch spells
    `_accelerator_graph_capture_health_check`: the missing name is added to torch's Optimizer class as an alias on
    this (oracle) side, the reference file is not touched."""
    if "opt" in _loaded:
        return _loaded["opt"]
    if load_ref_qoptim() is None or not os.path.exists(os.path.join(REF_DIR, "coat_ref", "optimizer", "fp8_adamw.py")):
        return None
    from torch.optim.optimizer import Optimizer
    if not hasattr(Optimizer, "_cuda_graph_capture_health_check"):
        alias = getattr(Optimizer, "_accelerator_graph_capture_health_check", None)
        Optimizer._cuda_graph_capture_health_check = alias if alias is not None else (lambda self: None)
    try:
        mod = importlib.import_module("coat_ref.optimizer.fp8_adamw")
        cfg = importlib.import_module("coat_ref.utils._fp8_quantization_config")
    except Exception:
        return None
    _loaded["opt"] = (mod.CoatAdamW, cfg.QuantizationConfig)
    return _loaded["opt"]


def reference_layer_operators(ref, mine):
    """name -> callable with this repository's operator signatures, running the REFERENCE's kernels: what has to be
    exchanged in coat_b200.models.coat_llama / coat_olmo (and the weight cache, and func_quantize) to run the
    decoder-layer composition on the reference's operators.  Four calls have no reference counterpart and are replaced
    by the reference calls they stand for (fp8_silu_mul_forward, fp8_mul_silu_backward, fp8_mul_silu_backward_joint,
    the scale-only weight pass); ONE
    operator stays this repository's: the RMSNorm backward, because the reference's kernel waits on a device-side
    spin lock without a bound (func_rmsnorm.py:186-196) and is not run on shared GPUs."""
    def silu_mul_forward(gate_x, gate_s, up_x, up_s, QB, transpose_output_2d=False):
        silu_x, silu_s = ref.fp8_silu_forward(gate_x, gate_s, QB)
        return (silu_x, silu_s), ref.fp8_mul_forward(silu_x, silu_s, up_x, up_s, QB, transpose_output_2d)

    def mul_silu_backward(silu_x, silu_s, up_x, up_s, gate_x, gate_s, g, QB, fp8type):
        d_silu, up_grad = ref.fp8_mul_backward(silu_x, silu_s, up_x, up_s, g, QB, fp8type,
                                               output_quantized_transpose=True)
        gate_grad = ref.fp8_silu_backward(gate_x, gate_s, d_silu, QB, fp8type, output_quantized_transpose=True)
        return up_grad, gate_grad

    def mul_silu_backward_joint(silu_x, silu_s, up_x, up_s, gate_x, gate_s, g, QB, fp8type):
        import torch
        # the OLMo block's sequence (coat/models/coat_olmo.py:596-611)
        mul_g1, (mul_g2, mul_gs2) = ref.fp8_mul_backward(silu_x, silu_s, up_x, up_s, g, QB, fp8type)
        silu_g, silu_gs = ref.fp8_silu_backward(gate_x, gate_s, mul_g1, QB, fp8type)
        gateup_g = torch.cat([mul_g2, silu_g], dim=-1)
        gateup_gs = torch.max(torch.cat([mul_gs2, silu_gs]))
        return ref.fp8_division_transpose(gateup_g, QB, fp8type, gateup_gs, stochastic=False)

    def rmsnorm_backward(x, s_x, g, w, v, QB, num_warps, more_g=()):
        for t in more_g:   # bf16 sums, left to right, as the separate add kernels of the reference's autograd give
            g = g + t.reshape(g.shape)
        return mine.fp8_rmsnorm_backward(x, s_x, g, w, v, QB, num_warps)

    ops = {n: getattr(ref, n) for n in (
        "fp8_add_Ifp_Ifp_Ofp_Og16", "fp8_add_Ifp_Ifp_Ofp_Opt", "fp8_division", "fp8_division_transpose",
        "fp8_linear_backward", "fp8_linear_forward", "fp8_quantize_pertensor", "fp8_quantize_pertensor_transpose",
        "fp8_rmsnorm_forward", "fp8_transpose", "fp8_quantize", "fp8_layernorm_noparam_forward",
        "fp8_layernorm_noparam_backward")}
    ops.update(fp8_silu_mul_forward=silu_mul_forward, fp8_mul_silu_backward=mul_silu_backward,
               fp8_mul_silu_backward_joint=mul_silu_backward_joint,
               fp8_rmsnorm_backward=rmsnorm_backward,
               fp8_pertensor_scale=lambda w, fp8type: ref.fp8_division_transpose(w, 16, fp8type)[1])
    return ops


def load_ref_liger():
    """The reference's loss-head module (coat/activation/liger/cross_entropy.py, staged unmodified), or None."""
    if not os.path.exists(os.path.join(REF_DIR, "coat_ref", "activation", "liger", "cross_entropy.py")):
        return None
    if REF_DIR not in sys.path:
        sys.path.insert(0, REF_DIR)
    try:
        return importlib.import_module("coat_ref.activation.liger.cross_entropy")
    except Exception:
        return None
