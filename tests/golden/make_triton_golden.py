"""Golden vectors for the quantizers, the fused operators and the FP8 GEMM from the reference's own Triton kernels.

    python tests/golden/make_triton_golden.py          (on a machine with a CUDA GPU)

Needs the reference's operator layer staged by `python oracle/build_ref.py` (oracle/_ref/coat_ref/).  Runs every
reference operator once on small seeded inputs (64 x 256, 0.5 % of the entries x100, group size 16; each autotuned
kernel with one of its own candidate configurations) and stores inputs and outputs in triton_golden.npz beside this
script.  FP8 tensors are stored as their bytes, bf16 tensors as fp32 values (exact).  The CPU test
tests/test_oracle_vs_reference_outputs.py holds the torch restatements under oracle/ to these outputs.
"""
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(HERE))
from _ref import load_ref_triton, ref_module  # noqa: E402

M, N, QB = 64, 256, 16


def seeded(seed, scale=1.0, outliers=True, shape=(M, N)):
    gen = torch.Generator().manual_seed(seed)
    x = torch.randn(*shape, generator=gen)
    if outliers:
        x[torch.rand(*shape, generator=gen) < 5e-3] *= 100
    return (x * scale).to(torch.bfloat16).cuda()


def main():
    R = load_ref_triton()
    if R is None:
        raise SystemExit("oracle/_ref/coat_ref is not staged: run python oracle/build_ref.py where the reference is")
    blob = {}

    def put(name, t):
        t = t.detach().cpu().contiguous()
        if t.dtype in (torch.float8_e4m3fn, torch.float8_e5m2):
            blob[name] = t.view(torch.uint8).numpy()
        else:
            blob[name] = t.float().numpy()

    x = seeded(1)
    g = seeded(2, 1e-2, outliers=False)
    put("x", x)
    put("g", g)
    for fmt in ("E4M3", "E5M2"):
        y, s = R.fp8_quantize(x, QB, fmt)
        put(f"quantize/{fmt}/y", y), put(f"quantize/{fmt}/s", s)
        y, s = R.fp8_quantize(x, QB, fmt, torch.float32)
        put(f"quantize_f32/{fmt}/y", y), put(f"quantize_f32/{fmt}/s", s)
        y, s_max, s = R.fp8_quantize_pertensor(x, QB, fmt)
        put(f"pertensor/{fmt}/y", y), put(f"pertensor/{fmt}/s_max", s_max), put(f"pertensor/{fmt}/s", s)
        y, s_max, y_t = R.fp8_quantize_pertensor_transpose(x, QB, fmt)
        put(f"pertensor_t/{fmt}/y", y), put(f"pertensor_t/{fmt}/s_max", s_max), put(f"pertensor_t/{fmt}/y_t", y_t)
        (y, s), (y_t, s_t) = ref_module("_quantize_transpose").fp8_quantize_transpose(x, QB, fmt)
        put(f"quantize_t/{fmt}/y", y), put(f"quantize_t/{fmt}/s", s)
        put(f"quantize_t/{fmt}/y_t", y_t), put(f"quantize_t/{fmt}/s_t", s_t)
        given = torch.tensor(0.0371, dtype=torch.bfloat16, device="cuda")
        y, _ = R.fp8_division(x, QB, fmt, given)
        put(f"division/{fmt}/y", y), put(f"division/{fmt}/s", given)
    q, s = R.fp8_quantize(seeded(3, 2.0), QB, "E4M3")
    q2, s2 = R.fp8_quantize(seeded(4, 3.0), QB, "E4M3")
    put("in/q", q), put("in/s", s), put("in/q2", q2), put("in/s2", s2)
    put("dequantize/y", R.fp8_dequantize(q, s, QB))
    y, s_y = R.fp8_silu_forward(q, s, QB)
    put("silu_fwd/y", y), put("silu_fwd/s", s_y)
    y, s_y = R.fp8_silu_backward(q, s, g, QB, "E5M2")
    put("silu_bwd/y", y), put("silu_bwd/s", s_y)
    qy, s_max, qy_t = R.fp8_silu_backward(q, s, g, QB, "E5M2", output_quantized_transpose=True)
    put("silu_bwd/q", qy), put("silu_bwd/s_max", s_max)
    qy, s_max, _ = R.fp8_gelu_forward(q, s, QB)
    put("gelu_fwd/q", qy), put("gelu_fwd/s_max", s_max)
    qy, s_max = R.fp8_gelu_backward(q, s, g, QB, "E5M2")
    put("gelu_bwd/q", qy), put("gelu_bwd/s_max", s_max)
    qy, s_max, qy_t = R.fp8_mul_forward(q, s, q2, s2, QB)
    put("mul_fwd/q", qy), put("mul_fwd/s_max", s_max), put("mul_fwd/q_t", qy_t)
    y1, (y2, s_y2) = R.fp8_mul_backward(q, s, q2, s2, g, QB, "E5M2")
    put("mul_bwd/y1", y1), put("mul_bwd/y2", y2), put("mul_bwd/s", s_y2)
    a, b = seeded(5), seeded(6, 0.5)
    put("add/a", a), put("add/b", b)
    y1, (y2, s_y2) = R.fp8_add_Ifp_Ifp_Ofp_Og16(a, b, torch.float8_e4m3fn, QB)
    put("add_fwd/y1", y1), put("add_fwd/y2", y2), put("add_fwd/s", s_y2)
    y1, (qy, s_max, s_g) = R.fp8_add_Ifp_Ifp_Ofp_Opt(a, b, QB, "E5M2")
    put("add_bwd/y1", y1), put("add_bwd/q", qy), put("add_bwd/s_max", s_max), put("add_bwd/s", s_g)
    w = (1 + 0.1 * torch.randn(N, generator=torch.Generator().manual_seed(7))).to(torch.bfloat16).cuda()
    bias = (0.1 * torch.randn(N, generator=torch.Generator().manual_seed(8))).to(torch.bfloat16).cuda()
    put("norm/w", w), put("norm/b", bias)
    qy, s_max, _, (_, rstd, _) = R.fp8_rmsnorm_forward(q, s, w, QB, 1e-5)
    put("rmsnorm_fwd/q", qy), put("rmsnorm_fwd/s_max", s_max), put("rmsnorm_fwd/rstd", rstd)
    qy, s_max, _, (mean, rstd, nw) = R.fp8_layernorm_noparam_forward(q, s, QB, 1e-5)
    put("ln_noparam_fwd/q", qy), put("ln_noparam_fwd/s_max", s_max)
    put("ln_noparam_fwd/mean", mean), put("ln_noparam_fwd/rstd", rstd)
    put("ln_noparam_bwd/dx", R.fp8_layernorm_noparam_backward(q, s, g, QB, mean, rstd, nw))
    qy, s_max, _, (_, _, mean, rstd, _) = R.fp8_layernorm_param_forward(q, s, w, bias, QB, 1e-5)
    put("ln_param_fwd/q", qy), put("ln_param_fwd/s_max", s_max)
    put("ln_param_fwd/mean", mean), put("ln_param_fwd/rstd", rstd)
    # FP8 GEMM: 64 x 256 activations times a 128 x 256 weight, and the backward pair with an E5M2 gradient
    wt = seeded(9, 0.02, outliers=False, shape=(128, N))
    gy = seeded(10, 1e-2, outliers=False, shape=(M, 128))
    qx, sx, qx_t = R.fp8_quantize_pertensor_transpose(x, QB, "E4M3")
    qw, sw, qw_t = R.fp8_quantize_pertensor_transpose(wt, QB, "E4M3")
    qg, sg, qg_t = R.fp8_quantize_pertensor_transpose(gy, QB, "E5M2")
    for name, t in (("qx", qx), ("sx", sx), ("qx_t", qx_t), ("qw", qw), ("sw", sw), ("qw_t", qw_t), ("qg", qg),
                    ("sg", sg), ("qg_t", qg_t)):
        put(f"gemm/{name}", t)
    put("gemm/y", R.fp8_linear_forward(qx, sx, qw, sw, False, QB))
    dx, dw = R.fp8_linear_backward(qx_t, sx, qg, sg, qg_t, qw_t, sw, QB)
    put("gemm/dx", dx), put("gemm/dw", dw)
    out = os.path.join(HERE, "triton_golden.npz")
    np.savez_compressed(out, **blob)
    print(f"{len(blob)} arrays -> {out} ({os.path.getsize(out)} bytes)")


if __name__ == "__main__":
    main()
