"""Generate golden vectors for the FP8 AdamW (expansion) step from the reference itself.

Run where the reference checkout is readable:
    python tests/golden/make_adamw_golden.py [/path/to/reference]

The reference's own test, tests/test_fp8_adamw_expand.py, builds its inputs and its
pure-PyTorch expectation (`simulated_optimizer_expand_step`, :111-215) at module level on
a GPU.  This script executes that file's TEXT on the CPU, with three textual patches and
nothing else changed:
  * `import qoptim_cuda` is dropped (the native module is what is under test),
  * `device="cuda"` becomes `device="cpu"`,
  * the Triton fake-quantizer is replaced by the reference's torch implementation of the
    same function (the swap the reference leaves as a comment at
    coat/activation/fake_quantization/quantize_function.py:250-251).
Per case it may also patch the seed, the shape and make the random sqrt-min-max inputs
positive.  It stores the kernel inputs the test would hand to
qoptim_cuda.fp8_adamw_expand_step and the nine tensors the test compares with
allclose(rtol=1e-4) (:296-308) in adamw_expand_golden.npz.
"""
import os
import sys

import numpy as np
import torch

CASES = [
    # name, seed, (M, N), make sqrt-min-max inputs positive
    ("ref_seed0_2x128", 0, (2, 128), False),
    ("seed1_2x128_pos", 1, (2, 128), True),
    ("seed2_8x128_pos", 2, (8, 128), True),
    ("seed3_64x128_pos", 3, (64, 128), True),
]


def run_case(ref_root, seed, shape, positive):
    src = open(os.path.join(ref_root, "tests", "test_fp8_adamw_expand.py")).read()
    src = src.replace("import qoptim_cuda\n", "")
    src = src.replace('device="cuda"', 'device="cpu"')
    src = src.replace("torch.manual_seed(0)\ntorch.set_printoptions(sci_mode=False)",
                      f"torch.manual_seed({seed})\ntorch.set_printoptions(sci_mode=False)")
    src = src.replace("M, N = 2, 128", f"M, N = {shape[0]}, {shape[1]}")
    if positive:
        src = src.replace("SQRTexp_avg = torch.randn_like(Sexp_avg).squeeze(2)",
                          "SQRTexp_avg = torch.randn_like(Sexp_avg).squeeze(2).abs() + 0.05")
        src = src.replace("SQRTexp_avg_sq = torch.randn_like(Sexp_avg_sq).squeeze(2)",
                          "SQRTexp_avg_sq = torch.randn_like(Sexp_avg_sq).squeeze(2).abs() + 0.05")
    # stop before the unittest class: only inputs + simulated step are wanted
    src = src.split("class TestExpandAdamW")[0]

    import coat.activation.fake_quantization.quantize_function as qf
    from coat.activation.fake_quantization.FloatPointQuantizeTorch import floatExMy_quantize_torch
    qf.floatExMy_quantize_triton = floatExMy_quantize_torch

    ns = {"__name__": "reference_test_text"}
    exec(compile(src, "test_fp8_adamw_expand.py", "exec"), ns)

    inputs = dict(
        params=ns["params_cuda"].clone(), grads=ns["grads_cuda"].clone(),
        exp_avg=ns["Qexp_avg"].clone().view(torch.uint8), scale_exp_avg=ns["Sexp_avg"].clone().flatten(),
        expand_exp_avg=ns["EXPexp_avg"].clone().flatten(), sqrtminmax_exp_avg=ns["SQRTexp_avg"].clone().flatten(),
        exp_avg_sq=ns["Qexp_avg_sq"].clone().view(torch.uint8),
        scale_exp_avg_sq=ns["Sexp_avg_sq"].clone().flatten(),
        expand_exp_avg_sq=ns["EXPexp_avg_sq"].clone().flatten(),
        sqrtminmax_exp_avg_sq=ns["SQRTexp_avg_sq"].clone().flatten(),
    )
    hyper = dict(beta1=ns["beta1"], beta2=ns["beta2"], lr=ns["lr"], wd=ns["wd"], eps=ns["eps"],
                 step=ns["step"], qgroup_size=ns["qgroup_size"], expand_min=16)
    out = ns["simulated_optimizer_expand_step"](
        ns["params_py"], ns["grads_py"], ns["fp_exp_avg"], ns["fp_exp_avg_sq"], ns["beta1"], ns["beta2"],
        ns["lr"], ns["wd"], ns["eps"], ns["step"], ns["qgroup_size"])
    names = ["Qexp_avg_py", "Sexp_avg_py", "B1Exp", "block_sqrt_minmax1", "Qexp_avg_sq_py", "Sexp_avg_sq_py",
             "B2Exp", "block_sqrt_minmax2"]
    expected = {n: t.detach().float().flatten() for n, t in zip(names, out)}
    expected["params_py"] = ns["params_py"].flatten()
    return inputs, hyper, expected


def main():
    ref_root = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("COAT_REFERENCE_ROOT")
    if not ref_root:
        raise SystemExit("usage: python " + sys.argv[0] + " /path/to/reference   (or COAT_REFERENCE_ROOT)")
    sys.path.insert(0, ref_root)
    blob = {}
    for name, seed, shape, positive in CASES:
        inputs, hyper, expected = run_case(ref_root, seed, shape, positive)
        for k, v in inputs.items():
            blob[f"{name}/in/{k}"] = v.numpy()
        for k, v in hyper.items():
            blob[f"{name}/hyper/{k}"] = np.float64(v)
        for k, v in expected.items():
            blob[f"{name}/out/{k}"] = v.numpy()
        nan = sum(int(torch.isnan(v).sum()) for v in expected.values())
        print(name, "NaNs in expectation:", nan)
    out = os.path.join(os.path.dirname(os.path.abspath(__file__)), "adamw_expand_golden.npz")
    np.savez_compressed(out, **blob)
    print("wrote", out, os.path.getsize(out), "bytes")


if __name__ == "__main__":
    main()
