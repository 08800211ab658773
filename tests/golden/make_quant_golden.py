"""Golden vectors for the quantizers from the reference's own pure-PyTorch expectation.

    python tests/golden/make_quant_golden.py [/path/to/reference]

Executes the TEXT of the reference's tests/test_utils.py on the CPU (it is plain torch; the only
patch is dropping `.cuda()` from its random-tensor helper, which is not used here) and stores, for
seeded inputs, what its `quantize_tensor` (:45-70) returns for per-group and per-tensor
quantization: the expectation the reference's tests compare its kernels with at ">= 95 % of the
dequantised elements exactly equal" (check_similarity, :98-119).
"""
import os
import sys

import numpy as np
import torch


def main():
    ref_root = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("COAT_REFERENCE_ROOT")
    if not ref_root:
        raise SystemExit("usage: python " + sys.argv[0] + " /path/to/reference   (or COAT_REFERENCE_ROOT)")
    sys.path.insert(0, ref_root)
    src = open(os.path.join(ref_root, "tests", "test_utils.py")).read().replace(".cuda()", "")
    ns = {"__name__": "reference_test_utils"}
    exec(compile(src, "test_utils.py", "exec"), ns)
    blob = {}
    BS, SL, CDIM, QB = 2, 32, 128, 16
    for seed in (0, 1):
        gen = torch.Generator().manual_seed(seed)
        x = torch.randn(BS, SL, CDIM, generator=gen)
        if seed == 1:  # outliers, as in the activation benchmark configuration
            x = torch.where(torch.rand(BS, SL, CDIM, generator=gen) < 1e-2, x * 100, x)
        x = x.to(torch.bfloat16).float()
        blob[f"s{seed}/x"] = x.numpy()
        for name, fp8 in (("E4M3", torch.float8_e4m3fn), ("E5M2", torch.float8_e5m2)):
            for kind in ("per_group", "per_tensor"):
                rqx, qx, sx = ns["quantize_tensor"](x, BS, SL, CDIM, QB, fp8, quant_type=kind)
                blob[f"s{seed}/{name}/{kind}/rqx"] = rqx.float().numpy()
                blob[f"s{seed}/{name}/{kind}/qx"] = qx.view(torch.uint8).numpy()
                blob[f"s{seed}/{name}/{kind}/sx"] = sx.float().numpy()
    out = os.path.join(os.path.dirname(os.path.abspath(__file__)), "quant_golden.npz")
    np.savez_compressed(out, **blob)
    print("wrote", out, os.path.getsize(out), "bytes")


if __name__ == "__main__":
    main()
