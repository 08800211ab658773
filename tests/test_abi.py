"""The C-ABI library loads and exports every function include/coat_b200.h declares (no compute
calls: this runs without a GPU), and the ctypes table of the python side covers the same set."""
import ctypes
import os
import re

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_functions():
    text = open(os.path.join(ROOT, "include", "coat_b200.h")).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(coat_[a-z0-9_]+)\s*\(", text)))


def test_header_declares_the_expected_surface():
    names = declared_functions()
    for must in ("coat_fp8_adamw_expand_step", "coat_fp8_adamw_step", "coat_fp8_adamw_multi_step",
                 "coat_fp8_quantize", "coat_fp8_group_scales_amax", "coat_fp8_division",
                 "coat_fp8_quantize_transpose", "coat_fp8_transpose", "coat_fp8_dequantize",
                 "coat_fp8_quantize_pertensor_static"):
        assert must in names


def test_library_exports_every_declared_symbol():
    from coat_b200.csrc import build
    lib_path = build.build()   # no-op when up to date; nvcc cross-compiles without a GPU
    lib = ctypes.CDLL(lib_path)
    missing = [n for n in declared_functions() if not hasattr(lib, n)]
    assert not missing, f"declared in include/coat_b200.h but not exported: {missing}"
    lib.coat_b200_version.restype = ctypes.c_char_p
    assert b"sm_100a" in lib.coat_b200_version()
    lib.coat_strerror.restype = ctypes.c_char_p
    lib.coat_strerror.argtypes = [ctypes.c_int]
    assert b"128" in lib.coat_strerror(-2)


def test_ctypes_table_matches_header():
    from coat_b200 import _lib
    declared = set(declared_functions()) - {"coat_b200_version", "coat_strerror"}
    assert declared == set(_lib.SIGNATURES), declared ^ set(_lib.SIGNATURES)
    _lib.lib()


def test_no_cpu_fallback():
    import pytest
    import torch
    from coat_b200.optimizer import qoptim_cuda
    p = torch.zeros(128)
    z = torch.zeros(1)
    with pytest.raises(RuntimeError, match="CUDA"):
        qoptim_cuda.fp8_adamw_expand_step(p, p, p.to(torch.uint8), z, z, z, p.to(torch.uint8), z, z, z,
                                          0.9, 0.95, 1e-4, 0.1, 1e-8, 1, 128, 16)
    import coat_b200.activation.real_quantization as r
    with pytest.raises(RuntimeError, match="CUDA"):
        r.fp8_quantize(torch.zeros(16, 16, dtype=torch.bfloat16), 16, "E4M3")
