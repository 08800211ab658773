"""coat_b200: B200-native (sm_100a) implementation of COAT's quantization hot path.

Host code mirrors the reference's python API; the work is done by hand-written CUDA
kernels in coat_b200/libcoat_b200.so, reached through the C ABI in include/coat_b200.h.
"""
__version__ = "0.1"
