"""CPU restatement of the reference's quantizer kernels in torch fp32 (TEST INFRASTRUCTURE ONLY).

Each function follows the arithmetic of one Triton kernel of coat/activation/real_quantization/:
    _quantize.py:74-92              scale = (max|x| + 1e-10) / fp8_max ; q = x / scale ; store scale rounded
    _quantize_pertensor.py:80-92    the same scale, stored only; then s_y.max() (:139) and _division.py:86-93
    _division.py:84-114             q = x / s with a scalar s
    _quantize_transpose.py:84-145   row groups and groups of the transposed tile
    _dequantize.py:87-97            code * scale -> bf16
with IEEE fp32 division in the place of the GPU's div.full.f32 (a CPU cannot reproduce the latter bit for
bit; the CUDA kernels offer IEEE division behind COAT_QUANT_IEEE_DIV for exactly this comparison), and the
saturating round-to-nearest-even cast written as clamp + torch's RNE cast.
"""
import torch

FP8_MAX = {torch.float8_e4m3fn: 448.0, torch.float8_e5m2: 57344.0}
FP8_DTYPE = {"E4M3": torch.float8_e4m3fn, "E5M2": torch.float8_e5m2}
SCALE_MIN_THRES = 1e-10


def _dt(fp8type):
    return FP8_DTYPE[fp8type] if isinstance(fp8type, str) else fp8type


def cast_fp8(x, fp8type):
    """float -> fp8, round to nearest even, saturate to the largest finite value."""
    fp8type = _dt(fp8type)
    m = FP8_MAX[fp8type]
    return x.float().clamp(-m, m).to(fp8type)


def group_scales(x, QB, fp8type):
    """fp32 (un-rounded) scale of every 1xQB group of a 2-D tensor."""
    M, N = x.shape
    amax = x.float().reshape(M, N // QB, QB).abs().amax(dim=-1)
    return (amax + torch.tensor(SCALE_MIN_THRES, dtype=torch.float32)) / torch.tensor(FP8_MAX[_dt(fp8type)],
                                                                                    dtype=torch.float32)


def fp8_quantize(x, QB, fp8type, scale_dtype=torch.bfloat16):
    M, N = x.shape
    s = group_scales(x, QB, fp8type)
    q = cast_fp8((x.float().reshape(M, N // QB, QB) / s.unsqueeze(-1)).reshape(M, N), fp8type)
    return q, s.to(scale_dtype)


def fp8_division(x, fp8type, s):
    return cast_fp8(x.float() / s.float(), fp8type)


def fp8_quantize_pertensor(x, QB, fp8type, scale_dtype=torch.bfloat16):
    """-> (q, s_max, s_y): group scales rounded to scale_dtype, their maximum, q = x / s_max."""
    s_y = group_scales(x, QB, fp8type).to(scale_dtype)
    s_max = s_y.max()
    return fp8_division(x, fp8type, s_max), s_max, s_y


def fp8_quantize_pertensor_transpose(x, QB, fp8type, scale_dtype=torch.bfloat16):
    q, s_max, _ = fp8_quantize_pertensor(x, QB, fp8type, scale_dtype)
    return q, s_max, q.view(torch.uint8).t().contiguous().view(q.dtype)


def fp8_quantize_transpose(x, QB, fp8type, scale_dtype=torch.bfloat16):
    y, s_y = fp8_quantize(x, QB, fp8type, scale_dtype)
    y_t, s_y_t = fp8_quantize(x.t().contiguous(), QB, fp8type, scale_dtype)
    return (y, s_y), (y_t, s_y_t)


def fp8_dequantize(q, s, QB):
    M, N = q.shape
    return (q.float().reshape(M, N // QB, QB) * s.float().unsqueeze(-1)).reshape(M, N).to(torch.bfloat16)


def near_rounding_boundary(x_over_s, fp8type, ulps=4):
    """Mask of quotients that lie within `ulps` fp32 ulps of an FP8 rounding boundary (where IEEE
    division and div.full.f32, which may differ by 2 ulp, can legitimately give different codes)."""
    fp8type = _dt(fp8type)
    q = x_over_s.float().abs().clamp(max=FP8_MAX[fp8type])
    lo = cast_fp8(q * (1 - ulps * 2.0 ** -23), fp8type).view(torch.uint8)
    hi = cast_fp8(q * (1 + ulps * 2.0 ** -23), fp8type).view(torch.uint8)
    return lo != hi


def fp8_quantize_block128(x, fp8type, scale_dtype=torch.float32):
    """128-wide granularities of the block-scaled linear layer, IEEE division
    (coat/activation/real_quantization/_quantize_perblock.py:70-84, _quantize_perblock_transpose_pergroup.py:145-160,
    _quantize_transpose.py with QB = 128).  Returns a dict of (codes, scales):
      "block"  [M,N], [M/128, N/128];   "block_t" [N,M], [N/128, M/128]
      "rows"   [M,N], [M, N/128];       "cols_t"  [N,M], [N, M/128]"""
    M, N = x.shape
    xf = x.float()
    fmax = FP8_MAX[fp8type]
    xb = xf.reshape(M // 128, 128, N // 128, 128)
    s_b = (xb.abs().amax(dim=(1, 3)) + 1e-10) / fmax
    q_b = cast_fp8((xb / s_b[:, None, :, None]).reshape(M, N), fp8type)
    s_r = (xf.reshape(M, N // 128, 128).abs().amax(dim=2) + 1e-10) / fmax
    q_r = cast_fp8((xf.reshape(M, N // 128, 128) / s_r[:, :, None]).reshape(M, N), fp8type)
    xt = xf.t().contiguous()
    s_c = (xt.reshape(N, M // 128, 128).abs().amax(dim=2) + 1e-10) / fmax
    q_c = cast_fp8((xt.reshape(N, M // 128, 128) / s_c[:, :, None]).reshape(N, M), fp8type)
    return {"block": (q_b, s_b.to(scale_dtype)), "block_t": (q_b.t().contiguous(), s_b.t().contiguous().to(scale_dtype)),
            "rows": (q_r, s_r.to(scale_dtype)), "cols_t": (q_c, s_c.to(scale_dtype))}


# ---- stochastic rounding (_division.py:96-112, 129-150) -------------------------------------------------
# The reference draws its noise with tl.rand(0, offset): Triton's counter-based generator, i.e. the published
# Philox-4x32 with 10 rounds (Salmon et al., "Parallel random numbers: as easy as 1, 2, 3", SC'11; Triton
# 3.x, triton/language/random.py) with key = (seed low word, seed high word), counter = (offset, 0, 0, 0),
# the first output word mapped to [0, 1) as int32 x -> (x if x >= 0 else -x - 1) * 4.6566127342e-10.
import numpy as np  # noqa: E402

_PHILOX_KEY_A, _PHILOX_KEY_B = 0x9E3779B9, 0xBB67AE85
_PHILOX_ROUND_A, _PHILOX_ROUND_B = 0xD2511F53, 0xCD9E8D57


def philox4x32(counter, key, rounds=10):
    """counter: 4 arrays of uint32; key: (k0, k1) ints.  Returns the 4 output arrays (uint32)."""
    c0, c1, c2, c3 = (np.asarray(c, dtype=np.uint64) for c in counter)
    k0, k1 = int(key[0]) & 0xffffffff, int(key[1]) & 0xffffffff
    mask = np.uint64(0xffffffff)
    for _ in range(rounds):
        pb = np.uint64(_PHILOX_ROUND_B) * c2
        pa = np.uint64(_PHILOX_ROUND_A) * c0
        c0, c2 = (pb >> np.uint64(32)) ^ c1 ^ np.uint64(k0), (pa >> np.uint64(32)) ^ c3 ^ np.uint64(k1)
        c1, c3 = pb & mask, pa & mask
        k0, k1 = (k0 + _PHILOX_KEY_A) & 0xffffffff, (k1 + _PHILOX_KEY_B) & 0xffffffff
    return tuple(c.astype(np.uint32) for c in (c0, c1, c2, c3))


def triton_rand(seed, offsets):
    """tl.rand(seed, offsets) for int32 offsets, as float32."""
    offs = np.asarray(offsets).astype(np.uint32)
    zero = np.zeros_like(offs)
    word = philox4x32((offs, zero, zero, zero), (seed & 0xffffffff, (seed >> 32) & 0xffffffff))[0]
    x = word.view(np.int32).astype(np.int64)
    x = np.where(x < 0, -x - 1, x)
    return x.astype(np.float32) * np.float32(4.6566127342e-10)


def stochastic_perturb(q, noise, fp8type):
    """_stochastic_rounding (_division.py:129-150) in fp32: |q| plus noise * (one step of the format at q's
    exponent), clamped to q's binade (to [2^-9, 2^-6] resp. [2^-16, 2^-14] below the normal range, so zeros
    become the smallest subnormal), with q's sign.  The caller's saturating RNE cast follows."""
    fp8type = _dt(fp8type)
    m_bit = 3 if fp8type == torch.float8_e4m3fn else 2
    sub_min = np.float32(2.0 ** -9 if fp8type == torch.float8_e4m3fn else 2.0 ** -16)
    q = np.asarray(q, dtype=np.float32)
    e = np.maximum((q.view(np.uint32) & np.uint32(0x7F800000)).view(np.float32), sub_min)
    sub = e == sub_min
    step = np.where(sub, np.float32(1.0), np.float32(2.0 ** -m_bit)).astype(np.float32)
    n = (e * np.asarray(noise, dtype=np.float32)) * step          # division by 2^m or 1: exact
    a = np.abs(q) + n
    hi = np.where(sub, np.float32(2.0 ** m_bit), np.float32(2.0)).astype(np.float32) * e
    a = np.minimum(np.maximum(a, e), hi)
    return np.where(np.signbit(q), -a, a).astype(np.float32)


def fp8_division_stochastic(x, fp8type, s, ld=None):
    """fp8_division(x, QB, fp8type, s, stochastic=True): noise offset of element (m, n) = m * ld + n with
    ld = x's row stride in elements (seed 0, _division.py:107-110)."""
    M, N = x.shape
    ld = N if ld is None else ld
    q = (x.float() / s.float()).numpy()
    offs = (np.arange(M, dtype=np.int64)[:, None] * ld + np.arange(N, dtype=np.int64)[None, :]).astype(np.int32)
    out = stochastic_perturb(q, triton_rand(0, offs), fp8type)
    return cast_fp8(torch.from_numpy(out), fp8type)
