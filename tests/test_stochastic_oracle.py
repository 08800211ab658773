"""CPU tests that pin the oracle of the stochastic-rounding division (oracle/quant.py): the Philox-4x32-10
generator against the known-answer vectors published with the generator (Random123's kat_vectors: zero
input, all-ones input, and the digits of pi), and the properties of the perturbation the reference applies
(coat/activation/real_quantization/_division.py:129-150)."""
import numpy as np
import torch

from oracle.quant import fp8_division, fp8_division_stochastic, philox4x32, stochastic_perturb, triton_rand


def _kat(counter, key):
    return [int(v[0]) for v in philox4x32([np.array([c], dtype=np.uint32) for c in counter], key)]


def test_philox_known_answers():
    assert _kat([0, 0, 0, 0], (0, 0)) == [0x6627e8d5, 0xe169c58d, 0xbc57ac4c, 0x9b00dbd8]
    assert _kat([0xffffffff] * 4, (0xffffffff, 0xffffffff)) == [0x408f276d, 0x41c83b0e, 0xa20bc7c6, 0x6d5451fd]
    assert _kat([0x243f6a88, 0x85a308d3, 0x13198a2e, 0x03707344], (0xa4093822, 0x299f31d0)) == \
        [0xd16cfe09, 0x94fdcceb, 0x5001e420, 0x24126ea1]


def test_rand_is_uniform_in_unit_interval():
    r = triton_rand(0, np.arange(1 << 16))
    assert r.dtype == np.float32 and r.min() >= 0.0 and r.max() < 1.0
    assert abs(float(r.mean()) - 0.5) < 5e-3 and abs(float(r.var()) - 1 / 12) < 2e-3
    # word 0x6627e8d5 (counter 0, key 0) is positive as int32: value * 4.6566127342e-10
    assert r[0] == np.float32(0x6627e8d5) * np.float32(4.6566127342e-10)


def test_perturbation_stays_in_the_binade_and_lifts_zero():
    q = np.array([0.0, -0.0, 1.0, -1.5, 3.999, 2.0 ** -9, 2.0 ** -7, 300.0], dtype=np.float32)
    for fmt, m, sub_min in (("E4M3", 3, 2.0 ** -9), ("E5M2", 2, 2.0 ** -16)):
        lo = stochastic_perturb(q, np.zeros_like(q), fmt)
        hi = stochastic_perturb(q, np.full_like(q, 0.99999994), fmt)
        # noise 0 leaves normal values alone; zeros become the smallest subnormal with the zero's sign
        assert lo[0] == np.float32(sub_min) and lo[1] == -np.float32(sub_min)
        assert np.array_equal(lo[2:5], q[2:5])
        # the largest noise adds just under one step 2^(e-m) and never leaves [2^e, 2^(e+1)]
        assert hi[2] <= 1.0 + 2.0 ** -m and hi[2] > 1.0 + 0.99 * 2.0 ** -m
        assert hi[3] >= -(1.5 + 2.0 ** -m) and hi[4] <= 4.0
        assert np.all(np.signbit(hi) == np.signbit(q))


def test_stochastic_division_moves_codes_up_by_at_most_one_step():
    gen = torch.Generator().manual_seed(5)
    x = torch.randn(64, 256, generator=gen).to(torch.bfloat16)
    s = torch.tensor(0.01, dtype=torch.bfloat16)
    for fmt in ("E4M3", "E5M2"):
        near = fp8_division(x, fmt, s).float()
        sto = fp8_division_stochastic(x, fmt, s).float()
        assert torch.all(sto.abs() >= near.abs() - 0)   # |q| + noise, then round to nearest: never smaller...
        up = (sto.abs() > near.abs()).float().mean()
        assert 0.3 < float(up) < 0.7                     # ...and one step larger about half of the time
        # same binade or the next power of two
        assert torch.all(sto.abs() <= 2 * near.abs().clamp(min=2.0 ** -16))
