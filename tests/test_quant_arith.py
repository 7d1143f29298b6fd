"""The division-free arithmetic of the activation quantiser (csrc/moe_quant.cu), checked on the CPU with exact
rational arithmetic: every intermediate is rounded to fp32 exactly once, as the GPU's FMA and multiply do.

* scale: RN(amax / 448) == RN(q0 + RN(amax - q0 * 448) * c), q0 = RN(amax * c), c = RN(1/448), for every finite
  positive bf16 amax (all 32,639 of them);
* quotient (Markstein's correction): with r = RN(1/s), y0 = RN(x * r), e = RN(x - y0 * s) and
  z = RN(y0 + e * r), e4m3(z) == e4m3(RN(x / s)) on sampled bf16 x with |x| <= amax and the fast-path scales
  (s >= 2^-64).  y0 can be up to 1.5 ulps from x / s, so e is not always exact and z is not always RN(x / s)
  (those cases round to zero in e4m3); the identity that matters is the e4m3 one.

The Newton reciprocal itself uses the hardware's rcp.approx and is pinned on the GPU
(tests/test_gpu_quant.py::test_quantize_act_exhaustive_bf16 sweeps the whole bf16 domain through the kernel)."""
import random
import struct
from fractions import Fraction

TWO = Fraction(2)


def rn32(v: Fraction) -> Fraction:
    """Round a rational to the nearest fp32 value (ties to even), subnormals included; no overflow handling."""
    if v == 0:
        return Fraction(0)
    neg = v < 0
    a = -v if neg else v
    e = a.numerator.bit_length() - a.denominator.bit_length()
    if TWO ** e > a:
        e -= 1
    while TWO ** (e + 1) <= a:
        e += 1
    quantum = TWO ** (max(e, -126) - 23)
    n = a / quantum
    fl = n.numerator // n.denominator
    rem = n - fl
    if rem > Fraction(1, 2) or (rem == Fraction(1, 2) and fl % 2 == 1):
        fl += 1
    r = fl * quantum
    return -r if neg else r


def rn_e4m3(v: Fraction) -> Fraction:
    """Round to e4m3 (3 mantissa bits, exponents -6..8, subnormal step 2^-9), ties to even, saturating at 448."""
    a = -v if v < 0 else v
    if a == 0:
        return Fraction(0)
    e = a.numerator.bit_length() - a.denominator.bit_length()
    if TWO ** e > a:
        e -= 1
    while TWO ** (e + 1) <= a:
        e += 1
    quantum = TWO ** (max(e, -6) - 3)
    n = a / quantum
    fl = n.numerator // n.denominator
    rem = n - fl
    if rem > Fraction(1, 2) or (rem == Fraction(1, 2) and fl % 2 == 1):
        fl += 1
    r = min(fl * quantum, Fraction(448))
    return -r if v < 0 else r


def bf16(bits: int) -> Fraction:
    return Fraction(struct.unpack("<f", struct.pack("<I", (bits & 0xFFFF) << 16))[0])


C = rn32(Fraction(1, 448))


def scale_fma(amax: Fraction) -> Fraction:
    q0 = rn32(amax * C)
    return rn32(q0 + rn32(amax - q0 * 448) * C)


def test_scale_fma_equals_division_for_every_bf16_amax():
    for b in range(1, 0x7F80):
        a = bf16(b)
        assert scale_fma(a) == rn32(a / 448), hex(b)


def test_markstein_quotient_on_sampled_bf16_pairs():
    rng = random.Random(7)
    amaxes = [b for b in range(1, 0x7F80, 97)] + [0x3F80, 0x4000, 0x43E0, 0x7F7F, 0x2080, 0x1F80]
    checked = 0
    for b in amaxes:
        a = bf16(b)
        s = scale_fma(a)
        if s < TWO ** -64:
            continue
        r = rn32(1 / s)
        xs = [rng.randrange(0, b + 1) for _ in range(24)] + [b, b - 1, 1, 0]
        for m in xs:
            for sign in (1, -1):
                x = sign * bf16(m)
                y0 = rn32(x * r)
                e = rn32(x - y0 * s)
                z, want = rn32(y0 + e * r), rn32(x / s)
                assert rn_e4m3(z) == rn_e4m3(want), (hex(b), hex(m), sign)
                checked += 1
    assert checked > 4000
