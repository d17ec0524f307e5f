"""The quantiser's division-free quotient (rows.cuh::quant8), restated in exact rational
arithmetic: q = RN(v y), n = RN(q s - v), q' = RN(n (-y) + q) with y = RN(1/s) gives
the int8 / e4m3 code of the IEEE quotient RN(v / s) for per-token scales s = max(amax / qmax,
1e-12), including values on and next to the codes' rounding boundaries, zeros of both
signs and values whose quotient underflows (Markstein's correction step, IBM J. Res.
Dev. 34(1), 1990)."""
from fractions import Fraction as Fr

import numpy as np
import pytest

from oracle import oracle as O


def rn32(x: Fr) -> Fr:
    """Round an exact rational to the nearest fp32 value (ties to even, subnormals kept)."""
    if x == 0:
        return Fr(0)
    sgn, a = (-1, -x) if x < 0 else (1, x)
    e = a.numerator.bit_length() - a.denominator.bit_length()
    while Fr(2) ** e > a:
        e -= 1
    while Fr(2) ** (e + 1) <= a:
        e += 1
    ulp = Fr(2) ** (max(e, -126) - 23)
    m = a / ulp
    fl = m.numerator // m.denominator
    rem = m - fl
    if rem > Fr(1, 2) or (rem == Fr(1, 2) and fl % 2):
        fl += 1
    return sgn * fl * ulp


def as_f32(x: Fr, negative_zero: bool = False) -> np.float32:
    if x == 0:
        return np.float32(-0.0) if negative_zero else np.float32(0.0)
    return np.float32(float(x))


def kernel_quotient(v: np.float32, s: Fr, y: Fr) -> np.float32:
    """The kernel's sequence, with IEEE signed-zero rules for the exact-zero cases."""
    vf = Fr(float(v))
    neg_v = np.signbit(v)
    q = rn32(vf * y)
    q_neg = (q < 0) or (q == 0 and neg_v)            # v * y keeps v's sign (y > 0)
    n = rn32(q * s - vf)
    # n == 0 happens only for v = 0 here: (+-0) * s + (-+0) = +0 in round-to-nearest
    n_neg = n < 0
    qq = rn32(n * (-y) + q)
    if qq == 0:
        # n * (-y) is a zero with sign (n_neg xor 1) when n == 0; x + y of two zeros is -0 only if both are -0
        prod_neg = (not n_neg) if n == 0 else (n * (-y) < 0)
        qq_neg = prod_neg and q_neg if (n == 0 and q == 0) else (q_neg if q != 0 else prod_neg)
        return as_f32(qq, qq_neg)
    return as_f32(qq)


def codes(x: np.float32, qmax: float):
    if qmax == 127.0:
        return int(np.int8(np.rint(x)))
    return int(O.f32_to_e4m3(np.array([x], np.float32))[0])


@pytest.mark.parametrize("qmax", [127.0, 448.0])
def test_quotient_matches_ieee_division(qmax):
    rng = np.random.default_rng(int(qmax))
    checked = 0
    for _ in range(1500):
        amax = np.float32(O.round_bf16(np.array([rng.standard_normal() * 10 ** rng.uniform(-30, 30)], np.float32))[0])
        amax = abs(amax)
        if amax == 0 or not np.isfinite(amax):
            continue
        s = max(rn32(Fr(float(amax)) / Fr(qmax)), rn32(Fr(1e-12)))
        y = rn32(1 / s)
        sf = np.float32(float(s))
        k = rng.integers(-int(qmax), int(qmax))
        cands = [np.float32(rng.uniform(-1, 1) * float(amax)),
                 np.float32((k + 0.5) * float(s)), np.float32(-0.0), np.float32(0.0),
                 np.float32(float(amax) * 1e-30)]
        for v in cands:
            v = np.float32(O.round_bf16(np.array([v], np.float32))[0]) if rng.random() < 0.5 else v
            ref = np.float32(v) / sf                                   # IEEE fp32 quotient
            got = kernel_quotient(np.float32(v), s, y)
            assert codes(got, qmax) == codes(ref, qmax), (v, sf, got, ref)
            if abs(float(ref)) >= 2.0 ** -12:
                assert got == ref
            checked += 1
    assert checked > 5000
