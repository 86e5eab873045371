"""The router-logit reduction of the tensor-core MoE path, restated on the CPU.

The down kernels of a decode chain add their 16-row partial router dots into
a carry-save fixed-point accumulator (pokit_moe.cu racc_add / racc_take):
eight 64-bit limbs per expert, limb i holding bits [32 i - 64, 32 i - 32); a
float m * 2^ex lands in at most two adjacent limbs; the reader resolves the
carries, keeps the three leading limbs in double and rounds to float.  These
tests pin the arithmetic: the result is the exactly rounded sum of the float
partials (to float) and does not depend on the order the CTAs arrive in.
"""
import struct
from fractions import Fraction

import numpy as np

LIMBS, BASE = 8, -64


def racc_add(limbs, p):
    b = struct.unpack("<I", struct.pack("<f", p))[0]
    eb = (b >> 23) & 0xFF
    assert eb != 0xFF
    m = b & 0x7FFFFF
    if eb == 0:
        if m == 0:
            return
        ex = -149
    else:
        m |= 0x800000
        ex = eb - 150
    pos = ex - BASE
    if pos < 0:
        if pos <= -24:
            return
        m >>= -pos
        pos = 0
        if m == 0:
            return
    i, o = pos >> 5, pos & 31
    v = m << o
    if b >> 31:
        v = -v
    limbs[i] += v & 0xFFFFFFFF
    limbs[i + 1] += v >> 32


def racc_take(limbs):
    d = float(limbs[LIMBS - 1])
    for i in range(LIMBS - 2, -1, -1):
        d = d * 4294967296.0 + float(limbs[i])      # fma: d * 2^32 is exact, one rounding
    return np.float32(d * 2.0 ** BASE)


def ulp(x):
    return float(np.spacing(np.float32(abs(x)))) if x != 0 else float(np.float32(1e-45))


def test_within_one_ulp_and_order_independent():
    rng = np.random.default_rng(0)
    for trial in range(300):
        scale = 10.0 ** rng.uniform(-12, 30)
        ps = (rng.standard_normal(128) * scale * 10.0 ** rng.uniform(-3, 3, 128)).astype(np.float32)
        exact = float(sum(Fraction(float(x)) for x in ps))
        got = []
        for _ in range(3):
            limbs = [0] * LIMBS
            for j in rng.permutation(128):
                racc_add(limbs, float(ps[j]))
            assert all(abs(v) < 2 ** 63 for v in limbs)
            got.append(racc_take(limbs))
        assert got[0] == got[1] == got[2]
        assert abs(float(got[0]) - exact) <= ulp(exact)


def test_cancellation_and_zero():
    limbs = [0] * LIMBS
    for p in (3.0e20, -3.0e20, 1.5, -0.25):
        racc_add(limbs, p)
    assert racc_take(limbs) == np.float32(1.25)
    limbs = [0] * LIMBS
    for p in (1.0, -1.0):
        racc_add(limbs, p)
    assert racc_take(limbs) == 0.0
