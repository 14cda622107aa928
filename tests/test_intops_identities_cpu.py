"""CPU proofs of the integer identities the sm_100a kernels use in place of the spec's direct formulas.

Each test restates, in Python integers (and exactly rounded binary64 where the kernel uses it), the short form a
kernel computes and checks it against the spec form on edge values and seeded random values:

- quant_pack4 (intops.cuh): q = ((v >> s1) + r) >> s2, then cvt.pack.sat.s16.s32 and max.s16x2 with -32767, split
  into hi / lo bytes  ==  quant16(v, e) = clamp(rshr(v, e), +-32767) split into planes;
- quant_pack4_e15: (v + 2^(e-1)) >> e for e <= 15 and |v| < 2^(15+e)  ==  rshr(v, e);
- the q|k|v / V plane sums: sum q = 256 sum hi + sum lo + 128 n;
- lut16_s (intops.cuh): the sentinel table indexed by clamp((x >> 10) + 1024, -1, 2048) + 1  ==  lut16;
- lut_act_s: x * lut / 2^16 rounded needs no saturation when 0 <= lut <= 65536;
- norm_val (rowops.cu): the binary64 quotient formed with the 1.5 * 2^52 constant and one fma residual test
  ==  floor((d 2^(25-e) + sd) / (2 sd));
- the int32 staging quantiser and the attention score identities are covered by the GPU parity tests.
"""
import random
import struct
from fractions import Fraction

INT_MIN, INT_MAX = -2**31, 2**31 - 1


def rshr(v, e):
    return v if e == 0 else (v + (1 << (e - 1))) >> e


def quant16(v, e):
    return max(-32767, min(32767, rshr(v, e)))


def planes(q):
    return q >> 8, (q & 255) - 128


def pack_sat16(q):          # cvt.pack.sat.s16.s32 of one source
    return max(-32768, min(32767, q))


def quant_pack4_model(vs, s1, r, s2):
    out = []
    for v in vs:
        q = ((v >> s1) + r) >> s2
        q = max(pack_sat16(q), -32767)                  # max.s16x2 with 0x8001 in each half
        out.append(planes(q))
    return out


def row_exp(m):             # max(0, bitlen(m) - 15)
    return max(0, m.bit_length() - 15)


def test_quant_pack4_is_quant16():
    rnd = random.Random(11)
    for e in range(0, 18):
        s1, r, s2 = (e - 1, 1, 1) if e > 0 else (0, 0, 0)
        lim = min(INT_MAX, (1 << (15 + e)) - 1)
        vals = [0, 1, -1, lim, -lim, INT_MAX, INT_MIN + 1, 32767 << e, -(32767 << e)]
        vals += [rnd.randint(INT_MIN + 1, INT_MAX) for _ in range(400)] + [rnd.randint(-lim, lim) for _ in range(400)]
        vals = [v for v in vals if INT_MIN <= v <= INT_MAX]
        for i in range(0, len(vals) - 3, 4):
            got = quant_pack4_model(vals[i:i + 4], s1, r, s2)
            assert got == [planes(quant16(v, e)) for v in vals[i:i + 4]], (e, vals[i:i + 4])


def test_two_operation_rounding_below_e16():
    rnd = random.Random(12)
    for e in range(0, 16):
        lim = (1 << (15 + e)) - 1
        h = (1 << e) >> 1
        for v in [0, 1, -1, lim, -lim, lim - h, -lim + h] + [rnd.randint(-lim, lim) for _ in range(2000)]:
            assert abs(v + h) < 2**31
            q = max(pack_sat16((v + h) >> e), -32767)
            assert q == quant16(v, e), (e, v)


def test_row_exponent_bounds_the_row():
    # row_exp(max |v|) gives every |v| of the row below 2^(15+e), the premise of the two-operation rounding
    rnd = random.Random(13)
    for _ in range(5000):
        m = rnd.randint(0, 2**32 - 1) >> rnd.randint(0, 31)
        e = row_exp(m)
        assert m < 2 ** (15 + e)


def test_plane_sums():
    rnd = random.Random(14)
    for _ in range(2000):
        e = rnd.randint(0, 17)
        qs = [quant16(rnd.randint(INT_MIN + 1, INT_MAX), e) for _ in range(64)]
        hs = sum(planes(q)[0] for q in qs)
        ls = sum(planes(q)[1] for q in qs)
        assert sum(qs) == 256 * hs + ls + 128 * len(qs)


def lut16(x, L):            # the spec: 2049 entries on [-16, 16) in Q16, 0 below and 65536 above
    z = x + (16 << 16)
    if z < 0:
        return 0
    if z >= (32 << 16):
        return 65536
    i, f = z >> 10, z & 1023
    return L[i] + (((L[i + 1] - L[i]) * f) >> 10)


def lut16_sentinel(x, L):   # lut16_s: T[0] = (0, 0), T[1 + i] = (L[i], L[i+1] - L[i]), T[2049] = (65536, 0)
    T = [(0, 0)] + [(L[i], L[i + 1] - L[i]) for i in range(2048)] + [(65536, 0)]
    ex, ey = T[min(max((x >> 10) + 1024, -1), 2048) + 1]
    return ex + ((ey * (x & 1023)) >> 10)


def test_sentinel_table():
    import math
    xs = [i / 64.0 - 16.0 for i in range(2049)]
    L = [round(65536.0 / (1.0 + math.exp(-x))) for x in xs]
    rnd = random.Random(15)
    probes = [INT_MIN, INT_MAX, -(16 << 16), -(16 << 16) - 1, (16 << 16) - 1, 16 << 16, 0, 1023, -1024]
    probes += [rnd.randint(-(20 << 16), 20 << 16) for _ in range(3000)] + [rnd.randint(INT_MIN, INT_MAX) for _ in range(500)]
    for x in probes:
        assert lut16_sentinel(x, L) == lut16(x, L), x
        lut = lut16(x, L)
        assert 0 <= lut <= 65536
        y = (x * lut + 32768) >> 16                 # lut_act_s: no saturation needed
        assert INT_MIN <= y <= INT_MAX and abs(y) <= abs(x) + 1


MAGIC = 6755399441055744.0  # 1.5 * 2^52


def f64(v):
    return struct.unpack("<d", struct.pack("<d", v))[0]


def fma(a, b, c):           # exact product and sum, one rounding to nearest-even binary64
    return float(Fraction(a) * Fraction(b) + Fraction(c))


def bits_low_word(v):
    return struct.unpack("<q", struct.pack("<d", v))[0] & 0xFFFFFFFF


def as_i32(u):
    return u - (1 << 32) if u >= 1 << 31 else u


def norm_quotient_kernel(x, mean, e, sd):
    c = f64(MAGIC + float(mean))
    scale = float(1 << (25 - e))
    D = 2.0 * float(sd)
    rcp = f64(1.0 / D)
    xb = MAGIC + x                                   # the bits of 1.5 * 2^52 + x (exact for |x| < 2^51)
    num = fma(xb - c, scale, float(sd))
    t = fma(num, rcp, MAGIC)
    q = as_i32(bits_low_word(t))
    r = fma(-(t - MAGIC), D, num)
    q += int(r >= D) - int(r < 0.0)
    return q


def test_norm_quotient():
    rnd = random.Random(16)
    for _ in range(3000):
        e = rnd.randint(0, 12)
        mean = rnd.randint(-(1 << 30), 1 << 30)
        rng = rnd.randint(1, min((1 << (20 + e)) - 1, 2**31 - 1 - abs(mean)))
        x = mean + rnd.randint(-rng, rng)
        if not INT_MIN <= x <= INT_MAX:
            continue
        # sd = isqrt((var + eps) << 16) of the group's e-scaled deviations bounds every |d| 2^(24-e) / sd by about
        # 2^16 sqrt(n) (n = group size), so the quotient fits 32 bits; draw sd anywhere from that bound to 2^28
        d = x - mean
        sd = rnd.randint(max(1, -(-abs(d) * (1 << (25 - e)) // (1 << 30))), 1 << 28)
        want = (d * (1 << (25 - e)) + sd) // (2 * sd)
        assert norm_quotient_kernel(x, mean, e, sd) == want, (x, mean, e, sd)
