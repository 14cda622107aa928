"""CPU proofs of the integer identities the sm_100a kernels use in place of the spec's direct formulas.

Each test restates, in Python integers (and exactly rounded binary64 where the kernel uses it), the short form a
kernel computes and checks it against the spec form on edge values and seeded random values:

- quant_pack4 (intops.cuh): q = ((v >> s1) + r) >> s2, then cvt.pack.sat.s16.s32 and max.s16x2 with -32767, split
  into hi / lo bytes  ==  quant16(v, e) = clamp(rshr(v, e), +-32767) split into planes;
- quant_pack4_e15: (v + 2^(e-1)) >> e for e <= 15 and |v| < 2^(15+e)  ==  rshr(v, e);
- quant_nosat / quant_pack4_e15_nosat: for a row maximum m with m + 2^(e-1) < 2^(15+e) (or e = 0) no value of the
  row saturates, and four byte selections of the 32-bit results give the hi / lo plane bytes;
- the q|k|v / V plane sums: sum q = 256 sum hi + sum lo + 128 n;
- lut16_s (intops.cuh): the sentinel table indexed by clamp((x >> 10) + 1024, -1, 2048) + 1  ==  lut16;
- lut_act_s: x * lut / 2^16 rounded needs no saturation when 0 <= lut <= 65536;
- norm_val (rowops.cu): the binary64 quotient formed with the 1.5 * 2^52 constant and one fma residual test
  ==  floor((d 2^(25-e) + sd) / (2 sd));
- the attention softmax forms (attn.cu): the 32-bit score (hh M + (T >> a)) >> b, its mixed-exponent
  variant, the exp-table index read from the quotient before its >> b, the table interpolated with one mad.hi, and
  P from the reciprocal's 32-bit halves saturated by the packing instruction;
- the int32 staging quantiser is covered by the GPU parity tests.
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


def byte_perm(x, y, sel):
    b = (x & 0xFFFFFFFF).to_bytes(4, "little") + (y & 0xFFFFFFFF).to_bytes(4, "little")
    return int.from_bytes(bytes(b[(sel >> (4 * i)) & 7] for i in range(4)), "little")


def quant_nosat(m, e):
    return e == 0 or m + (1 << (e - 1)) < (1 << (15 + e))


def test_no_saturation_rows():
    # quant_nosat(m, e) with e = row_exp(m) holds exactly when no v in [-m, m] saturates (the extremes decide,
    # rshr being monotone); when it fails, v = m does saturate
    rnd = random.Random(15)
    ms = [0, 1, 32767, 32768, 65535, 65536, 2**31 - 1, 2**32 - 1]
    for e in range(1, 18):
        top = (1 << (15 + e)) - 1
        ms += [top, top - (1 << (e - 1)), top - (1 << (e - 1)) + 1, 1 << (14 + e), (1 << (14 + e)) + 1]
    ms += [rnd.randint(0, 2**32 - 1) >> rnd.randint(0, 31) for _ in range(20000)]
    for m in ms:
        e = row_exp(m)
        if m >= 2**31:
            continue                      # int32 activations: |v| <= 2^31
        free = -32767 <= rshr(-m, e) and rshr(m, e) <= 32767
        assert quant_nosat(m, e) == free, (m, e)
        if not free:
            assert quant16(m, e) != rshr(m, e)


def test_nosat_byte_packing():
    rnd = random.Random(16)
    for _ in range(20000):
        q = [rnd.randint(-32767, 32767) for _ in range(4)]
        if rnd.random() < 0.1:
            q = [rnd.choice([-32767, 32767, 0, -1, 255, -256]) for _ in range(4)]
        a, b = byte_perm(q[0], q[1], 0x4051), byte_perm(q[2], q[3], 0x4051)
        hw, lw = byte_perm(a, b, 0x5410), byte_perm(a, b, 0x7632) ^ 0x80808080
        his = [(hw >> (8 * i)) & 255 for i in range(4)]
        los = [(lw >> (8 * i)) & 255 for i in range(4)]
        for i in range(4):
            h, l = planes(q[i])
            assert his[i] == h & 255 and los[i] == l & 255, (q, i)


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


# ---------------------------------------------------------------- attention softmax (attn.cu)
def s32(v):                 # two's-complement wrap to int32
    v &= 0xFFFFFFFF
    return v - (1 << 32) if v >= 1 << 31 else v


def mulhi32(a, b):          # mul.hi.s32 of two int32 values
    return (a * b) >> 32


def div_pow2_model(hh, T, sh):
    """attn.cu div_pow2 then >> b, for a = min(sh, 16), b = sh - a, M = 2^(16-a): (hh M + (T >> a)) mod 2^32, then >> b"""
    a = min(sh, 16)
    return s32(hh * (1 << (16 - a)) + (T >> a)) >> (sh - a)


def _score_operands(rnd, n):
    """(hh, xx, ll, kc, cq, S) drawn like the accumulators of a 64-dim head of 16-bit values (edges included)"""
    out = []
    for _ in range(n):
        q = [rnd.choice([-32767, 32767, rnd.randint(-32767, 32767)]) for _ in range(64)]
        k = [rnd.choice([-32767, 32767, rnd.randint(-32767, 32767)]) for _ in range(64)]
        qh, ql = zip(*(planes(v) for v in q))
        kh, kl = zip(*(planes(v) for v in k))
        hh = sum(a * b for a, b in zip(qh, kh))
        xx = sum(a * b for a, b in zip(qh, kl)) + sum(a * b for a, b in zip(ql, kh))
        ll = sum(a * b for a, b in zip(ql, kl))
        cq = 32768 * sum(qh) + 128 * sum(ql)
        kc = 128 * sum(k)
        S = sum(a * b for a, b in zip(q, k))
        assert S == 65536 * hh + 256 * xx + ll + cq + kc
        out.append((hh, xx, ll, kc, cq, S))
    return out


def test_attention_score_32bit_form():
    """one key exponent per chunk: (hh M + (T >> a)) >> b == rshr(S, sh) for every shift the fast path takes"""
    rnd = random.Random(21)
    ops = _score_operands(rnd, 300)
    ops.append((64 * 128 * 128, 0, 0, 0, 0, 64 * 128 * 128 * 65536))      # every plane product at its largest magnitude
    for hh, xx, ll, kc, cq, S in ops:
        for sh in range(5, 20):
            T = 256 * xx + ll + kc + cq + (1 << (sh - 1))
            assert INT_MIN <= T <= INT_MAX
            want = rshr(S, sh)
            if INT_MIN <= want <= INT_MAX:
                assert div_pow2_model(hh, T, sh) == want, (hh, T, sh)


def test_attention_score_mixed_exponents():
    """keys of a chunk with different exponents: the smallest shift sh0 = shq - max ek for the division, each key's own
    rounding term 2^(shq - ek - 1) in T, then >> (b0 + max ek - ek)  ==  rshr(S, shq - ek)"""
    rnd = random.Random(22)
    for hh, xx, ll, kc, cq, S in _score_operands(rnd, 200):
        for shq in range(7, 20):
            for emax in range(0, min(4, shq - 5) + 1):
                a0 = min(shq - emax, 16)
                b0 = shq - emax - a0
                for ek in range(0, emax + 1):
                    T = 256 * xx + ll + kc + cq + ((1 << (shq - 1)) >> ek)
                    got = s32(hh * (1 << (16 - a0)) + (T >> a0)) >> (b0 + emax - ek)
                    assert got == rshr(S, shq - ek), (shq, emax, ek)


def exp_lut_ref(z, L):
    """src/kernels.cu:671-722 lut_exp: 0 from z = 2^20 on, else L[i] + ((L[i+1] - L[i]) f >> 10), truncated to int32"""
    if z >= 1 << 20:
        return 0
    i, f = z >> 10, z & 1023
    return s32(L[i] + (((L[i + 1] - L[i]) * f) >> 10))


def exp_fast_model(z, L):
    """attn.cu exp_fast: zc = min(z, 2^20); entry (L[i], 2 (L[i+1] - L[i])), sentinel (0, 0) at 1024;
    E = mad.hi.s32(2 D, f 2^21, L[i])"""
    zc = min(z, 1 << 20)
    i, f = zc >> 10, zc & 1023
    Li, D2 = (L[i], 2 * (L[i + 1] - L[i])) if i < 1024 else (0, 0)
    assert INT_MIN <= D2 <= INT_MAX and 0 <= f << 21 < 2**31
    return s32(mulhi32(D2, f << 21) + Li)


def test_attention_exp_table_fast_form():
    import math
    rnd = random.Random(23)
    tables = [[round(2**30 * math.exp(-i / 64.0)) for i in range(1025)]]
    # random tables that still qualify: values in [0, 2^31), neighbour differences below 2^30
    for _ in range(3):
        t = [rnd.randint(0, 2**31 - 1)]
        for _ in range(1024):
            t.append(min(2**31 - 1, max(0, t[-1] + rnd.randint(-(2**30) + 1, 2**30 - 1))))
        tables.append(t)
    for L in tables:
        assert all(0 <= v < 2**31 for v in L) and all(abs(L[i + 1] - L[i]) < 2**30 for i in range(1024))
        zs = [0, 1, 1023, 1024, (1 << 20) - 1, 1 << 20, (1 << 20) + 5, 2**32 - 1] + [rnd.randint(0, 1 << 20) for _ in range(3000)]
        for z in zs:
            assert exp_fast_model(z, L) == exp_lut_ref(z, L), z


def exp_fast_d_model(d, b, L):
    """attn.cu exp_fast_d on d (uint32): i = min(d >> (b + 10), 1024), f 2^21 = (d 2^(21 - b) mod 2^32) & (1023 << 21),
    E = mad.hi.s32(2 D, f 2^21, L[i]) with the sentinel (0, 0) at 1024"""
    i = min(d >> (b + 10), 1024)
    F = (d * (1 << (21 - b))) & 0x7FE00000
    Li, D2 = (L[i], 2 * (L[i + 1] - L[i])) if i < 1024 else (0, 0)
    return s32(mulhi32(D2, F) + Li)


def test_attention_exp_index_from_quotient():
    """the exp-table index and fraction from d = mx 2^b + 2^b - 1 - u (mod 2^32), u the score before its >> b, equal the
    table at z = mx - (u >> b) for every shift the fast path takes and every valid key (u >> b <= mx); the default table
    also qualifies for the three-term 32-bit sums (every entry <= 2^32 / 3)"""
    import math
    rnd = random.Random(25)
    L = [round(2**30 * math.exp(-i / 64.0)) for i in range(1025)]
    assert max(L) <= 0x55555555 and 3 * max(L) < 2**32
    for hh, xx, ll, kc, cq, S in _score_operands(rnd, 150):
        for sh in range(5, 20):
            a = min(sh, 16)
            b = sh - a
            T = 256 * xx + ll + kc + cq + (1 << (sh - 1))
            u = s32(hh * (1 << (16 - a)) + (T >> a))
            s = u >> b
            if b > 0:
                assert abs(u) < 2**21
            for z in (0, 1, 1023, 1024, (1 << 20) - 1, 1 << 20, (1 << 20) + 3, rnd.randint(0, 1 << 21), rnd.randint(0, 1 << 20)):
                mx = s + z
                if mx > INT_MAX:
                    continue
                mxb = (mx << b) + (1 << b) - 1
                assert b == 0 or INT_MIN <= mxb <= INT_MAX
                d = (mxb - u) & 0xFFFFFFFF
                assert exp_fast_d_model(d, b, L) == exp_lut_ref(z, L), (sh, z)


def test_attention_p_short_form():
    """P = min(32767, (E r + 2^46) >> 47) with r = floor(2^62 / sum E) == sat16((E rhi + hi32(E rlo) + 2^14) >> 15), the
    saturation being that of cvt.pack.sat.s16.s32 (the value is below 2^17); sum P is read from the P.V products as
    256 sum ph + sum pl + 128 n (the plane-sum identity of test_plane_sums, padded keys carrying P = 0)"""
    rnd = random.Random(24)
    for _ in range(3000):
        n = rnd.randint(1, 4096)
        Es = [rnd.choice([0, 2**30, rnd.randint(0, 2**30), rnd.randint(0, 1000)]) for _ in range(min(n, 8))]
        tot = sum(Es) + rnd.randint(0, (n - len(Es)) * 2**30 if n > len(Es) else 0)
        if tot == 0:
            continue
        r = (1 << 62) // tot
        rhi, rlo = r >> 32, r & 0xFFFFFFFF
        for E in Es:
            want = min(32767, (E * r + (1 << 46)) >> 47)
            h = (E * rhi + ((E * rlo) >> 32) + 16384) & 0xFFFFFFFF
            assert h >> 15 < 2**17 and pack_sat16(h >> 15) == want
    # a single key carries the whole sum: P = 32768 before the clamp
    r = (1 << 62) // (2**30)
    h = (2**30 * (r >> 32) + ((2**30 * (r & 0xFFFFFFFF)) >> 32) + 16384) & 0xFFFFFFFF
    assert h >> 15 == 32768 and pack_sat16(h >> 15) == 32767
