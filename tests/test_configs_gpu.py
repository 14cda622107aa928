"""The BASELINE configurations at their stated shapes on the B200, bit-exact against the CPU oracle.

Config 2 -- exact attention at 8 x 5 heads x 4096 queries x 4096 keys x 64, on activations uniform over
[-127, 127] (the configuration's value range: every exponent 0) and on the reference's own test distribution
(random bit widths 1..31, src/engine.cu:578-581, so exponents and shifts vary per row and key); the
cross-attention shape (4096 queries, 77 keys padded to 128) and the 32x32 / 16x16 levels' self-attention
(10 heads x 1024, 20 heads x 256).  Query rows are independent, so where the oracle would take minutes the
check covers, per batch, one 128-row query tile at a seeded offset plus 32 scattered rows -- every output word
and row maximum of those rows, all heads, all keys.

Config 3 -- GroupNorm (32 groups) + SiLU of seeded uniform int16 activations, int32 NHWC [8, H*W, C], then the
implicit 3x3 convolution C -> C: 320 ch at 64x64, 640 ch at 32x32, 1280 ch at 16x16.  Every statistics
record, normalised value, pixel maximum, window exponent and convolution output word is compared.
"""
import numpy as np
import pytest

from oracle import pyoracle as O

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")
if not torch.cuda.is_available():
    pytest.skip("no CUDA device", allow_module_level=True)

import ctypes  # noqa: E402

import vela_b200 as V  # noqa: E402
from vela_b200 import abi  # noqa: E402
from tests.gpu_util import Dev, P, A, H, rbits  # noqa: E402


def lexp_lut():
    return np.rint(1073741824.0 * np.exp(-np.arange(1025) / 64.0)).astype(np.int32)


def gpu_attention(d, Q, K, Vv, B, heads, Tq, Tk, lexp):
    """quantise Q, K, V with the library's quantisers and run vela_fused_attention; returns out, rowmax and the host
    copies of the quantised operands"""
    C, G = 64 * heads, B * heads
    Tqp, Tkp = (Tq + 127) // 128 * 128, (Tk + 63) // 64 * 64
    L = V.lib()
    q = [d.zeros((G, Tqp, 64), torch.int8), d.zeros((G, Tqp, 64), torch.int8), d.zeros((G, Tqp), torch.int32)] + [d.zeros((G, Tqp), torch.int64) for _ in range(3)]
    k = [d.zeros((G, Tkp, 64), torch.int8), d.zeros((G, Tkp, 64), torch.int8), d.zeros((G, Tkp), torch.int32)] + [d.zeros((G, Tkp), torch.int64) for _ in range(3)]
    V.check(L.vela_quant_heads(None, P(d(Q)), B, Tq, C, heads, Tqp, *[P(t) for t in q]))
    V.check(L.vela_quant_heads(None, P(d(K)), B, Tk, C, heads, Tkp, *[P(t) for t in k]))
    vh, vl = d.zeros((G, 64, Tkp), torch.int8), d.zeros((G, 64, Tkp), torch.int8)
    ev, vs, scr = d.zeros((G, 64), torch.int32), d.zeros((G, 64), torch.int64), d.zeros((G, 64), torch.int32)
    V.check(L.vela_quant_v(None, P(d(Vv)), B, Tk, C, heads, Tkp, P(vh), P(vl), P(ev), P(vs), P(scr)))
    out = d.empty((B, Tq, C), torch.int32, 0x5A); rm = d.zeros((B * Tq,), torch.int32)
    V.check(L.vela_fused_attention(None, P(q[0]), P(q[1]), P(q[2]), P(q[3]), P(q[4]), P(k[0]), P(k[1]), P(k[2]), P(k[5]),
                                   P(vh), P(vl), P(ev), P(vs), B, heads, Tq, Tqp, Tk, Tkp, 0, P(d(lexp)), C, None, None, P(out), P(rm)))
    torch.cuda.synchronize()
    assert L.vela_device_error(1) == 0
    return H(out), H(rm).view(np.uint32), [H(t) for t in q[:3]], [H(t) for t in k[:3]], [H(t) for t in (vh, vl, ev)]


def sample_rows(rng, B, Tq, n_tile=128, n_scatter=32):
    """per batch: one aligned 128-row query tile at a seeded offset and 32 scattered rows (all distinct, sorted)"""
    rows = []
    for _ in range(B):
        if Tq <= n_tile + n_scatter:
            rows.append(np.arange(Tq))
            continue
        t0 = int(rng.integers(0, Tq // n_tile)) * n_tile
        rest = np.setdiff1d(np.arange(Tq), np.arange(t0, t0 + n_tile))
        rows.append(np.sort(np.concatenate([np.arange(t0, t0 + n_tile), rng.choice(rest, n_scatter, replace=False)])))
    return np.stack(rows)


def check_attention(B, heads, Tq, Tk, make, seed, sampled):
    rng = np.random.default_rng(seed); d = Dev()
    C = 64 * heads
    Q, K, Vv = make(rng, (B, Tq, C)), make(rng, (B, Tk, C)), make(rng, (B, Tk, C))
    lex = lexp_lut()
    out, rm, q, k, v = gpu_attention(d, Q, K, Vv, B, heads, Tq, Tk, lex)
    rows = sample_rows(rng, B, Tq) if sampled else np.tile(np.arange(Tq), (B, 1))
    n = rows.shape[1]
    # the oracle on the chosen query rows only: head g = b * heads + h takes batch b's rows
    G = B * heads
    gi = np.repeat(np.arange(B), heads)
    qs = [np.ascontiguousarray(t[np.arange(G)[:, None], rows[gi]]) for t in q]
    eo, erm = O.attention(qs[0], qs[1], qs[2], k[0], k[1], k[2], v[0], v[1], v[2], B, heads, n, Tk, False, lex)
    got = out[np.arange(B)[:, None], rows]
    assert np.array_equal(got, eo), "attention output words differ from the oracle"
    assert np.array_equal(rm.reshape(B, Tq)[np.arange(B)[:, None], rows], erm.reshape(B, n)), "attention row maxima differ"


def uniform127(rng, shape):
    return rng.integers(-127, 128, shape, dtype=np.int64).astype(np.int32)


def random_bits(rng, shape):
    return rbits(rng, shape, 31)


@pytest.mark.parametrize("make", [uniform127, random_bits], ids=["uniform127", "random_bits"])
def test_config2_self_attention_8x5x4096(make):
    check_attention(8, 5, 4096, 4096, make, 20 if make is uniform127 else 21, sampled=True)


@pytest.mark.parametrize("B,heads,Tq,Tk,sampled", [(8, 5, 4096, 77, False), (8, 10, 1024, 1024, True), (8, 20, 256, 256, False)],
                         ids=["cross_5h_4096x77", "self_10h_1024", "self_20h_256"])
def test_config2_other_attention_shapes(B, heads, Tq, Tk, sampled):
    check_attention(B, heads, Tq, Tk, random_bits, 22 + heads, sampled)


def sigmoid_lut():
    xs = np.arange(2049, dtype=np.float64) / 64.0 - 16.0
    return np.rint(65536.0 / (1.0 + np.exp(-xs))).astype(np.int32)


@pytest.mark.parametrize("Hh,C", [(64, 320), (32, 640), (16, 1280)], ids=["320ch_64x64", "640ch_32x32", "1280ch_16x16"])
def test_config3_groupnorm_then_implicit_conv(Hh, C):
    L = V.lib(); d = Dev(); rng = np.random.default_rng(30 + C)
    B, T, N, K = 8, Hh * Hh, C, 9 * C
    X = rng.integers(-32768, 32768, (B, T, C), dtype=np.int64).astype(np.int32)
    gam = rng.integers(65536 - 16384, 65536 + 16384, C, dtype=np.int64).astype(np.int32)
    beta = rng.integers(-8192, 8192, C, dtype=np.int64).astype(np.int32)
    sig = sigmoid_lut()
    W = rng.integers(-127, 128, (N, K), dtype=np.int64).astype(np.int8)          # tap-major K = (ky*3+kx)*C + c
    cst = np.zeros((N, 4), np.int32)
    cst[:, 0] = rng.integers(16384, 32768, N); cst[:, 1] = rng.integers(20, 30, N)
    cst[:, 2] = rng.integers(-50000, 50000, N); cst[:, 3] = W.astype(np.int64).sum(1)
    # ---- GPU: statistics, normalise + SiLU (+ pixel max), window exponents, implicit conv
    dX = d(X); gs = d.zeros((B * 32, 6), torch.int64)
    V.check(L.vela_gn_stats(None, P(dX), B, T, C, 32, 100000, P(gs)))
    Y, pm = d.empty((B, T, C), torch.int32, 0x5A), d.empty((B * T,), torch.int32, 0x5A)
    V.check(L.vela_gn_apply_row(None, P(dX), B, T, C, 32, P(gs), P(d(gam)), P(d(beta)), P(d(sig)), P(Y), P(pm), None, None, None, 0))
    e = d.empty((B * T,), torch.int32, 0x5A)
    V.check(L.vela_conv_e(None, P(pm), B, Hh, Hh, 1, P(e)))
    out = d.empty((B * T, N), torch.int32, 0x5A)
    a = abi.ASrc(); a.src = abi.SRC_CONV32; a.img = A(Y); a.H = Hh; a.W = Hh; a.C = C; a.stride = 1; a.Ho = Hh; a.Wo = Hh; a.K = K; a.e = A(e)
    E = abi.AEpi(); E.epi = abi.EPI_PLAIN; E.Y = A(out); E.ldy = N
    V.check(L.vela_gemm_w8a16(None, ctypes.byref(a), B * T, B * T, P(d(W)), K, N, N, K, P(d(cst)), ctypes.byref(E)))
    torch.cuda.synchronize()
    assert L.vela_device_error(1) == 0
    # ---- oracle, step by step
    egs = O.gn_stats(X, B, T, C, 32, 100000)
    got = H(gs)
    assert np.array_equal(got[:, [0, 1, 2, 4, 5]], egs[:, [0, 1, 2, 4, 5]]), "GroupNorm statistics records"
    assert np.array_equal(np.ascontiguousarray(got[:, 3]).view(np.int32)[0::2], np.ascontiguousarray(egs[:, 3]).view(np.int32)[0::2]), "GroupNorm exponents"
    eY, epm = O.gn_apply_row(X, B, T, C, 32, egs, gam, beta, sig)
    assert np.array_equal(H(Y).reshape(B * T, C), eY), "GroupNorm + SiLU output"
    assert np.array_equal(H(pm).view(np.uint32), epm), "pixel maxima"
    ee = O.conv_e(epm, B, Hh, Hh, 1)
    assert np.array_equal(H(e), ee), "3x3 window exponents"
    hi, lo, e_im = O.im2col3(eY, epm, B, Hh, Hh, C, 1, K, B * T)
    assert np.array_equal(e_im, ee)
    eo = np.zeros((B * T, N), np.int32)
    O.gemm_hl(hi, lo, B * T, W, N, K, cst, e_im, O.EPI_PLAIN, Y=eo, ldy=N)
    assert np.array_equal(H(out), eo), "implicit convolution output"
