"""Memory-bound operators on the B200 through the C ABI vs the reference's own outputs (tests/golden/):
row quantisation, pixel max, im2col + conv exponent, GroupNorm stats / apply, LayerNorm,
noise / finalize, concat / upsample / LUT activations, attention operand quantisers.  Bit-exact."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")
if not torch.cuda.is_available():
    pytest.skip("no CUDA device", allow_module_level=True)

import vela_b200 as V  # noqa: E402
from tests.gpu_util import Dev, P, H  # noqa: E402

L = None


def lib():
    global L
    if L is None:
        L = V.lib()
    return L


def ok(rc):
    V.check(rc)
    torch.cuda.synchronize()


def test_quant_rows(golden):
    g = golden("quant_rows"); d = Dev()
    for mode in range(3):
        X = g[f"X{mode}"]; M, K = X.shape; Kp, Mp = 336, 96
        hi, lo, e = d.empty((Mp, Kp), torch.int8, 0x5A), d.empty((Mp, Kp), torch.int8, 0x5A), d.empty((Mp,), torch.int32, 0x5A)
        ok(lib().vela_quant_rows(None, P(d(X)), M, K, K, P(hi), P(lo), P(e), Kp))
        assert np.array_equal(H(hi), g[f"hi{mode}"]) and np.array_equal(H(lo), g[f"lo{mode}"]) and np.array_equal(H(e)[:M], g[f"e{mode}"])


def test_quant_rows_with_known_maxima(golden):
    """vela_quant_rows_rm (the engine's form: row maxima from the producer) equals vela_quant_rows on the golden rows,
    padding rows [M, Mpad) included"""
    g = golden("quant_rows"); d = Dev()
    for mode in range(3):
        X = g[f"X{mode}"]; M, K = X.shape; Kp, Mp = 336, 96
        rm = np.zeros(Mp, np.uint32); rm[:M] = np.abs(X.astype(np.int64)).max(1)
        hi, lo, e = d.empty((Mp, Kp), torch.int8, 0x5A), d.empty((Mp, Kp), torch.int8, 0x5A), d.empty((Mp,), torch.int32, 0x5A)
        ok(lib().vela_quant_rows_rm(None, P(d(X)), P(d(rm.view(np.int32))), M, K, K, P(hi), P(lo), P(e), Kp, Mp))
        assert np.array_equal(H(hi), g[f"hi{mode}"]) and np.array_equal(H(lo), g[f"lo{mode}"]) and np.array_equal(H(e)[:M], g[f"e{mode}"])
        assert (H(e)[M:] == 0).all()


def test_im2col_pixmax_conv_e(golden):
    g = golden("im2col"); d = Dev()
    i = 0
    while f"c{i}_meta" in g:
        B, Hh, W, C, stride, Kp, Mp = [int(v) for v in g[f"c{i}_meta"]]
        rows = B * ((Hh - 1) // stride + 1) * ((W - 1) // stride + 1)
        dX = d(g[f"c{i}_X"]); pm = d.empty((B * Hh * W,), torch.int32, 0x5A)
        ok(lib().vela_pixmax(None, P(dX), B * Hh * W, C, P(pm)))
        assert np.array_equal(H(pm), g[f"c{i}_pm"])
        hi, lo, e = d.empty((Mp, Kp), torch.int8, 0x5A), d.empty((Mp, Kp), torch.int8, 0x5A), d.empty((Mp,), torch.int32, 0x5A)
        ok(lib().vela_im2col3(None, P(dX), P(pm), B, Hh, W, C, stride, P(hi), P(lo), P(e), Kp))
        assert np.array_equal(H(hi), g[f"c{i}_hi"]) and np.array_equal(H(lo), g[f"c{i}_lo"]) and np.array_equal(H(e)[:rows], g[f"c{i}_e"]), i
        e2 = d.empty((rows,), torch.int32, 0x5A)
        ok(lib().vela_conv_e(None, P(pm), B, Hh, W, stride, P(e2)))
        assert np.array_equal(H(e2), g[f"c{i}_conv_e"])
        i += 1


def test_groupnorm(golden):
    g = golden("norms"); d = Dev()
    for i in range(3):
        X = g[f"gn{i}_X"]; B, T, C = X.shape
        dX = d(X); gs = d.zeros((B * 32, 6), torch.int64)
        ok(lib().vela_gn_stats(None, P(dX), B, T, C, 32, 100000, P(gs)))
        ref, got = g[f"gn{i}_stats"], H(gs)
        assert np.array_equal(got[:, [0, 1, 2, 4, 5]], ref[:, [0, 1, 2, 4, 5]])
        assert np.array_equal(np.ascontiguousarray(got[:, 3]).view(np.int32)[0::2], np.ascontiguousarray(ref[:, 3]).view(np.int32)[0::2])
        dg, db, dsig = d(g[f"gn{i}_g"]), d(g[f"gn{i}_beta"]), d(g["sig"])
        Y, pm = d.empty((B, T, C), torch.int32, 0x5A), d.empty((B * T,), torch.int32, 0x5A)
        ok(lib().vela_gn_apply_row(None, P(dX), B, T, C, 32, P(gs), P(dg), P(db), P(dsig), P(Y), P(pm), None, None, None, 0))
        assert np.array_equal(H(Y), g[f"gn{i}_Y"]) and np.array_equal(H(pm), g[f"gn{i}_pm"])
        hi, lo, e = d.empty((B * T, C), torch.int8, 0x5A), d.empty((B * T, C), torch.int8, 0x5A), d.empty((B * T,), torch.int32, 0x5A)
        ok(lib().vela_gn_apply_row(None, P(dX), B, T, C, 32, P(gs), P(dg), P(db), None, None, None, P(hi), P(lo), P(e), C))
        assert np.array_equal(H(hi), g[f"gn{i}_hi"]) and np.array_equal(H(lo), g[f"gn{i}_lo"]) and np.array_equal(H(e), g[f"gn{i}_e"])


def test_layernorm(golden):
    g = golden("norms"); d = Dev()
    j = 0
    while f"ln{j}_X" in g:
        X = g[f"ln{j}_X"]; M, C = X.shape; Kp = (C + 15) // 16 * 16
        hi, lo, e = d.empty((M, Kp), torch.int8, 0x5A), d.empty((M, Kp), torch.int8, 0x5A), d.empty((M,), torch.int32, 0x5A)
        ok(lib().vela_lnorm_q(None, P(d(X)), M, C, P(d(g[f"ln{j}_g"])), P(d(g[f"ln{j}_beta"])), 100000, P(hi), P(lo), P(e), Kp))
        assert np.array_equal(H(hi), g[f"ln{j}_hi"]) and np.array_equal(H(lo), g[f"ln{j}_lo"]) and np.array_equal(H(e), g[f"ln{j}_e"]), (j, C)
        j += 1
    X = g["lnf_X"]; M, C = X.shape
    Y = d.empty((M, C), torch.int32, 0x5A)
    ok(lib().vela_lnorm(None, P(d(X)), M, C, P(d(g["lnf_g"])), P(d(g["lnf_beta"])), 100000, P(Y)))
    assert np.array_equal(H(Y), g["lnf_Y"])


def test_noise_finalize_elementwise(golden):
    g = golden("misc"); d = Dev()
    seeds = g["seeds"]; B = seeds.shape[0]
    n, x = d.empty((B, 16384), torch.int32, 0x5A), d.empty((B, 16384), torch.int32, 0x5A)
    ok(lib().vela_noise(None, P(d(seeds)), B, P(d(g["gauss"])), 73343000, P(n), P(x)))
    assert np.array_equal(H(n), g["noise_n"]) and np.array_equal(H(x), g["noise_x"])
    out = d.empty((B, 32768), torch.uint8, 0x5A)
    ok(lib().vela_finalize(None, P(n), P(d(g["eps"])), B, 957800, P(out)))
    assert np.array_equal(H(out), g["x0"])
    cat = d.empty((15, 96), torch.int32, 0x5A)
    ok(lib().vela_concat(None, P(d(g["cat_A"])), 64, P(d(g["cat_B"])), 32, 15, P(cat)))
    assert np.array_equal(H(cat), g["cat"])
    up = d.empty((2, 6, 8, 16), torch.int32, 0x5A)
    ok(lib().vela_upsample2(None, P(d(g["up_X"])), 2, 3, 4, 16, P(up)))
    assert np.array_equal(H(up), g["up"])
    a = d(g["act_X"])
    ok(lib().vela_act(None, P(a), 4096, P(d(g["sig"]))))
    assert np.array_equal(H(a), g["act"])
    a = d(g["geglu_A"])
    ok(lib().vela_geglu(None, P(a), P(d(g["geglu_G"])), 4096, P(d(g["phi"]))))
    assert np.array_equal(H(a), g["geglu"])


def test_attention_operands(golden):
    g = golden("attention"); d = Dev()
    i = 0
    while f"a{i}_meta" in g:
        B, heads, Tq, Tk, causal, Tqp, Tkp = [int(v) for v in g[f"a{i}_meta"]]
        C, G = 64 * heads, B * heads
        for nm, X, T, Tp in (("q", g[f"a{i}_Q"], Tq, Tqp), ("k", g[f"a{i}_K"], Tk, Tkp)):
            bufs = [d.empty((G, Tp, 64), torch.int8, 0x5A), d.empty((G, Tp, 64), torch.int8, 0x5A), d.empty((G, Tp), torch.int32, 0x5A)] + \
                   [d.empty((G, Tp), torch.int64, 0x5A) for _ in range(3)]
            ok(lib().vela_quant_heads(None, P(d(X)), B, T, C, heads, Tp, *[P(b) for b in bufs]))
            for b, f in zip(bufs, ("hi", "lo", "e", "hs", "ls", "ts")):
                assert np.array_equal(H(b), g[f"a{i}_{nm}{f}"]), (i, nm, f)
        vh, vl = d.empty((G, 64, Tkp), torch.int8, 0x5A), d.empty((G, 64, Tkp), torch.int8, 0x5A)
        ev, vs, scr = d.empty((G, 64), torch.int32, 0x5A), d.empty((G, 64), torch.int64, 0x5A), d.empty((G, 64), torch.int32, 0x5A)
        ok(lib().vela_quant_v(None, P(d(g[f"a{i}_V"])), B, Tk, C, heads, Tkp, P(vh), P(vl), P(ev), P(vs), P(scr)))
        for b, f in zip((vh, vl, ev, vs), ("vhi", "vlo", "ev", "vsum")):
            assert np.array_equal(H(b), g[f"a{i}_{f}"]), (i, f)
        i += 1


def test_quant_heads_pad():
    d = Dev(); G, T, Tp = 3, 70, 128
    bufs = [d.empty((G, Tp, 64), torch.int8, 0x5A), d.empty((G, Tp, 64), torch.int8, 0x5A), d.empty((G, Tp), torch.int32, 0x5A)] + \
           [d.empty((G, Tp), torch.int64, 0x5A) for _ in range(3)]
    ok(lib().vela_quant_heads_pad(None, G, T, Tp, *[P(b) for b in bufs]))
    hi, lo, e, hs, ls, ts = [H(b) for b in bufs]
    assert (hi[:, T:] == 0).all() and (lo[:, T:] == -128).all() and (e[:, T:] == 0).all()
    assert (hs[:, T:] == 0).all() and (ls[:, T:] == -8192).all() and (ts[:, T:] == 0).all()
    assert (hi[:, :T].view(np.uint8) == 0x5A).all()      # rows below T untouched
