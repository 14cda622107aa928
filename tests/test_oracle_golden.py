"""Pin the CPU oracle (oracle/vela_oracle.c) to the REFERENCE implementation.

Every fixture under tests/golden/ was produced by the reference's own kernels
and engine on a B200 (tests/golden/make_golden.py via oracle/_ref).  The
oracle must reproduce every output byte on the same inputs.
"""
import hashlib
import json
import os

import numpy as np
import pytest

from oracle import pyoracle as O

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def test_quant_rows(golden):
    g = golden("quant_rows")
    for mode in range(3):
        X = g[f"X{mode}"]
        hi, lo, e = O.quant_rows(X, 336, 96)
        assert np.array_equal(hi, g[f"hi{mode}"]) and np.array_equal(lo, g[f"lo{mode}"])
        assert np.array_equal(e, g[f"e{mode}"])


def test_gemm_epilogues(golden):
    g = golden("gemm")
    Mreal, Nreal, Kp = 200, 192, 336
    Ahi, Alo, W, cst, e = g["Ahi"], g["Alo"], g["W"], g["cst"], g["e"]
    Y = np.zeros((Mreal, Nreal), np.int32); rm = np.zeros(Mreal, np.uint32)
    O.gemm_hl(Ahi, Alo, Mreal, W, Nreal, Kp, cst, e, O.EPI_PLAIN, Y=Y, ldy=Nreal, residual=g["R"], rowmax=rm)
    assert np.array_equal(Y, g["Y_plain"]) and np.array_equal(rm, g["rm_plain"].view(np.uint32))
    Y = np.zeros((Mreal, Nreal // 2), np.int32); rm = np.zeros(Mreal, np.uint32)
    O.gemm_hl(Ahi, Alo, Mreal, W, Nreal, Kp, cst, e, O.EPI_GEGLU, Y=Y, ldy=Nreal // 2, Lphi=g["phi"], rowmax=rm)
    assert np.array_equal(Y, g["Y_geglu"]) and np.array_equal(rm, g["rm_geglu"].view(np.uint32))
    Y = np.zeros((Mreal, Nreal), np.int32)
    O.gemm_hl(Ahi, Alo, Mreal, W, Nreal, Kp, cst, e, O.EPI_GELU, Y=Y, ldy=Nreal, Lphi=g["phi"])
    assert np.array_equal(Y, g["Y_gelu"])
    Ys = [np.zeros((Mreal, 64), np.int32) for _ in range(3)]
    O.gemm_hl(Ahi, Alo, Mreal, W, Nreal, Kp, cst, e, O.EPI_SPLIT3, Y=Ys[0], ldy=64, Cs=64, Y1=Ys[1], Y2=Ys[2])
    for i in range(3):
        assert np.array_equal(Ys[i], g[f"Y_split{i}"])


def test_gemm_qkv(golden):
    g = golden("gemm")
    C, heads, T, B, Tp = 128, 2, 100, 2, 128
    G = B * heads
    bufs = {}
    for p in ("q", "k"):
        bufs[p + "hi"] = np.zeros((G, Tp, 64), np.int8); bufs[p + "lo"] = np.full((G, Tp, 64), -128, np.int8)
        bufs[p + "e"] = np.zeros((G, Tp), np.int32); bufs[p + "hs"] = np.zeros((G, Tp), np.int64)
        bufs[p + "ls"] = np.full((G, Tp), -8192, np.int64); bufs[p + "ts"] = np.zeros((G, Tp), np.int64)
    V = np.zeros((200, C), np.int32)
    qkv = dict(heads=heads, T=T, TpQ=Tp, TpK=Tp, C=C, qhi=bufs["qhi"], qlo=bufs["qlo"], khi=bufs["khi"], klo=bufs["klo"], qe=bufs["qe"], ke=bufs["ke"],
               qhs=bufs["qhs"], qls=bufs["qls"], qts=bufs["qts"], khs=bufs["khs"], kls=bufs["kls"], kts=bufs["kts"])
    O.gemm_hl(g["Ahi"], g["Alo"], 200, g["Wq"], 3 * C, 336, g["cq"], g["e"], O.EPI_QKV, Y2=V, qkv=qkv)
    assert np.array_equal(V, g["qkv_V"])
    for p in ("q", "k"):
        for f in ("hi", "lo", "e", "hs", "ls", "ts"):
            assert np.array_equal(bufs[p + f], g[f"qkv_{p}{f}"]), p + f


def test_gemm_sources(golden):
    g = golden("gemm_sources")
    X = g["x32_X"]; rows, K = X.shape; N = 128
    hi, lo, e = O.quant_rows(X, K, rows)
    Y = np.zeros((rows, N), np.int32); rm = np.zeros(rows, np.uint32)
    O.gemm_hl(hi, lo, rows, g["x32_W"], N, K, g["x32_cst"], e, O.EPI_PLAIN, Y=Y, ldy=N, residual=g["x32_R"], rowmax=rm)
    assert np.array_equal(Y, g["x32_Y"]) and np.array_equal(rm, g["x32_rm"].view(np.uint32))
    Xc = g["conv_X"]; B, H, W, C = Xc.shape; N = 64
    pm = O.pixmax(Xc, B * H * W, C)
    assert np.array_equal(pm, g["conv_pm"].view(np.uint32))
    for stride in (1, 2):
        Ho = (H - 1) // stride + 1; rows = B * Ho * Ho
        hi, lo, e = O.im2col3(Xc, pm, B, H, W, C, stride, 9 * C, rows)
        assert np.array_equal(e, g[f"conv{stride}_e"])
        Y = np.zeros((rows, N), np.int32)
        O.gemm_hl(hi, lo, rows, g["conv_W"], N, 9 * C, g["conv_cst"], e, O.EPI_PLAIN, Y=Y, ldy=N)
        assert np.array_equal(Y, g[f"conv{stride}_Y"])
        if stride == 1:
            assert np.array_equal(Y, g["lt_Y"])      # the reference's cuBLASLt deep-K path agrees


def test_im2col(golden):
    g = golden("im2col")
    i = 0
    while f"c{i}_meta" in g:
        B, H, W, C, stride, Kp, Mp = [int(v) for v in g[f"c{i}_meta"]]
        X = g[f"c{i}_X"]
        pm = O.pixmax(X, B * H * W, C)
        assert np.array_equal(pm, g[f"c{i}_pm"].view(np.uint32))
        hi, lo, e = O.im2col3(X, pm, B, H, W, C, stride, Kp, Mp)
        assert np.array_equal(hi, g[f"c{i}_hi"]) and np.array_equal(lo, g[f"c{i}_lo"]) and np.array_equal(e, g[f"c{i}_e"]), i
        assert np.array_equal(O.conv_e(pm, B, H, W, stride), g[f"c{i}_conv_e"])
        i += 1
    assert i == 18


def test_groupnorm(golden):
    g = golden("norms")
    for i in range(3):
        X = g[f"gn{i}_X"]; B, T, C = X.shape
        gs = O.gn_stats(X, B, T, C, 32, 100000)
        ref = g[f"gn{i}_stats"]
        # fields: sum | mn,mx | mean | e,(pad) | ss | sd
        assert np.array_equal(gs[:, [0, 1, 2, 4, 5]], ref[:, [0, 1, 2, 4, 5]])
        assert np.array_equal(np.ascontiguousarray(gs[:, 3]).view(np.int32)[0::2], np.ascontiguousarray(ref[:, 3]).view(np.int32)[0::2])
        Y, pm = O.gn_apply_row(X, B, T, C, 32, gs, g[f"gn{i}_g"], g[f"gn{i}_beta"], Lsig=g["sig"])
        assert np.array_equal(Y.reshape(B, T, C), g[f"gn{i}_Y"]) and np.array_equal(pm, g[f"gn{i}_pm"].view(np.uint32))
        hi, lo, e = O.gn_apply_row(X, B, T, C, 32, gs, g[f"gn{i}_g"], g[f"gn{i}_beta"], quant=True, Kp=C)
        assert np.array_equal(hi, g[f"gn{i}_hi"]) and np.array_equal(lo, g[f"gn{i}_lo"]) and np.array_equal(e, g[f"gn{i}_e"])


def test_layernorm(golden):
    g = golden("norms")
    j = 0
    while f"ln{j}_X" in g:
        X = g[f"ln{j}_X"]; M, C = X.shape; Kp = (C + 15) // 16 * 16
        hi, lo, e = O.lnorm_q(X, g[f"ln{j}_g"], g[f"ln{j}_beta"], 100000, Kp)
        assert np.array_equal(hi, g[f"ln{j}_hi"]) and np.array_equal(lo, g[f"ln{j}_lo"]) and np.array_equal(e, g[f"ln{j}_e"]), j
        j += 1
    assert j == 24
    Y = O.lnorm(g["lnf_X"], g["lnf_g"].astype(np.int32), g["lnf_beta"].astype(np.int32), 100000)
    assert np.array_equal(Y, g["lnf_Y"])


def test_noise_finalize_elementwise(golden):
    g = golden("misc")
    n, x = O.noise(g["seeds"], g["gauss"].astype(np.int32), 73343000)
    assert np.array_equal(n, g["noise_n"]) and np.array_equal(x, g["noise_x"])
    assert np.array_equal(O.finalize(n, g["eps"], 957800), g["x0"])
    A, Bm = g["cat_A"], g["cat_B"]
    cat = np.concatenate([A.reshape(15, 64), Bm.reshape(15, 32)], 1)
    assert np.array_equal(cat, g["cat"])
    U = g["up_X"]
    assert np.array_equal(U.repeat(2, 1).repeat(2, 2), g["up"])
    sig, phi, G = g["sig"], g["phi"], g["geglu_G"]
    a = g["act_X"].copy(); O.lib().or_act(O.ptr(a), a.size, O.ptr(sig))
    assert np.array_equal(a, g["act"])
    a = g["geglu_A"].copy(); O.lib().or_geglu(O.ptr(a), O.ptr(G), a.size, O.ptr(phi))
    assert np.array_equal(a, g["geglu"])
    O.unpin()


def test_attention(golden):
    g = golden("attention")
    i = 0
    while f"a{i}_meta" in g:
        B, heads, Tq, Tk, causal, Tqp, Tkp = [int(v) for v in g[f"a{i}_meta"]]
        C = 64 * heads
        q = O.quant_heads(g[f"a{i}_Q"], B, Tq, C, heads, Tqp)
        k = O.quant_heads(g[f"a{i}_K"], B, Tk, C, heads, Tkp)
        for j, f in enumerate(("hi", "lo", "e", "hs", "ls", "ts")):
            assert np.array_equal(q[j], g[f"a{i}_q{f}"]), (i, "q" + f)
            assert np.array_equal(k[j], g[f"a{i}_k{f}"]), (i, "k" + f)
        v = O.quant_v(g[f"a{i}_V"], B, Tk, C, heads, Tkp)
        for j, f in enumerate(("vhi", "vlo", "ev", "vsum")):
            assert np.array_equal(v[j], g[f"a{i}_{f}"]), (i, f)
        out, rm = O.attention(q[0], q[1], q[2], k[0], k[1], k[2], v[0], v[1], v[2], B, heads, Tq, Tk, causal, g["lexp"])
        assert np.array_equal(out, g[f"a{i}_out"]), i
        assert np.array_equal(rm, g[f"a{i}_rm"].view(np.uint32)), i
        i += 1
    assert i == 6


@pytest.mark.slow
def test_unet_step_matches_reference_engine(tmp_path):
    """The oracle's whole UNet step == the reference engine's on the synthetic model (seed 1):
    the prompt context, every block output (sha256) and the x0 bytes."""
    from vela_b200 import synth_model_write
    path = str(tmp_path / "synth.poisd")
    synth_model_write(path, 1)
    e = np.load(os.path.join(GOLDEN, "engine.npz"))
    taps = json.load(open(os.path.join(GOLDEN, "engine_taps.json")))
    m = O.Model(path)
    m.set_prompt([320, 736, 3240])
    assert np.array_equal(m.context(), e["ctx"])
    got = {}
    x0, _ = m.step(e["seeds"], taps=lambda name, a: got.__setitem__(name, hashlib.sha256(a.tobytes()).hexdigest()))
    assert list(got) == list(taps)
    bad = [k for k in taps if got[k] != taps[k]]
    assert not bad, bad
    assert np.array_equal(x0, e["x0"]) and np.array_equal(x0, e["x0_graph"])
    m.close()
