"""Generate the golden fixtures of tests/golden/ from the REFERENCE implementation.

Runs on a B200: calls the reference's own kernels and engine, compiled from the
reference sources into oracle/_ref/libvela_ref.so (see oracle/Makefile and
oracle/ref_harness.cu), on seeded inputs, and stores inputs + outputs as .npz.
The cases mirror the reference's own tests (src/test_gemm_hl.cu,
src/test_im2col.cu, src/test_normalization.cpp, Engine::testAttention) at
sizes the CPU oracle finishes in seconds.  tests/test_oracle_golden.py then
pins the oracle (oracle/vela_oracle.c) to these outputs on the CPU.

usage:  python tests/golden/make_golden.py OUTDIR [--model PATH] [--bench]
"""
import argparse
import ctypes
import hashlib
import json
import os
import sys
import time

import numpy as np
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
R = ctypes.CDLL(os.path.join(ROOT, "oracle", "_ref", "libvela_ref.so"))
R.ref_last_error.restype = ctypes.c_char_p
R.ref_open.restype = ctypes.c_void_p
R.ref_open.argtypes = [ctypes.c_char_p, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int]
for f in ("ref_set_prompt", "ref_run", "ref_submit", "ref_collect", "ref_bench", "ref_context", "ref_unet_taps"):
    getattr(R, f).argtypes = None
R.ref_close.argtypes = [ctypes.c_void_p]
LL = ctypes.c_longlong
V = ctypes.c_void_p


_KEEP = []   # device copies stay referenced until the case ends: a temporary freed inside an argument list
             # could hand its memory to the next temporary before the kernel reads it


def D(a):
    t = torch.from_numpy(np.ascontiguousarray(a)).cuda()
    _KEEP.append(t)
    return t


def P(t):
    return V(t.data_ptr()) if t is not None else V(0)


def H(t):
    torch.cuda.synchronize()
    return t.cpu().numpy()


def ck(rc):
    if rc != 0:
        raise RuntimeError(R.ref_last_error().decode())


def sentinel(shape, dtype):
    t = torch.empty(shape, dtype=dtype, device="cuda")
    t.view(torch.uint8).fill_(0x5A)
    return t


def rbits(rng, shape, maxbits=31):
    """values of random bit-width 1..maxbits (the distribution of src/test_gemm_hl.cu:16 / src/engine.cu:578-581)"""
    bits = rng.integers(1, maxbits + 1, size=shape).astype(np.int64)
    x = rng.integers(0, 2**62, size=shape, dtype=np.int64)
    return ((x & ((np.int64(1) << bits) - 1)) - (np.int64(1) << (bits - 1))).astype(np.int32)


def cst_for(rng, W, N, Np, K):
    """per-column {m, s, b, wsum} in the ranges of src/test_gemm_hl.cu:63"""
    c = np.zeros((Np, 4), np.int32)
    c[:N, 0] = rng.integers(16384, 32768, N)
    c[:N, 1] = rng.integers(20, 30, N)
    c[:N, 2] = rng.integers(-50000, 50000, N)
    c[:N, 3] = W[:N, :].astype(np.int64).sum(1)
    return c


def luts():
    x = (np.arange(2049) - 1024) / 64.0
    sig = np.rint(65536.0 / (1.0 + np.exp(-x))).astype(np.int32)
    from math import erfc, sqrt
    phi = np.array([round(65536.0 * 0.5 * erfc(-v / sqrt(2.0))) for v in x], np.int32)
    ex = np.rint(1073741824.0 * np.exp(-np.arange(1025) / 64.0)).astype(np.int32)
    return sig, phi, ex


def case_quant_rows(out, rng):
    M, K, Kp = 70, 332, 336
    res = {}
    for mode in range(3):
        X = np.zeros((M, K), np.int32) if mode == 0 else (rng.integers(-1000000, 1000001, (M, K)).astype(np.int32) if mode == 1 else rng.integers(-2**31, 2**31, (M, K), dtype=np.int64).astype(np.int32))
        if mode == 2:
            X[0, 0], X[1, 1] = -2**31, 2**31 - 1
        Mp = (M + 31) // 32 * 32
        hi, lo, e = sentinel((Mp, Kp), torch.int8), sentinel((Mp, Kp), torch.int8), sentinel((Mp,), torch.int32)
        ck(R.ref_quant_rows(P(D(X)), M, K, K, P(hi), P(lo), P(e), Kp))
        res.update({f"X{mode}": X, f"hi{mode}": H(hi), f"lo{mode}": H(lo), f"e{mode}": H(e)[:M]})
    np.savez_compressed(os.path.join(out, "quant_rows.npz"), **res)


def case_gemm(out, rng):
    sig, phi, _ = luts()
    Mreal, Mp, Nreal, Np, K, Kp = 200, 256, 192, 192, 330, 336
    Ahi = rng.integers(-128, 128, (Mp, Kp), dtype=np.int64).astype(np.int8)
    Alo = rng.integers(-128, 128, (Mp, Kp), dtype=np.int64).astype(np.int8)
    W = np.zeros((Np, Kp), np.int8)
    W[:Nreal, :K] = rng.integers(-128, 128, (Nreal, K))
    cst = cst_for(rng, W, Nreal, Np, K)
    e = rng.integers(0, 12, Mp).astype(np.int32)
    Rs = rng.integers(-2**31, 2**31, (Mreal, Nreal), dtype=np.int64).astype(np.int32)
    res = dict(Ahi=Ahi, Alo=Alo, W=W, cst=cst, e=e, R=Rs, phi=phi)
    dA, dB, dW, dc, de = D(Ahi), D(Alo), D(W), D(cst), D(e)
    Lphi = D(phi)
    # EPI_PLAIN + residual + rowmax
    Y = sentinel((Mreal, Nreal), torch.int32); rm = torch.zeros(Mp, dtype=torch.int32, device="cuda")
    ck(R.ref_gemm_hl(P(dA), P(dB), Kp, Mp, Mreal, P(dW), Kp, Np, Nreal, Kp, P(dc), P(de), P(Y), Nreal, P(D(Rs)), 0, 0, V(0), V(0), V(0), P(rm)))
    res.update(Y_plain=H(Y), rm_plain=H(rm)[:Mreal])
    # EPI_GEGLU (interleaved a|g) + rowmax
    Y = sentinel((Mreal, Nreal // 2), torch.int32); rm = torch.zeros(Mp, dtype=torch.int32, device="cuda")
    ck(R.ref_gemm_hl(P(dA), P(dB), Kp, Mp, Mreal, P(dW), Kp, Np, Nreal, Kp, P(dc), P(de), P(Y), Nreal // 2, V(0), 2, 0, V(0), V(0), P(Lphi), P(rm)))
    res.update(Y_geglu=H(Y), rm_geglu=H(rm)[:Mreal])
    # EPI_GELU
    Y = sentinel((Mreal, Nreal), torch.int32)
    ck(R.ref_gemm_hl(P(dA), P(dB), Kp, Mp, Mreal, P(dW), Kp, Np, Nreal, Kp, P(dc), P(de), P(Y), Nreal, V(0), 3, 0, V(0), V(0), P(Lphi), V(0)))
    res.update(Y_gelu=H(Y))
    # EPI_SPLIT3 (Cs = 64)
    Ys = [sentinel((Mreal, 64), torch.int32) for _ in range(3)]
    ck(R.ref_gemm_hl(P(dA), P(dB), Kp, Mp, Mreal, P(dW), Kp, Np, Nreal, Kp, P(dc), P(de), P(Ys[0]), 64, V(0), 1, 64, P(Ys[1]), P(Ys[2]), V(0), V(0)))
    res.update(Y_split0=H(Ys[0]), Y_split1=H(Ys[1]), Y_split2=H(Ys[2]))
    # EPI_QKV: C = 128 (2 heads), N = 384, B = 2, T = 100
    C, heads, T, Bq = 128, 2, 100, 2
    Wq = np.zeros((3 * C, Kp), np.int8); Wq[:, :K] = rng.integers(-128, 128, (3 * C, K))
    cq = cst_for(rng, Wq, 3 * C, 3 * C, K)
    TpQ, TpK, G = 128, 128, Bq * heads
    bufs = {}
    for nm, Tp in (("q", TpQ), ("k", TpK)):
        bufs[nm] = [sentinel((G, Tp, 64), torch.int8), sentinel((G, Tp, 64), torch.int8), sentinel((G, Tp), torch.int32)] + [sentinel((G, Tp), torch.int64) for _ in range(3)]
    Vt = sentinel((Mreal, C), torch.int32)
    ck(R.ref_gemm_qkv(P(dA), P(dB), Kp, P(de), Mp, Mreal, P(D(Wq)), Kp, 3 * C, 3 * C, Kp, P(D(cq)), heads, T, TpQ, TpK, C,
                      *[P(t) for t in bufs["q"]], *[P(t) for t in bufs["k"]], P(Vt)))
    res.update(Wq=Wq, cq=cq, qkv_V=H(Vt))
    for nm in ("q", "k"):
        for i, field in enumerate(("hi", "lo", "e", "hs", "ls", "ts")):
            res[f"qkv_{nm}{field}"] = H(bufs[nm][i])
    np.savez_compressed(os.path.join(out, "gemm.npz"), **res)


def case_gemm_sources(out, rng):
    res = {}
    # SRC_X32: rows 150, K 320, N 128
    rows, K, N = 150, 320, 128
    Mp, Kp, Np = 192, 320, 128
    X = rbits(rng, (rows, K))
    W = np.zeros((Np, Kp), np.int8); W[:N, :K] = rng.integers(-128, 128, (N, K))
    cst = cst_for(rng, W, N, Np, K)
    rmx = np.zeros(Mp, np.uint32); rmx[:rows] = np.abs(X.astype(np.int64)).max(1).astype(np.uint32)
    Y = sentinel((rows, N), torch.int32); rmo = torch.zeros(Mp, dtype=torch.int32, device="cuda")
    Rs = rbits(rng, (rows, N), 30)
    ck(R.ref_gemm_x32(P(D(X)), K, P(D(rmx.view(np.int32))), K, Mp, rows, P(D(W)), Kp, Np, N, Kp, P(D(cst)), P(Y), N, P(D(Rs)), 0, V(0), P(rmo)))
    res.update(x32_X=X, x32_W=W, x32_cst=cst, x32_R=Rs, x32_Y=H(Y), x32_rm=H(rmo)[:rows])
    # SRC_CONV32: B 2, 8x8, C 64 -> 64, stride 1 and 2; plus the deep-K cuBLASLt path on the same operand
    B, Hh, Ww, C, N = 2, 8, 8, 64, 64
    Xc = rbits(rng, (B, Hh, Ww, C))
    Wc = rng.integers(-128, 128, (N, 9 * C)).astype(np.int8)      # tap-major K order (src/engine.cu:36)
    cc = cst_for(rng, Wc, N, N, 9 * C)
    pm = torch.zeros(B * Hh * Ww, dtype=torch.int32, device="cuda")
    dX = D(Xc)
    ck(R.ref_pixmax(P(dX), B * Hh * Ww, C, P(pm)))
    res.update(conv_X=Xc, conv_W=Wc, conv_cst=cc, conv_pm=H(pm))
    for stride in (1, 2):
        Ho = (Hh - 1) // stride + 1; rows = B * Ho * Ho; Mp = (rows + 63) // 64 * 64
        e = sentinel((Mp,), torch.int32); Y = sentinel((rows, N), torch.int32)
        ck(R.ref_gemm_conv(P(dX), B, Hh, Ww, C, stride, P(pm), P(e), Mp, P(D(Wc)), 9 * C, N, N, 9 * C, P(D(cc)), P(Y), N, V(0)))
        res.update({f"conv{stride}_e": H(e)[:rows], f"conv{stride}_Y": H(Y)})
    # cuBLASLt + k_epilogue on the im2col planes (stride 1)
    rows, Mp, Kp = B * Hh * Ww, 128, 9 * C
    hl = sentinel((2 * Mp, Kp), torch.int8); e = sentinel((Mp,), torch.int32)
    ck(R.ref_im2col3(P(dX), P(pm), B, Hh, Ww, C, 1, P(hl), P(hl[Mp:]), P(e), Kp))
    Cs = torch.empty((2 * Mp, N), dtype=torch.int32, device="cuda"); Y = sentinel((rows, N), torch.int32)
    ck(R.ref_gemm_lt(P(hl), Mp, rows, P(D(Wc)), N, N, Kp, P(D(cc)), P(e), P(Cs), P(Y), N, V(0)))
    res.update(lt_Y=H(Y))
    np.savez_compressed(os.path.join(out, "gemm_sources.npz"), **res)


def case_im2col(out, rng):
    res = {}
    i = 0
    for C in (4, 16, 320):
        for stride in (1, 2):
            for mode in range(3):
                B, Hh, Ww = 2, 5, 7
                Ho, Wo = (Hh - 1) // stride + 1, (Ww - 1) // stride + 1
                rows = B * Ho * Wo; Mp = (rows + 31) // 32 * 32; Kp = (9 * C + 15) // 16 * 16
                X = np.zeros((B, Hh, Ww, C), np.int32) if mode == 0 else (rng.integers(-32768, 32769, (B, Hh, Ww, C)).astype(np.int32) if mode == 1 else rng.integers(-2**31, 2**31, (B, Hh, Ww, C), dtype=np.int64).astype(np.int32))
                if mode == 2:
                    flat = X.reshape(-1); flat[::19] = np.where(np.arange(flat[::19].size) % 2 == 1, -2**31, 2**31 - 1)
                dX = D(X); pm = torch.zeros(B * Hh * Ww, dtype=torch.int32, device="cuda")
                hi, lo, e = sentinel((Mp, Kp), torch.int8), sentinel((Mp, Kp), torch.int8), sentinel((Mp,), torch.int32)
                ck(R.ref_pixmax(P(dX), B * Hh * Ww, C, P(pm)))
                ck(R.ref_im2col3(P(dX), P(pm), B, Hh, Ww, C, stride, P(hi), P(lo), P(e), Kp))
                e2 = sentinel((rows,), torch.int32)
                ck(R.ref_conv_e(P(pm), B, Hh, Ww, stride, P(e2)))
                res.update({f"c{i}_meta": np.array([B, Hh, Ww, C, stride, Kp, Mp]), f"c{i}_X": X, f"c{i}_pm": H(pm), f"c{i}_hi": H(hi), f"c{i}_lo": H(lo), f"c{i}_e": H(e)[:rows], f"c{i}_conv_e": H(e2)})
                i += 1
    np.savez_compressed(os.path.join(out, "im2col.npz"), **res)


def case_norms(out, rng):
    sig, _, _ = luts()
    res = {"sig": sig}
    # GroupNorm: stats + apply (+SiLU, int32 + pm) and (no act, quantised), B 2, T 64, C 320 / 640
    for i, (C, mode) in enumerate(((320, 1), (640, 2), (320, 3))):
        B, T = 2, 64
        if mode == 1: X = rng.integers(-1000000, 1000001, (B, T, C)).astype(np.int32)
        elif mode == 2: X = rbits(rng, (B, T, C), 24)
        else: X = (rng.integers(-3000, 3000, (B, T, C)) * 1024 + 77).astype(np.int32)
        g = rng.integers(65536 - 16384, 65536 + 16384, C).astype(np.int32); beta = rng.integers(-8192, 8192, C).astype(np.int32)
        den = 100000
        gs = torch.zeros((B * 32, 6), dtype=torch.int64, device="cuda")
        dX = D(X)
        ck(R.ref_gn_stats(P(dX), B, T, C, 32, LL(den), P(gs)))
        Y = sentinel((B, T, C), torch.int32); pm = sentinel((B * T,), torch.int32)
        ck(R.ref_gn_apply_row(P(dX), B, T, C, 32, P(gs), P(D(g)), P(D(beta)), P(D(sig)), P(Y), P(pm), V(0), V(0), V(0), 0))
        Kp = C
        hi, lo, e = sentinel((B * T, Kp), torch.int8), sentinel((B * T, Kp), torch.int8), sentinel((B * T,), torch.int32)
        ck(R.ref_gn_apply_row(P(dX), B, T, C, 32, P(gs), P(D(g)), P(D(beta)), V(0), V(0), V(0), P(hi), P(lo), P(e), Kp))
        res.update({f"gn{i}_X": X, f"gn{i}_g": g, f"gn{i}_beta": beta, f"gn{i}_stats": H(gs), f"gn{i}_Y": H(Y), f"gn{i}_pm": H(pm),
                    f"gn{i}_hi": H(hi), f"gn{i}_lo": H(lo), f"gn{i}_e": H(e)})
    # LayerNorm with quantised output: the cases of src/test_normalization.cpp:59-66
    j = 0
    for C in (4, 12, 124, 128, 132, 320, 640, 1280):
        for mode in range(3):
            M, den = 9, 100000
            Kp = (C + 15) // 16 * 16
            X = np.zeros((M, C), np.int32) if mode == 0 else (rng.integers(-1000000, 1000001, (M, C)).astype(np.int32) if mode == 1 else rng.integers(-2**31, 2**31, (M, C), dtype=np.int64).astype(np.int32))
            if mode == 2:
                X[0, 0], X[0, 1 % C] = -2**31, 2**31 - 1
            g = (rng.integers(-2**31, 2**31, C, dtype=np.int64).astype(np.int32) if mode == 2 else np.full(C, 65536, np.int32))
            beta = (rng.integers(-2**31, 2**31, C, dtype=np.int64).astype(np.int32) if mode == 2 else np.zeros(C, np.int32))
            hi, lo, e = sentinel((M, Kp), torch.int8), sentinel((M, Kp), torch.int8), sentinel((M,), torch.int32)
            ck(R.ref_lnorm_q(P(D(X)), M, C, P(D(g)), P(D(beta)), LL(den), P(hi), P(lo), P(e), Kp))
            res.update({f"ln{j}_X": X, f"ln{j}_g": g, f"ln{j}_beta": beta, f"ln{j}_hi": H(hi), f"ln{j}_lo": H(lo), f"ln{j}_e": H(e)})
            j += 1
    # LayerNorm, int32 output (text encoder final norm)
    M, C = 9, 1024
    X = rbits(rng, (M, C), 26)
    g = rng.integers(65536 - 16384, 65536 + 16384, C).astype(np.int64); beta = rng.integers(-8192, 8192, C).astype(np.int64)
    Y = sentinel((M, C), torch.int32)
    ck(R.ref_lnorm(P(D(X)), M, C, P(D(g)), P(D(beta)), LL(100000), P(Y)))
    res.update(lnf_X=X, lnf_g=g, lnf_beta=beta, lnf_Y=H(Y))
    np.savez_compressed(os.path.join(out, "norms.npz"), **res)


def case_misc(out, rng):
    sig, phi, ex = luts()
    res = {}
    B = 3
    seeds = rng.integers(0, 256, (B, 32)).astype(np.uint8)
    gauss = rng.integers(-300000, 300000, 65536).astype(np.int64)
    cin, sg = 73343000, 957800
    n, x = sentinel((B, 16384), torch.int32), sentinel((B, 16384), torch.int32)
    ck(R.ref_noise(P(D(seeds)), B, P(D(gauss)), LL(cin), P(n), P(x)))
    eps = rbits(rng, (B, 16384), 21)
    out8 = sentinel((B, 32768), torch.uint8)
    ck(R.ref_finalize(P(n), P(D(eps)), B, LL(sg), P(out8)))
    res.update(seeds=seeds, gauss=gauss, noise_n=H(n), noise_x=H(x), eps=eps, x0=H(out8))
    # elementwise
    A = rbits(rng, (3, 5, 64), 30); Bm = rbits(rng, (3, 5, 32), 30)
    cat = sentinel((15, 96), torch.int32)
    ck(R.ref_concat(P(D(A)), 64, P(D(Bm)), 32, 15, P(cat)))
    U = rbits(rng, (2, 3, 4, 16), 30); up = sentinel((2, 6, 8, 16), torch.int32)
    ck(R.ref_upsample2(P(D(U)), 2, 3, 4, 16, P(up)))
    Xa = rbits(rng, (4096,), 24); ta = D(Xa)
    ck(R.ref_act(P(ta), ctypes.c_size_t(4096), P(D(sig))))
    Ga = rbits(rng, (4096,), 24); Xg = rbits(rng, (4096,), 24); tg = D(Xg)
    ck(R.ref_geglu(P(tg), P(D(Ga)), ctypes.c_size_t(4096), P(D(phi))))
    res.update(cat_A=A, cat_B=Bm, cat=H(cat), up_X=U, up=H(up), act_X=Xa, act=H(ta), geglu_A=Xg, geglu_G=Ga, geglu=H(tg), sig=sig, phi=phi)
    np.savez_compressed(os.path.join(out, "misc.npz"), **res)


def case_attention(out, rng):
    _, _, ex = luts()
    res = {"lexp": ex}
    cases = [  # (B, heads, Tq, Tk, causal, maxbits)  -- the fused 3-pass kernel, the small kernel, causal text-encoder shape
        (1, 2, 256, 256, 0, 31), (1, 2, 256, 256, 0, 8), (2, 1, 256, 77, 0, 31), (1, 2, 77, 77, 1, 31), (1, 1, 1024, 1024, 0, 20), (1, 2, 200, 180, 0, 24)]
    for i, (B, heads, Tq, Tk, causal, mb) in enumerate(cases):
        C = 64 * heads; G = B * heads
        Tqp = (Tq + 127) // 128 * 128; Tkp = (Tk + 63) // 64 * 64
        Q = rbits(rng, (B, Tq, C), mb); K = rbits(rng, (B, Tk, C), mb); Vv = rbits(rng, (B, Tk, C), mb)
        if mb == 8:
            Q = rng.integers(-127, 128, (B, Tq, C)).astype(np.int32); K = rng.integers(-127, 128, (B, Tk, C)).astype(np.int32); Vv = rng.integers(-127, 128, (B, Tk, C)).astype(np.int32)
        q = [torch.zeros((G, Tqp, 64), dtype=torch.int8, device="cuda") for _ in range(2)] + [torch.zeros((G, Tqp), dtype=torch.int32, device="cuda")] + [torch.zeros((G, Tqp), dtype=torch.int64, device="cuda") for _ in range(3)]
        k = [torch.zeros((G, Tkp, 64), dtype=torch.int8, device="cuda") for _ in range(2)] + [torch.zeros((G, Tkp), dtype=torch.int32, device="cuda")] + [torch.zeros((G, Tkp), dtype=torch.int64, device="cuda") for _ in range(3)]
        ck(R.ref_quant_heads(P(D(Q)), B, Tq, C, heads, Tqp, *[P(t) for t in q]))
        ck(R.ref_quant_heads(P(D(K)), B, Tk, C, heads, Tkp, *[P(t) for t in k]))
        vh, vl = torch.zeros((G, 64, Tkp), dtype=torch.int8, device="cuda"), torch.zeros((G, 64, Tkp), dtype=torch.int8, device="cuda")
        ev, vs, scr = torch.zeros((G, 64), dtype=torch.int32, device="cuda"), torch.zeros((G, 64), dtype=torch.int64, device="cuda"), torch.zeros((G, 64), dtype=torch.int32, device="cuda")
        ck(R.ref_quant_v(P(D(Vv)), B, Tk, C, heads, Tkp, P(vh), P(vl), P(ev), P(vs), P(scr)))
        gmx, gr = torch.zeros((G, Tqp), dtype=torch.int32, device="cuda"), torch.zeros((G, Tqp), dtype=torch.int64, device="cuda")
        o = sentinel((B, Tq, C), torch.int32); rm = torch.zeros((B * Tq,), dtype=torch.int32, device="cuda")
        ck(R.ref_fused_attention(P(q[0]), P(q[1]), P(q[2]), P(q[3]), P(q[4]), P(k[0]), P(k[1]), P(k[2]), P(k[5]),
                                 P(vh), P(vl), P(ev), P(vs), B, heads, Tq, Tqp, Tk, Tkp, causal, P(D(ex.astype(np.int64))), C, P(gmx), P(gr), P(o), P(rm)))
        res.update({f"a{i}_meta": np.array([B, heads, Tq, Tk, causal, Tqp, Tkp]), f"a{i}_Q": Q, f"a{i}_K": K, f"a{i}_V": Vv, f"a{i}_out": H(o), f"a{i}_rm": H(rm)})
        for nm, lst in (("q", q), ("k", k)):
            for j, field in enumerate(("hi", "lo", "e", "hs", "ls", "ts")):
                res[f"a{i}_{nm}{field}"] = H(lst[j])
        res.update({f"a{i}_vhi": H(vh), f"a{i}_vlo": H(vl), f"a{i}_ev": H(ev), f"a{i}_vsum": H(vs)})
    np.savez_compressed(os.path.join(out, "attention.npz"), **res)


def case_engine(out, model, bench):
    """the reference engine on the synthetic model: context, per-block digests, x0 (eager and graph)"""
    B = 2
    h = R.ref_open(model.encode(), 0, B, 1, 1)
    if not h:
        raise RuntimeError(R.ref_last_error().decode())
    toks = (ctypes.c_int * 3)(320, 736, 3240)
    ck(R.ref_set_prompt(V(h), toks, 3))
    ctx = np.zeros((77, 1024), np.int32)
    ck(R.ref_context(V(h), toks, 3, ctx.ctypes.data_as(V)))
    seeds = np.stack([np.frombuffer(hashlib.sha256(b"vela-b200" + bytes([b])).digest(), np.uint8) for b in range(B)])
    taps = {}
    TAP = ctypes.CFUNCTYPE(None, V, ctypes.c_char_p, ctypes.POINTER(ctypes.c_int32), ctypes.c_size_t)

    def tap(u, name, data, n):
        a = np.ctypeslib.as_array(data, shape=(n,))
        taps[name.decode()] = hashlib.sha256(a.tobytes()).hexdigest()
    cb = TAP(tap)
    x0e = np.zeros((B, 32768), np.uint8)
    ck(R.ref_unet_taps(V(h), seeds.ctypes.data_as(V), x0e.ctypes.data_as(V), cb, V(0)))
    x0g = np.zeros((B, 32768), np.uint8)
    ms = ctypes.c_float(0)
    ck(R.ref_run(V(h), 0, seeds.ctypes.data_as(V), x0g.ctypes.data_as(V), ctypes.byref(ms)))
    ck(R.ref_run(V(h), 0, seeds.ctypes.data_as(V), x0g.ctypes.data_as(V), ctypes.byref(ms)))
    R.ref_close(V(h))
    np.savez_compressed(os.path.join(out, "engine.npz"), seeds=seeds, ctx=ctx, x0=x0e, x0_graph=x0g)
    with open(os.path.join(out, "engine_taps.json"), "w") as f:
        json.dump(taps, f, indent=1)
    print("engine: eager == graph:", bool((x0e == x0g).all()), "taps:", len(taps))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("out")
    ap.add_argument("--model", default="")
    ap.add_argument("--only", default="")
    a = ap.parse_args()
    os.makedirs(a.out, exist_ok=True)
    rng = np.random.default_rng(20261201)
    cases = [case_quant_rows, case_gemm, case_gemm_sources, case_im2col, case_norms, case_misc, case_attention]
    for c in cases:
        if a.only and a.only not in c.__name__:
            continue
        t0 = time.time()
        c(a.out, rng)
        torch.cuda.synchronize()
        _KEEP.clear()
        print(f"{c.__name__}: {time.time() - t0:.1f}s", flush=True)
    if a.model:
        t0 = time.time()
        case_engine(a.out, a.model, False)
        print(f"case_engine: {time.time() - t0:.1f}s", flush=True)


if __name__ == "__main__":
    main()
