"""W8A16 GEMM on the B200 (vela_gemm_w8a16 through the C ABI) vs the CPU oracle: bit-exact.

Covers the three A sources (planar int8, int32 quantised on load, implicit 3x3 conv),
every epilogue (plain + residual + row max, GELU, GEGLU, split3, q|k|v head quantisation),
the split-K path for deep K, padded / ragged M and N, and the config-1 shape
(M 4096, N 320, K 320).  The reference's own test shapes are src/test_gemm_hl.cu:12,55.
"""
import ctypes

import numpy as np
import pytest

from oracle import pyoracle as O

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")
if not torch.cuda.is_available():
    pytest.skip("no CUDA device", allow_module_level=True)

import vela_b200 as V  # noqa: E402
from vela_b200 import abi  # noqa: E402
from tests.gpu_util import Dev, P, A, H, rbits, cst_for  # noqa: E402


def run_gemm(A_, Mp, Mreal, dW, ldw, Np, Nreal, Kp, dcst, E):
    V.check(V.lib().vela_gemm_w8a16(None, ctypes.byref(A_), Mp, Mreal, P(dW), ldw, Np, Nreal, Kp, P(dcst), ctypes.byref(E)))
    torch.cuda.synchronize()
    assert V.lib().vela_device_error(1) == 0


def planar_src(dhi, dlo, ld, de):
    a = abi.ASrc(); a.src = abi.SRC_I8; a.hi = A(dhi); a.lo = A(dlo); a.ld8 = ld; a.e = A(de)
    return a


def test_planar_epilogues(golden):
    g = golden("gemm"); d = Dev()
    Mreal, Mp, Nreal, Np, Kp = 200, 256, 192, 192, 336
    Ahi, Alo, W, cst, e, R = g["Ahi"], g["Alo"], g["W"], g["cst"], g["e"], g["R"]
    src = planar_src(d(Ahi), d(Alo), Kp, d(e)); dW, dc, dphi = d(W), d(cst), d(g["phi"])
    # plain + residual + row max
    Y = d.empty((Mreal, Nreal), torch.int32, 0x5A); rm = d.zeros(Mp, torch.int32)
    E = abi.AEpi(); E.epi = abi.EPI_PLAIN; E.Y = A(Y); E.ldy = Nreal; E.residual = A(d(R)); E.rowmax = A(rm)
    run_gemm(src, Mp, Mreal, dW, Kp, Np, Nreal, Kp, dc, E)
    ey = np.zeros((Mreal, Nreal), np.int32); erm = np.zeros(Mreal, np.uint32)
    O.gemm_hl(Ahi, Alo, Mreal, W, Nreal, Kp, cst, e, O.EPI_PLAIN, Y=ey, ldy=Nreal, residual=R, rowmax=erm)
    assert np.array_equal(H(Y), ey)
    assert np.array_equal(H(rm)[:Mreal].view(np.uint32), erm)
    # GELU
    Y = d.empty((Mreal, Nreal), torch.int32, 0x5A)
    E = abi.AEpi(); E.epi = abi.EPI_GELU; E.Y = A(Y); E.ldy = Nreal; E.Lphi = A(dphi)
    run_gemm(src, Mp, Mreal, dW, Kp, Np, Nreal, Kp, dc, E)
    assert np.array_equal(H(Y), g["Y_gelu"])
    # GEGLU + row max
    Y = d.empty((Mreal, Nreal // 2), torch.int32, 0x5A); rm = d.zeros(Mp, torch.int32)
    E = abi.AEpi(); E.epi = abi.EPI_GEGLU; E.Y = A(Y); E.ldy = Nreal // 2; E.Lphi = A(dphi); E.rowmax = A(rm)
    run_gemm(src, Mp, Mreal, dW, Kp, Np, Nreal, Kp, dc, E)
    assert np.array_equal(H(Y), g["Y_geglu"])
    assert np.array_equal(H(rm)[:Mreal], g["rm_geglu"])
    # split3
    Ys = [d.empty((Mreal, 64), torch.int32, 0x5A) for _ in range(3)]
    E = abi.AEpi(); E.epi = abi.EPI_SPLIT3; E.Y = A(Ys[0]); E.Y1 = A(Ys[1]); E.Y2 = A(Ys[2]); E.Cs = 64; E.ldy = 64
    run_gemm(src, Mp, Mreal, dW, Kp, Np, Nreal, Kp, dc, E)
    for i in range(3):
        assert np.array_equal(H(Ys[i]), g[f"Y_split{i}"])


def test_qkv_epilogue(golden):
    g = golden("gemm"); d = Dev()
    C, heads, T, B, Tp, Kp = 128, 2, 100, 2, 128, 336
    G = B * heads
    Wq, cq = g["Wq"], g["cq"]
    exp = {}
    for p in ("q", "k"):
        exp[p + "hi"] = np.zeros((G, Tp, 64), np.int8); exp[p + "lo"] = np.full((G, Tp, 64), -128, np.int8)
        exp[p + "e"] = np.zeros((G, Tp), np.int32); exp[p + "hs"] = np.zeros((G, Tp), np.int64)
        exp[p + "ls"] = np.full((G, Tp), -8192, np.int64); exp[p + "ts"] = np.zeros((G, Tp), np.int64)
    ev = np.zeros((200, C), np.int32)
    O.gemm_hl(g["Ahi"], g["Alo"], 200, Wq, 3 * C, Kp, cq, g["e"], O.EPI_QKV, Y2=ev,
              qkv=dict(heads=heads, T=T, TpQ=Tp, TpK=Tp, C=C, **{k: exp[k] for k in exp if k[1:] in ("hi", "lo", "e")},
                       qhs=exp["qhs"], qls=exp["qls"], qts=exp["qts"], khs=exp["khs"], kls=exp["kls"], kts=exp["kts"]))
    dev = {}
    for p in ("q", "k"):
        dev[p + "hi"] = d(exp[p + "hi"] * 0); dev[p + "lo"] = d(np.full((G, Tp, 64), -128, np.int8)); dev[p + "e"] = d(np.zeros((G, Tp), np.int32))
        dev[p + "hs"] = d(np.zeros((G, Tp), np.int64)); dev[p + "ls"] = d(np.full((G, Tp), -8192, np.int64)); dev[p + "ts"] = d(np.zeros((G, Tp), np.int64))
    Vt = d.empty((200, C), torch.int32, 0x5A)
    src = planar_src(d(g["Ahi"]), d(g["Alo"]), Kp, d(g["e"]))
    E = abi.AEpi(); E.epi = abi.EPI_QKV; E.Y2 = A(Vt); E.heads = heads; E.T = T; E.TpQ = Tp; E.TpK = Tp; E.C = C
    for k in ("qhi", "qlo", "khi", "klo", "qe", "ke", "qhs", "qls", "qts", "khs", "kls", "kts"):
        setattr(E, k, A(dev[k[0] + k[1:]]))
    run_gemm(src, 256, 200, d(Wq), Kp, 3 * C, 3 * C, Kp, d(cq), E)
    assert np.array_equal(H(Vt), ev)
    for k in exp:
        assert np.array_equal(H(dev[k]), exp[k]), k


def test_x32_source(golden):
    g = golden("gemm_sources"); d = Dev()
    X, W, cst, R = g["x32_X"], g["x32_W"], g["x32_cst"], g["x32_R"]
    rows, K = X.shape; N, Mp = 128, 192
    rmx = np.zeros(Mp, np.uint32); rmx[:rows] = np.abs(X.astype(np.int64)).max(1)
    a = abi.ASrc(); a.src = abi.SRC_X32; a.x = A(d(X)); a.ldx = K; a.rowmax = A(d(rmx.view(np.int32))); a.K = K
    Y = d.empty((rows, N), torch.int32, 0x5A); rm = d.zeros(Mp, torch.int32)
    E = abi.AEpi(); E.epi = abi.EPI_PLAIN; E.Y = A(Y); E.ldy = N; E.residual = A(d(R)); E.rowmax = A(rm)
    run_gemm(a, Mp, rows, d(W), K, N, N, K, d(cst), E)
    assert np.array_equal(H(Y), g["x32_Y"])
    assert np.array_equal(H(rm)[:rows], g["x32_rm"])


def conv_case(d, X, Wc, cc, stride, Kp=None):
    B, Hh, Ww, C = X.shape; N = Wc.shape[0]
    Ho = (Hh - 1) // stride + 1; Wo = (Ww - 1) // stride + 1; rows = B * Ho * Wo; Mp = (rows + 63) // 64 * 64
    Kp = Kp or 9 * C
    pm = O.pixmax(X, B * Hh * Ww, C)
    e = d.zeros(Mp, torch.int32)
    V.check(V.lib().vela_conv_e(None, P(d(pm.view(np.int32))), B, Hh, Ww, stride, P(e)))
    a = abi.ASrc(); a.src = abi.SRC_CONV32; a.img = A(d(X)); a.H = Hh; a.W = Ww; a.C = C; a.stride = stride; a.Ho = Ho; a.Wo = Wo; a.K = 9 * C; a.e = A(e)
    Y = d.empty((rows, N), torch.int32, 0x5A)
    E = abi.AEpi(); E.epi = abi.EPI_PLAIN; E.Y = A(Y); E.ldy = N
    Wp = np.zeros((N, Kp), np.int8); Wp[:, :9 * C] = Wc
    run_gemm(a, Mp, rows, d(Wp), Kp, N, N, Kp, d(cc), E)
    hi, lo, ee = O.im2col3(X, pm, B, Hh, Ww, C, stride, Kp, rows)
    exp = np.zeros((rows, N), np.int32)
    O.gemm_hl(hi, lo, rows, Wp, N, Kp, cc, ee, O.EPI_PLAIN, Y=exp, ldy=N)
    assert np.array_equal(H(e)[:rows], ee)
    return H(Y), exp


def test_conv_source(golden):
    g = golden("gemm_sources"); d = Dev()
    for stride in (1, 2):
        got, exp = conv_case(d, g["conv_X"], g["conv_W"], g["conv_cst"], stride)
        assert np.array_equal(got, exp)
        assert np.array_equal(got, g[f"conv{stride}_Y"])


def test_conv_320ch_16x16():
    rng = np.random.default_rng(5); d = Dev()
    X = rbits(rng, (2, 16, 16, 320), 22)
    W = rng.integers(-127, 128, (320, 2880)).astype(np.int8)
    c = cst_for(rng, W, 320, 320)
    for stride in (1, 2):
        got, exp = conv_case(d, X, W, c, stride)
        assert np.array_equal(got, exp), stride


@pytest.mark.parametrize("B,Hh,C,N,stride,Kp", [(8, 16, 256, 1280, 1, 2304), (8, 16, 256, 1536, 1, 2304),
                                                 (4, 16, 128, 1280, 2, 1216)])
def test_conv_explicit_im2col_deep(B, Hh, C, N, stride, Kp):
    """the engine's deep-level convolution (640 or more output channels at 32x32 and below): the window-quantised
    im2col planes (one warp per row and tap) against the oracle's im2col; then the planar GEMM -- at deep K (36
    k-blocks) on 160-column tiles (N 1280: 128 tiles in one wave) and 256-column tiles (N 1536: 96 tiles, where 160
    columns would need two waves), at 19 k-blocks on the short-K tiles -- the first 128 rows against the oracle's
    GEMM, every row against the implicit conv of the same image"""
    rng = np.random.default_rng(7 + stride); d = Dev()
    X = rbits(rng, (B, Hh, Hh, C), 22)
    Ho = (Hh - 1) // stride + 1; rows = B * Ho * Ho; Mp = (rows + 63) // 64 * 64
    W = np.zeros((N, Kp), np.int8); W[:, :9 * C] = rng.integers(-127, 128, (N, 9 * C)).astype(np.int8)
    c = cst_for(rng, W, N, N)
    pm = O.pixmax(X, B * Hh * Hh, C)
    dX, dpm, dW, dc = d(X), d(pm.view(np.int32)), d(W), d(c)
    hi, lo, e = d.empty((Mp, Kp), torch.int8, 0x5A), d.empty((Mp, Kp), torch.int8, 0x5A), d.empty((Mp,), torch.int32, 0x5A)
    V.check(V.lib().vela_im2col3(None, P(dX), P(dpm), B, Hh, Hh, C, stride, P(hi), P(lo), P(e), Kp))
    ohi, olo, oe = O.im2col3(X, pm, B, Hh, Hh, C, stride, Kp, rows)
    assert np.array_equal(H(hi)[:rows], ohi) and np.array_equal(H(lo)[:rows], olo) and np.array_equal(H(e)[:rows], oe)
    Y = d.empty((rows, N), torch.int32, 0x5A)
    E = abi.AEpi(); E.epi = abi.EPI_PLAIN; E.Y = A(Y); E.ldy = N
    run_gemm(planar_src(hi, lo, Kp, e), Mp, rows, dW, Kp, N, N, Kp, dc, E)
    exp = np.zeros((128, N), np.int32)
    O.gemm_hl(ohi[:128], olo[:128], 128, W, N, Kp, c, oe[:128], O.EPI_PLAIN, Y=exp, ldy=N)
    got = H(Y)
    assert np.array_equal(got[:128], exp)
    ce = d.zeros(Mp, torch.int32)
    V.check(V.lib().vela_conv_e(None, P(dpm), B, Hh, Hh, stride, P(ce)))
    a = abi.ASrc(); a.src = abi.SRC_CONV32; a.img = A(dX); a.H = Hh; a.W = Hh; a.C = C; a.stride = stride; a.Ho = Ho; a.Wo = Ho
    a.K = 9 * C; a.e = A(ce)
    Yi = d.empty((rows, N), torch.int32, 0x5A)
    Ei = abi.AEpi(); Ei.epi = abi.EPI_PLAIN; Ei.Y = A(Yi); Ei.ldy = N
    run_gemm(a, Mp, rows, dW, Kp, N, N, Kp, dc, Ei)
    assert np.array_equal(got, H(Yi))


@pytest.mark.parametrize("B,Hh,N", [(2, 64, 320), (3, 10, 64)])
def test_conv_4ch_input(B, Hh, N):
    """the UNet's input conv (4 channels, K = 36 padded to 48): nine 16-byte pixels per row quantised on load, no im2col
    buffer; stride 1 and 2, full-range random bit widths"""
    rng = np.random.default_rng(B * 10 + Hh); d = Dev()
    X = rbits(rng, (B, Hh, Hh, 4), 30)
    W = rng.integers(-127, 128, (N, 36)).astype(np.int8)
    c = cst_for(rng, W, N, N)
    for stride in (1, 2):
        got, exp = conv_case(d, X, W, c, stride, Kp=48)
        assert np.array_equal(got, exp), (B, Hh, N, stride)


@pytest.mark.parametrize("B,Hh,C,N", [(2, 12, 64, 128), (3, 8, 96, 64), (1, 32, 64, 192)])
def test_conv_shapes_both_loaders(B, Hh, C, N):
    """image sizes whose 128-row tiles are not whole output rows (12x12, stride-2 6x6) keep the per-thread loader;
    8x8 (whole images per tile, odd batch) and 32x32 (whole rows) stage the image by TMA"""
    rng = np.random.default_rng(B * 100 + Hh); d = Dev()
    X = rbits(rng, (B, Hh, Hh, C), 24)
    W = rng.integers(-127, 128, (N, 9 * C)).astype(np.int8)
    c = cst_for(rng, W, N, N)
    for stride in (1, 2):
        got, exp = conv_case(d, X, W, c, stride)
        assert np.array_equal(got, exp), (B, Hh, C, N, stride)


@pytest.mark.parametrize("B,Hh,C,N", [(2, 64, 64, 320), (4, 32, 64, 640), (8, 16, 64, 1280)])
def test_conv_wide_outputs(B, Hh, C, N):
    """outputs of 2, 4 and 8 column tiles of 160 over many row tiles (the UNet's conv widths)"""
    rng = np.random.default_rng(N + Hh); d = Dev()
    X = rbits(rng, (B, Hh, Hh, C), 26)
    W = rng.integers(-127, 128, (N, 9 * C)).astype(np.int8)
    c = cst_for(rng, W, N, N)
    got, exp = conv_case(d, X, W, c, 1)
    assert np.array_equal(got, exp), (B, Hh, C, N)


def test_x32_many_row_tiles():
    rng = np.random.default_rng(5); d = Dev()
    M, K, N = 8192, 256, 320
    X = rbits(rng, (M, K), 28)
    W = rng.integers(-127, 128, (N, K)).astype(np.int8); c = cst_for(rng, W, N, N)
    rowmax = np.abs(X.astype(np.int64)).max(1).astype(np.uint32)
    a = abi.ASrc(); a.src = abi.SRC_X32; a.x = A(d(X)); a.ldx = K; a.K = K; a.rowmax = A(d(rowmax.view(np.int32)))
    Y = d.empty((M, N), torch.int32, 0x5A)
    E = abi.AEpi(); E.epi = abi.EPI_PLAIN; E.Y = A(Y); E.ldy = N
    run_gemm(a, M, M, d(W), K, N, N, K, d(c), E)
    hi, lo, e = O.quant_rows(X, K, M)
    exp = np.zeros((M, N), np.int32)
    O.gemm_hl(hi, lo, M, W, N, K, c, e, O.EPI_PLAIN, Y=exp, ldy=N)
    assert np.array_equal(H(Y), exp)


@pytest.mark.parametrize("M,K,N", [(300, 96, 128), (130, 160, 64)])
def test_x32_ragged_k(M, K, N):
    """int32 source whose K is not a multiple of 64: the staged box past K reads zeros (quantised value 0)"""
    rng = np.random.default_rng(M + K); d = Dev()
    Kp = (K + 15) // 16 * 16; Mp = (M + 63) // 64 * 64
    X = rbits(rng, (M, K), 28)
    W = rng.integers(-127, 128, (N, Kp)).astype(np.int8); c = cst_for(rng, W, N, N)
    rowmax = np.abs(X.astype(np.int64)).max(1).astype(np.uint32)
    a = abi.ASrc(); a.src = abi.SRC_X32; a.x = A(d(X)); a.ldx = K; a.K = K; a.rowmax = A(d(rowmax.view(np.int32)))
    Y = d.empty((M, N), torch.int32, 0x5A)
    E = abi.AEpi(); E.epi = abi.EPI_PLAIN; E.Y = A(Y); E.ldy = N
    run_gemm(a, Mp, M, d(W), Kp, N, N, Kp, d(c), E)
    hi, lo, e = O.quant_rows(X, Kp, Mp)
    exp = np.zeros((M, N), np.int32)
    O.gemm_hl(hi, lo, M, W, N, Kp, c, e, O.EPI_PLAIN, Y=exp, ldy=N)
    assert np.array_equal(H(Y), exp)


@pytest.mark.parametrize("M,N,ldy", [(150, 200, 204), (150, 200, 201), (37, 72, 76)])
def test_plain_ragged_n_strided_y(M, N, ldy):
    """plain epilogue (+ residual + row max) with N not a multiple of 16 into a strided Y: the last 16-column chunk
    is partial (shared-memory box + TMA store clipped at N when ldy % 4 == 0, per-element stores otherwise), and the
    columns [N, ldy) and the rows past M keep their contents"""
    rng = np.random.default_rng(M + N + ldy); d = Dev()
    K = 320; Np = (N + 15) // 16 * 16; Mp = (M + 63) // 64 * 64
    q = rng.integers(-32768, 32768, (Mp, K))
    Ahi = (q >> 8).astype(np.int8); Alo = ((q & 255) - 128).astype(np.int8)
    W = rng.integers(-127, 128, (Np, K)).astype(np.int8)
    c = cst_for(rng, W, N, Np); e = rng.integers(0, 8, Mp).astype(np.int32)
    R = np.zeros((M, ldy), np.int32); R[:, :N] = rbits(rng, (M, N), 30)
    Y = d.empty((M + 3, ldy), torch.int32, 0x5A); rm = d.zeros(Mp, torch.int32)
    E = abi.AEpi(); E.epi = abi.EPI_PLAIN; E.Y = A(Y); E.ldy = ldy; E.residual = A(d(R)); E.rowmax = A(rm)
    run_gemm(planar_src(d(Ahi), d(Alo), K, d(e)), Mp, M, d(W), K, Np, N, K, d(c), E)
    exp = np.full((M + 3, ldy), np.int32(0x5A5A5A5A), np.int32); erm = np.zeros(M, np.uint32)
    O.gemm_hl(Ahi, Alo, M, W, N, K, c, e, O.EPI_PLAIN, Y=exp, ldy=ldy, residual=R, rowmax=erm)
    assert np.array_equal(H(Y), exp)
    assert np.array_equal(H(rm)[:M].view(np.uint32), erm)


def test_config1_shape():
    """config 1: A 16-bit uniform over [-32768, 32767] as planes, M 4096, N = K = 320, e in [0, 12)."""
    rng = np.random.default_rng(1); d = Dev()
    M, N, K = 4096, 320, 320
    q = rng.integers(-32768, 32768, (M, K))
    Ahi = (q >> 8).astype(np.int8); Alo = ((q & 255) - 128).astype(np.int8)
    W = rng.integers(-127, 128, (N, K)).astype(np.int8)
    c = cst_for(rng, W, N, N); e = rng.integers(0, 12, M).astype(np.int32)
    Y = d.empty((M, N), torch.int32, 0x5A)
    E = abi.AEpi(); E.epi = abi.EPI_PLAIN; E.Y = A(Y); E.ldy = N
    run_gemm(planar_src(d(Ahi), d(Alo), K, d(e)), M, M, d(W), K, N, N, K, d(c), E)
    exp = np.zeros((M, N), np.int32)
    O.gemm_hl(Ahi, Alo, M, W, N, K, c, e, O.EPI_PLAIN, Y=exp, ldy=N)
    assert np.array_equal(H(Y), exp)


@pytest.mark.parametrize("M,N,K", [(256, 256, 5760), (512, 192, 2880), (100, 1280, 1024)])
def test_deep_k_split(M, N, K):
    """deep K with a workspace: split-K partial sums + reduction epilogue (+ residual + row max)"""
    rng = np.random.default_rng(M + N + K); d = Dev()
    Mp = (M + 63) // 64 * 64
    Ahi = rng.integers(-128, 128, (Mp, K)).astype(np.int8); Alo = rng.integers(-128, 128, (Mp, K)).astype(np.int8)
    W = rng.integers(-127, 128, (N, K)).astype(np.int8)
    c = cst_for(rng, W, N, N); e = rng.integers(0, 12, Mp).astype(np.int32)
    R = rbits(rng, (M, N), 30)
    ws = d.zeros(64 << 20, torch.uint8)
    Y = d.empty((M, N), torch.int32, 0x5A); rm = d.zeros(Mp, torch.int32)
    E = abi.AEpi(); E.epi = abi.EPI_PLAIN; E.Y = A(Y); E.ldy = N; E.residual = A(d(R)); E.rowmax = A(rm)
    E.workspace = A(ws); E.workspace_bytes = 64 << 20
    run_gemm(planar_src(d(Ahi), d(Alo), K, d(e)), Mp, M, d(W), K, N, N, K, d(c), E)
    exp = np.zeros((M, N), np.int32); erm = np.zeros(M, np.uint32)
    O.gemm_hl(Ahi, Alo, M, W, N, K, c, e, O.EPI_PLAIN, Y=exp, ldy=N, residual=R, rowmax=erm)
    assert np.array_equal(H(Y), exp)
    assert np.array_equal(H(rm)[:M].view(np.uint32), erm)


def test_bad_shape_is_an_error():
    d = Dev()
    a = abi.ASrc(); a.src = abi.SRC_I8
    E = abi.AEpi(); E.epi = abi.EPI_PLAIN
    rc = V.lib().vela_gemm_w8a16(None, ctypes.byref(a), 64, 64, None, 16, 64, 64, 20, None, ctypes.byref(E))
    assert rc == -1 and b"multiples of 16" in V.lib().vela_last_error()
