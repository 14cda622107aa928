"""Failure paths on the B200 without a GPU fault: bounded waits that run out, and arena exhaustion.

Every barrier wait in the GEMM and attention kernels gives up after a limit of SM clock cycles, records a
timeout code in a device error word and lets the kernel drain and return.  The *_stalled entry points launch
the real kernels with their TMA producers idle and a short limit (10^6 cycles, about half a millisecond), so
every consumer's wait runs out with nothing in flight.  The tests check that the call returns, that
vela_device_error reports the timeout, and that the next normal launch on the same context is still
bit-exact against the CPU oracle.  The engine's arena test asks for an arena far too small for a step and
expects VELA_ERR_ARENA (the reference throws at src/engine.cu:108).
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

LIMIT = 1_000_000          # SM clock cycles before a wait gives up in the stalled launches
VELA_ERR_ARENA = -3


def test_gemm_wait_timeout_then_exact():
    L = V.lib(); d = Dev(); rng = np.random.default_rng(11)
    assert L.vela_device_error(1) == 0
    Mreal, Mp, N, Np, K, Kp = 300, 384, 320, 320, 320, 320
    X = rbits(rng, (Mreal, K), 24)
    W = rng.integers(-127, 128, (Np, Kp), dtype=np.int64).astype(np.int8)
    cst = cst_for(rng, W, N, Np)
    rm_in = np.abs(X.astype(np.int64)).max(1).astype(np.uint32)
    dW, dc = d(W), d(cst)
    for src in (abi.SRC_I8, abi.SRC_X32):
        a = abi.ASrc()
        if src == abi.SRC_I8:
            hi, lo, e = O.quant_rows(X, Kp, Mp)
            a.src = src; a.hi = A(d(hi)); a.lo = A(d(lo)); a.ld8 = Kp; a.e = A(d(e))
        else:
            a.src = src; a.x = A(d(X)); a.ldx = K; a.K = K; a.rowmax = A(d(rm_in.view(np.int32)))
        Y = d.empty((Mreal, N), torch.int32, 0x5A)
        E = abi.AEpi(); E.epi = abi.EPI_PLAIN; E.Y = A(Y); E.ldy = N
        V.check(L.vela_gemm_w8a16_stalled(None, ctypes.byref(a), Mp, Mreal, P(dW), Kp, Np, N, Kp, P(dc), ctypes.byref(E), LIMIT))
        torch.cuda.synchronize()
        assert L.vela_device_error(1) != 0, "the stalled GEMM did not report its timed-out waits"
        assert L.vela_device_error(0) == 0, "the error word was not cleared"
        # the same context runs the normal launch bit-exactly afterwards
        V.check(L.vela_gemm_w8a16(None, ctypes.byref(a), Mp, Mreal, P(dW), Kp, Np, N, Kp, P(dc), ctypes.byref(E)))
        torch.cuda.synchronize()
        assert L.vela_device_error(1) == 0
        hi, lo, e = O.quant_rows(X, Kp, Mp)
        ey = np.zeros((Mreal, N), np.int32)
        O.gemm_hl(hi, lo, Mreal, W, N, Kp, cst, e, O.EPI_PLAIN, Y=ey, ldy=N)
        assert np.array_equal(H(Y), ey)


def test_attention_wait_timeout_then_exact():
    L = V.lib(); d = Dev(); rng = np.random.default_rng(12)
    B, heads, Tq, Tk = 1, 2, 256, 320
    C, G, Tqp, Tkp = 64 * heads, B * heads, 256, 320
    Q, K_, Vv = (rbits(rng, (B, T, C), 24) for T in (Tq, Tk, Tk))
    q = [d.zeros((G, Tqp, 64), torch.int8), d.zeros((G, Tqp, 64), torch.int8), d.zeros((G, Tqp), torch.int32)] + [d.zeros((G, Tqp), torch.int64) for _ in range(3)]
    k = [d.zeros((G, Tkp, 64), torch.int8), d.zeros((G, Tkp, 64), torch.int8), d.zeros((G, Tkp), torch.int32)] + [d.zeros((G, Tkp), torch.int64) for _ in range(3)]
    v = [d.zeros((G, 64, Tkp), torch.int8), d.zeros((G, 64, Tkp), torch.int8), d.zeros((G, 64), torch.int32), d.zeros((G, 64), torch.int64)]
    V.check(L.vela_quant_heads(None, P(d(Q)), B, Tq, C, heads, Tqp, *[P(t) for t in q]))
    V.check(L.vela_quant_heads(None, P(d(K_)), B, Tk, C, heads, Tkp, *[P(t) for t in k]))
    V.check(L.vela_quant_v(None, P(d(Vv)), B, Tk, C, heads, Tkp, *[P(t) for t in v], P(d.zeros((G, 64), torch.int32))))
    lexp = np.rint(1073741824.0 * np.exp(-np.arange(1025) / 64.0)).astype(np.int32)
    dl = d(lexp)
    out = d.zeros((B, Tq, C), torch.int32); rm = d.zeros(B * Tq, torch.int32)
    args = [P(q[0]), P(q[1]), P(q[2]), P(q[3]), P(q[4]), P(k[0]), P(k[1]), P(k[2]), P(k[5]), P(v[0]), P(v[1]), P(v[2]), P(v[3]),
            B, heads, Tq, Tqp, Tk, Tkp, 0, P(dl), C]
    torch.cuda.synchronize()
    assert L.vela_device_error(1) == 0
    V.check(L.vela_fused_attention_stalled(None, *args, P(out), P(rm), LIMIT))
    torch.cuda.synchronize()
    assert L.vela_device_error(1) != 0, "the stalled attention did not report its timed-out waits"
    V.check(L.vela_fused_attention(None, *args, None, None, P(out), P(rm)))
    torch.cuda.synchronize()
    assert L.vela_device_error(1) == 0
    eo, erm = O.attention(H(q[0]), H(q[1]), H(q[2]), H(k[0]), H(k[1]), H(k[2]), H(v[0]), H(v[1]), H(v[2]), B, heads, Tq, Tk, False, lexp)
    assert np.array_equal(H(out), eo)
    assert np.array_equal(H(rm).view(np.uint32), erm)


def test_engine_arena_exhausted(synth_model_path):
    m = V.Model(synth_model_path, 0)
    try:
        e = V.Engine(m, batch=2, graph=False, arena_bytes=16 << 20)
        with pytest.raises(V.VelaError) as ex:
            e.set_prompt([320, 736, 3240])
        assert ex.value.code == VELA_ERR_ARENA
        assert "arena" in str(ex.value)
        assert e.device_error() == 0
        e.close()
    finally:
        m.close()
