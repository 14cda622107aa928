"""vela_quant_v_static: the V quantiser for callers that must not allocate device memory.

Such a caller (a host whose device memory is already committed to its engines and models, or one on a
latency-critical path where cudaFree would wait for the whole device) cannot hand vela_quant_v the u32[G*64]
scratch buffer it asks for; vela_quant_v_static keeps that scratch in a fixed array inside the library.  It
must give exactly what vela_quant_v gives, call after call: the shared array keeps the previous call's column
maxima, so two calls in a row, the second on smaller values, would expose a missing clear.  Sizes beyond the
array are refused with VELA_ERR_ARG.  This file runs last (test_zz_*), alone or after the other GPU tests.
"""
import ctypes

import numpy as np
import pytest

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")
if not torch.cuda.is_available():
    pytest.skip("no CUDA device", allow_module_level=True)

import vela_b200 as V  # noqa: E402

MAX_COLS = 65536      # VELA_QUANT_V_STATIC_MAX_COLS


def P(t):
    return ctypes.c_void_p(t.data_ptr())


def outputs(G, Tkp):
    return [torch.full((G, 64, Tkp), 0x55, dtype=torch.int8, device="cuda"), torch.full((G, 64, Tkp), 0x55, dtype=torch.int8, device="cuda"),
            torch.full((G, 64), -1, dtype=torch.int32, device="cuda"), torch.full((G, 64), -1, dtype=torch.int64, device="cuda")]


@pytest.mark.parametrize("B,Tk,heads,bits", [(2, 4096, 5, (24, 12)), (8, 77, 10, (31, 9)), (1, 1000, 20, (16, 30))])
def test_matches_vela_quant_v_on_two_calls(B, Tk, heads, bits):
    L = V.lib()
    rng = np.random.default_rng(B * 1000 + Tk)
    C, G, Tkp = 64 * heads, B * heads, (Tk + 63) // 64 * 64
    for nbits in bits:       # two calls in a row on the shared scratch; the second call's maxima differ from the first's
        lim = 2 ** (nbits - 1)
        X = torch.from_numpy(rng.integers(-lim, lim, (B, Tk, C), dtype=np.int64).astype(np.int32)).cuda()
        ref, got = outputs(G, Tkp), outputs(G, Tkp)
        scratch = torch.empty((G, 64), dtype=torch.int32, device="cuda")
        V.check(L.vela_quant_v(None, P(X), B, Tk, C, heads, Tkp, *[P(t) for t in ref], P(scratch)))
        V.check(L.vela_quant_v_static(None, P(X), B, Tk, C, heads, Tkp, *[P(t) for t in got]))
        torch.cuda.synchronize()
        for r, g in zip(ref, got):
            assert torch.equal(r, g), (B, Tk, heads, nbits)


def test_rejects_more_columns_than_the_static_scratch():
    L = V.lib()
    heads = 8
    B = MAX_COLS // (64 * heads) + 1
    dummy = ctypes.c_void_p(256)
    rc = L.vela_quant_v_static(None, dummy, B, 64, 64 * heads, heads, 64, dummy, dummy, dummy, dummy)
    assert rc == -1
    assert "static scratch" in L.vela_last_error().decode()
