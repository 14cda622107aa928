"""Exact attention on the B200 (vela_fused_attention through the C ABI), bit-exact vs the reference.

Golden cases (tests/golden/attention.npz, produced by the reference's fused kernels): 3-pass
self-attention (256 and 1024 keys, ragged 200x180), the BASELINE config-2 value range
([-127, 127] inputs), cross-attention with 77 keys padded to 128, causal text-encoder attention.
A 2048-key case is checked against the CPU oracle (pinned to the reference).
"""
import numpy as np
import pytest

from oracle import pyoracle as O

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")
if not torch.cuda.is_available():
    pytest.skip("no CUDA device", allow_module_level=True)

import vela_b200 as V  # noqa: E402
from tests.gpu_util import Dev, P, H, rbits  # noqa: E402


def lexp_lut():
    return np.rint(1073741824.0 * np.exp(-np.arange(1025) / 64.0)).astype(np.int32)


def run(d, Q, K, Vv, B, heads, Tq, Tk, causal, lexp):
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
                                   P(vh), P(vl), P(ev), P(vs), B, heads, Tq, Tqp, Tk, Tkp, int(causal), P(d(lexp)), C, None, None, P(out), P(rm)))
    torch.cuda.synchronize()
    assert V.lib().vela_device_error(1) == 0
    return H(out), H(rm), [H(t) for t in q], [H(t) for t in k], [H(t) for t in (vh, vl, ev, vs)]


def test_golden_cases(golden):
    g = golden("attention"); d = Dev()
    i = 0
    while f"a{i}_meta" in g:
        B, heads, Tq, Tk, causal, Tqp, Tkp = [int(v) for v in g[f"a{i}_meta"]]
        out, rm, *_ = run(d, g[f"a{i}_Q"], g[f"a{i}_K"], g[f"a{i}_V"], B, heads, Tq, Tk, causal, g["lexp"])
        assert np.array_equal(out, g[f"a{i}_out"]), (i, B, heads, Tq, Tk, causal)
        assert np.array_equal(rm, g[f"a{i}_rm"]), i
        i += 1


@pytest.mark.parametrize("Tq,Tk,maxbits,seed", [(2048, 2048, 31, 1), (512, 4096, 20, 2), (300, 77, 24, 3), (256, 192, 32, 4)])
def test_against_oracle(Tq, Tk, maxbits, seed):
    """maxbits 32: uniform over the whole int32 range, so exponents reach 17, shifts go negative and scores saturate"""
    rng = np.random.default_rng(seed); d = Dev()
    B, heads = 1, 2
    if maxbits == 32:
        Q, K, Vv = [rng.integers(-2**31, 2**31, (B, T, 64 * heads), dtype=np.int64).astype(np.int32) for T in (Tq, Tk, Tk)]
    else:
        Q = rbits(rng, (B, Tq, 64 * heads), maxbits); K = rbits(rng, (B, Tk, 64 * heads), maxbits); Vv = rbits(rng, (B, Tk, 64 * heads), maxbits)
    lex = lexp_lut()
    out, rm, q, k, v = run(d, Q, K, Vv, B, heads, Tq, Tk, False, lex)
    eo, erm = O.attention(q[0], q[1], q[2], k[0], k[1], k[2], v[0], v[1], v[2], B, heads, Tq, Tk, False, lex)
    assert np.array_equal(out, eo)
    assert np.array_equal(rm.view(np.uint32), erm)
