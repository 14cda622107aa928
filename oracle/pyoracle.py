"""ctypes bindings of liboracle.so (oracle/vela_oracle.c) for tests and the bench's CPU baseline.

TEST INFRASTRUCTURE ONLY: the checker and the timed CPU baseline.  The product
(vela_b200/) never imports this module.  All arrays are numpy, host memory.
"""
import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "liboracle.so")
_lib = None


def build():
    """Compile liboracle.so if missing or stale (gcc + OpenMP)."""
    srcs = [os.path.join(HERE, f) for f in ("vela_oracle.c", "vela_oracle.h", "synth_model.c")]
    if not os.path.exists(LIB_PATH) or os.path.getmtime(LIB_PATH) < max(os.path.getmtime(f) for f in srcs):
        subprocess.run(["make", "-s", "-C", HERE, "liboracle.so"], check=True)
    return LIB_PATH


def lib():
    global _lib
    if _lib is None:
        build()
        L = ctypes.CDLL(LIB_PATH)
        L.or_model_load.restype = ctypes.c_void_p
        L.or_model_load.argtypes = [ctypes.c_char_p, ctypes.c_char_p, ctypes.c_int]
        L.or_model_free.argtypes = [ctypes.c_void_p]
        L.or_set_prompt.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int]
        L.or_context.restype = ctypes.POINTER(ctypes.c_int32)
        L.or_context.argtypes = [ctypes.c_void_p]
        L.or_unet_step.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p]
        for f in ("or_rshr", "or_floor_div", "or_quant16", "or_isqrt", "or_sat32"):
            getattr(L, f).restype = ctypes.c_int64
        L.or_rshr.argtypes = [ctypes.c_int64, ctypes.c_int64]
        L.or_floor_div.argtypes = [ctypes.c_int64, ctypes.c_int64]
        L.or_quant16.argtypes = [ctypes.c_int64, ctypes.c_int]
        L.or_isqrt.argtypes = [ctypes.c_int64]
        L.or_sat32.argtypes = [ctypes.c_int64]
        L.or_row_exp.argtypes = [ctypes.c_int64]
        L.or_score.argtypes = [ctypes.c_int64, ctypes.c_int]
        L.or_score_batch.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_size_t]
        L.or_gn_stats.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int64, ctypes.c_void_p]
        L.or_lnorm_q.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64] + [ctypes.c_void_p] * 3 + [ctypes.c_int]
        L.or_lnorm.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64, ctypes.c_void_p]
        L.or_noise.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p, ctypes.c_int64, ctypes.c_void_p, ctypes.c_void_p]
        L.or_finalize.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int, ctypes.c_int64, ctypes.c_void_p]
        L.or_act.argtypes = [ctypes.c_void_p, ctypes.c_size_t, ctypes.c_void_p]
        L.or_geglu.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_size_t, ctypes.c_void_p]
        L.or_gemm_hl.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_void_p, ctypes.c_int, ctypes.c_int, ctypes.c_int,
                                 ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p]
        L.or_chacha20_block.argtypes = [ctypes.c_void_p, ctypes.c_uint32, ctypes.c_void_p]
        L.or_set_threads.argtypes = [ctypes.c_int]
        L.or_synth_model_write.argtypes = [ctypes.c_char_p, ctypes.c_uint64]
        _lib = L
    return _lib


_PINNED = []


def ptr(a):
    """address of a numpy array; the array stays referenced until the next unpin() (a temporary
    passed inline could otherwise be freed before the C call reads it)"""
    if a is None:
        return ctypes.c_void_p(0)
    _PINNED.append(a)
    return ctypes.c_void_p(a.ctypes.data)


def unpin():
    _PINNED.clear()


def pinned(fn):
    """release the arrays a wrapper pinned once its C calls have returned"""
    import functools

    @functools.wraps(fn)
    def run(*a, **k):
        try:
            return fn(*a, **k)
        finally:
            unpin()
    return run


class Epi(ctypes.Structure):
    """or_epi_t"""
    _fields_ = [("epi", ctypes.c_int), ("Y", ctypes.c_void_p), ("ldy", ctypes.c_int), ("residual", ctypes.c_void_p),
                ("Cs", ctypes.c_int), ("Y1", ctypes.c_void_p), ("Y2", ctypes.c_void_p), ("Lphi", ctypes.c_void_p),
                ("rowmax", ctypes.c_void_p),
                ("heads", ctypes.c_int), ("T", ctypes.c_int), ("TpQ", ctypes.c_int), ("TpK", ctypes.c_int), ("C", ctypes.c_int),
                ("qhi", ctypes.c_void_p), ("qlo", ctypes.c_void_p), ("khi", ctypes.c_void_p), ("klo", ctypes.c_void_p),
                ("qe", ctypes.c_void_p), ("ke", ctypes.c_void_p),
                ("qhs", ctypes.c_void_p), ("qls", ctypes.c_void_p), ("qts", ctypes.c_void_p),
                ("khs", ctypes.c_void_p), ("kls", ctypes.c_void_p), ("kts", ctypes.c_void_p)]


EPI_PLAIN, EPI_SPLIT3, EPI_GEGLU, EPI_GELU, EPI_QKV = 0, 1, 2, 3, 4


def c32(a):
    return np.ascontiguousarray(a, dtype=np.int32)


@pinned
def quant_rows(X, Kp, Mpad):
    M, K = X.shape
    X = c32(X)
    hi = np.zeros((Mpad, Kp), np.int8); lo = np.zeros((Mpad, Kp), np.int8); e = np.zeros(M, np.int32)
    lib().or_quant_rows(ptr(X), M, K, K, ptr(hi), ptr(lo), ptr(e), Kp, Mpad)
    return hi, lo, e


@pinned
def gemm_hl(Ahi, Alo, Mreal, W, Nreal, Kp, cst, e, epi=EPI_PLAIN, Y=None, ldy=0, residual=None, Cs=0, Y1=None, Y2=None, Lphi=None, rowmax=None, qkv=None):
    E = Epi()
    E.epi = epi; E.Y = ptr(Y).value; E.ldy = ldy; E.residual = ptr(residual).value; E.Cs = Cs
    E.Y1 = ptr(Y1).value; E.Y2 = ptr(Y2).value; E.Lphi = ptr(Lphi).value; E.rowmax = ptr(rowmax).value
    if qkv:
        for k, v in qkv.items():
            setattr(E, k, ptr(v).value if isinstance(v, np.ndarray) else v)
    lib().or_gemm_hl(ptr(Ahi), ptr(Alo), Ahi.shape[1], Mreal, ptr(W), W.shape[1], Nreal, Kp, ptr(c32(cst)), ptr(c32(e)), ctypes.byref(E))


@pinned
def pixmax(X, rows, C):
    pm = np.zeros(rows, np.uint32)
    lib().or_pixmax(ptr(c32(X)), rows, C, ptr(pm))
    return pm


@pinned
def conv_e(pm, B, H, W, stride):
    Ho, Wo = (H - 1) // stride + 1, (W - 1) // stride + 1
    e = np.zeros(B * Ho * Wo, np.int32)
    lib().or_conv_e(ptr(pm), B, H, W, stride, ptr(e))
    return e


@pinned
def im2col3(X, pm, B, H, W, C, stride, Kp, Mpad):
    Ho, Wo = (H - 1) // stride + 1, (W - 1) // stride + 1
    rows = B * Ho * Wo
    hi = np.zeros((Mpad, Kp), np.int8); lo = np.zeros((Mpad, Kp), np.int8); e = np.zeros(rows, np.int32)
    lib().or_im2col3(ptr(c32(X)), ptr(pm), B, H, W, C, stride, ptr(hi), ptr(lo), ptr(e), Kp, Mpad)
    return hi, lo, e


@pinned
def gn_stats(X, B, T, C, groups, den):
    gs = np.zeros((B * groups, 6), np.int64)
    lib().or_gn_stats(ptr(c32(X)), B, T, C, groups, den, ptr(gs))
    return gs


@pinned
def gn_apply_row(X, B, T, C, groups, gs, g, beta, Lsig=None, quant=False, Kp=0):
    M = B * T
    if quant:
        hi = np.zeros((M, Kp), np.int8); lo = np.zeros((M, Kp), np.int8); e = np.zeros(M, np.int32)
        lib().or_gn_apply_row(ptr(c32(X)), B, T, C, groups, ptr(gs), ptr(c32(g)), ptr(c32(beta)), ptr(Lsig), None, None, ptr(hi), ptr(lo), ptr(e), Kp)
        return hi, lo, e
    Y = np.zeros((M, C), np.int32); pm = np.zeros(M, np.uint32)
    lib().or_gn_apply_row(ptr(c32(X)), B, T, C, groups, ptr(gs), ptr(c32(g)), ptr(c32(beta)), ptr(Lsig), ptr(Y), ptr(pm), None, None, None, 0)
    return Y, pm


@pinned
def lnorm_q(X, g, beta, den, Kp):
    M, C = X.shape
    hi = np.zeros((M, Kp), np.int8); lo = np.zeros((M, Kp), np.int8); e = np.zeros(M, np.int32)
    lib().or_lnorm_q(ptr(c32(X)), M, C, ptr(c32(g)), ptr(c32(beta)), den, ptr(hi), ptr(lo), ptr(e), Kp)
    return hi, lo, e


@pinned
def lnorm(X, g, beta, den):
    M, C = X.shape
    Y = np.zeros((M, C), np.int32)
    lib().or_lnorm(ptr(c32(X)), M, C, ptr(c32(g)), ptr(c32(beta)), den, ptr(Y))
    return Y


@pinned
def noise(seeds, gauss, cin):
    B = seeds.shape[0]
    n = np.zeros((B, 16384), np.int32); x = np.zeros((B, 16384), np.int32)
    lib().or_noise(ptr(np.ascontiguousarray(seeds, np.uint8)), B, ptr(c32(gauss)), cin, ptr(n), ptr(x))
    return n, x


@pinned
def finalize(n, eps, sig):
    B = n.shape[0]
    out = np.zeros((B, 32768), np.uint8)
    lib().or_finalize(ptr(c32(n)), ptr(c32(eps)), B, sig, ptr(out))
    return out


@pinned
def quant_heads(X, B, T, C, heads, Tp):
    G = B * heads
    hi = np.zeros((G, Tp, 64), np.int8); lo = np.zeros((G, Tp, 64), np.int8); e = np.zeros((G, Tp), np.int32)
    hs = np.zeros((G, Tp), np.int64); ls = np.zeros((G, Tp), np.int64); ts = np.zeros((G, Tp), np.int64)
    lib().or_quant_heads(ptr(c32(X)), B, T, C, heads, Tp, ptr(hi), ptr(lo), ptr(e), ptr(hs), ptr(ls), ptr(ts))
    return hi, lo, e, hs, ls, ts


@pinned
def quant_v(X, B, Tk, C, heads, Tkp):
    G = B * heads
    vh = np.zeros((G, 64, Tkp), np.int8); vl = np.zeros((G, 64, Tkp), np.int8); ev = np.zeros((G, 64), np.int32); vs = np.zeros((G, 64), np.int64)
    lib().or_quant_v(ptr(c32(X)), B, Tk, C, heads, Tkp, ptr(vh), ptr(vl), ptr(ev), ptr(vs))
    return vh, vl, ev, vs


@pinned
def attention(qhi, qlo, eq, khi, klo, ek, vhi, vlo, ev, B, heads, Tq, Tk, causal, lexp):
    G, Tqp, _ = qhi.shape
    Tkp = khi.shape[1]
    C = heads * 64
    out = np.zeros((B, Tq, C), np.int32); rm = np.zeros(B * Tq, np.uint32)
    lib().or_attention(ptr(qhi), ptr(qlo), ptr(c32(eq)), Tqp, ptr(khi), ptr(klo), ptr(c32(ek)), ptr(vhi), ptr(vlo), ptr(c32(ev)),
                       B, heads, Tq, Tk, Tkp, int(causal), ptr(c32(lexp)), C, ptr(out), ptr(rm))
    return out, rm


def synth_model_write(path, seed=1):
    """the seeded random-init POISD model written by the test side (oracle/synth_model.c); the same bytes as the
    product's vela_synth_model_write for the same seed"""
    rc = lib().or_synth_model_write(path.encode(), int(seed))
    if rc != 0:
        raise RuntimeError(f"oracle model writer failed ({rc}) for {path}")
    return path


class Model:
    """The oracle's UNet step on a POISD file (src/engine.cu semantics)."""

    def __init__(self, path):
        err = ctypes.create_string_buffer(256)
        self.h = lib().or_model_load(path.encode(), err, 256)
        if not self.h:
            raise RuntimeError("oracle model load: " + err.value.decode())

    def set_prompt(self, tokens):
        t = np.ascontiguousarray(tokens, np.int32)
        if lib().or_set_prompt(self.h, ptr(t), len(t)) != 0:
            raise RuntimeError("oracle: prompt too long")

    def context(self):
        p = lib().or_context(self.h)
        return np.ctypeslib.as_array(p, shape=(77, 1024)).copy()

    def step(self, seeds, taps=None):
        """seeds uint8 [B, 32] -> (x0 uint8 [B, 32768], eps int32 [B, 4096, 4]); taps: optional callable(name, int32 array)"""
        seeds = np.ascontiguousarray(seeds, np.uint8)
        B = seeds.shape[0]
        x0 = np.zeros((B, 32768), np.uint8); eps = np.zeros((B, 4096, 4), np.int32)
        TAP = ctypes.CFUNCTYPE(None, ctypes.c_void_p, ctypes.c_char_p, ctypes.POINTER(ctypes.c_int32), ctypes.c_size_t)
        cb = TAP(lambda u, name, data, n: taps(name.decode(), np.ctypeslib.as_array(data, shape=(n,)))) if taps else None
        rc = lib().or_unet_step(self.h, ptr(seeds), B, ptr(x0), ptr(eps), ctypes.cast(cb, ctypes.c_void_p) if cb else None, None)
        if rc != 0:
            raise RuntimeError("oracle: no prompt set")
        return x0, eps

    def close(self):
        if self.h:
            lib().or_model_free(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
