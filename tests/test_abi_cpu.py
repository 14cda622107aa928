"""The C ABI without a GPU: libvela_b200.so loads, exports every entry point that include/vela_b200.h declares
(with the signatures vela_b200.abi gives ctypes), and rejects malformed arguments on the host with VELA_ERR_ARG
and a message, before any device work (the reference's shape guards, src/engine.cu:108, src/gemm_hl.cu:317-330)."""
import ctypes
import os
import re

import pytest

import vela_b200 as V
from vela_b200 import abi

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "vela_b200.h")


def declared():
    return sorted(set(re.findall(r"\b(vela_[a-z0-9_]+)\s*\(", open(HEADER).read())))


def test_header_and_table_agree():
    assert declared() == sorted(abi.SIGNATURES), "include/vela_b200.h and vela_b200/abi.py list different entry points"


def test_library_exports_every_declared_symbol():
    L = ctypes.CDLL(V.LIB_PATH)
    missing = [n for n in declared() if not hasattr(L, n)]
    assert not missing, missing


def test_status_codes_match_header():
    h = open(HEADER).read()
    codes = dict((k, int(v)) for k, v in re.findall(r"#define (VELA_(?:OK|ERR_[A-Z]+))\s+(-?\d+)", h))
    assert codes["VELA_OK"] == 0 and codes["VELA_ERR_ARG"] == -1 and codes["VELA_ERR_CUDA"] == -2
    assert len(set(codes.values())) == len(codes)


def test_version_string():
    assert V.lib().vela_version().decode().startswith("vela_b200")


def test_struct_layouts_match_header():
    """ctypes mirrors of vela_asrc / vela_aepi / vela_engine_config have the C sizes (LP64)"""
    assert ctypes.sizeof(abi.EngineConfig) == 16
    assert ctypes.sizeof(abi.ASrc) % 8 == 0 and ctypes.sizeof(abi.AEpi) % 8 == 0
    assert abi.AEpi.workspace_bytes.offset == ctypes.sizeof(abi.AEpi) - 8


@pytest.mark.parametrize("case", ["null_src", "bad_src_kind", "k_not_multiple_of_16", "qkv_without_heads"])
def test_gemm_rejects_bad_arguments(case):
    L = V.lib()
    a = abi.ASrc(); E = abi.AEpi()
    a.src = abi.SRC_I8; a.hi = 16; a.lo = 32; a.ld8 = 64; a.e = 48
    E.epi = abi.EPI_PLAIN; E.Y = 64; E.ldy = 64
    Mp, M, Np, N, Kp = 128, 100, 64, 64, 64
    if case == "null_src":
        rc = L.vela_gemm_w8a16(None, None, Mp, M, 8, Kp, Np, N, Kp, 8, ctypes.byref(E))
    else:
        if case == "bad_src_kind":
            a.src = 7
        elif case == "k_not_multiple_of_16":
            Kp = 40; a.ld8 = 40
        elif case == "qkv_without_heads":
            E.epi = abi.EPI_QKV
        rc = L.vela_gemm_w8a16(None, ctypes.byref(a), Mp, M, 8, Kp, Np, N, Kp, 8, ctypes.byref(E))
    assert rc == -1, (case, rc, L.vela_last_error())
    assert L.vela_last_error().decode()


def test_attention_rejects_bad_shapes():
    L = V.lib()
    p = ctypes.c_void_p(16)
    # Tqp not a multiple of 64
    rc = L.vela_fused_attention(None, p, p, p, p, p, p, p, p, p, p, p, p, p, 1, 1, 100, 100, 64, 64, 0, p, 64, None, None, p, p)
    assert rc == -1 and L.vela_last_error().decode()


def test_engine_rejects_null_model():
    cfg = abi.EngineConfig(8, 1, 0)
    assert not V.lib().vela_engine_create(None, ctypes.byref(cfg))
    assert "model" in V.lib().vela_last_error().decode()


def test_model_load_missing_file():
    with pytest.raises(V.VelaError):
        V.Model("/nonexistent/vela.poisd")
