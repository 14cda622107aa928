"""ctypes declarations of the C ABI in include/vela_b200.h (one entry per exported function)."""
import ctypes

P = ctypes.c_void_p
I = ctypes.c_int
U = ctypes.c_uint
LL = ctypes.c_longlong
SZ = ctypes.c_size_t
U64 = ctypes.c_uint64


class ASrc(ctypes.Structure):
    """vela_asrc"""
    _fields_ = [("src", I), ("hi", P), ("lo", P), ("ld8", I), ("e", P),
                ("x", P), ("ldx", I), ("rowmax", P), ("K", I),
                ("img", P), ("H", I), ("W", I), ("C", I), ("stride", I), ("Ho", I), ("Wo", I)]


class AEpi(ctypes.Structure):
    """vela_aepi"""
    _fields_ = [("epi", I), ("Y", P), ("ldy", I), ("residual", P),
                ("Cs", I), ("Y1", P), ("Y2", P), ("Lphi", P),
                ("rowmax", P),
                ("heads", I), ("T", I), ("TpQ", I), ("TpK", I), ("C", I),
                ("qhi", P), ("qlo", P), ("khi", P), ("klo", P), ("qe", P), ("ke", P),
                ("qhs", P), ("qls", P), ("qts", P), ("khs", P), ("kls", P), ("kts", P),
                ("workspace", P), ("workspace_bytes", SZ)]


SRC_I8, SRC_X32, SRC_CONV32 = 0, 1, 2
EPI_PLAIN, EPI_SPLIT3, EPI_GEGLU, EPI_GELU, EPI_QKV = 0, 1, 2, 3, 4

SIGNATURES = {
    "vela_last_error": (ctypes.c_char_p, []),
    "vela_version": (ctypes.c_char_p, []),
    "vela_device_error": (U, [I]),
    "vela_synth_model_write": (I, [ctypes.c_char_p, U64]),
    "vela_sha256d": (I, [P, SZ, P]),
    "vela_poi_out": (I, [P, P, P]),
    "vela_poi_out_batch": (I, [P, P, I, I, P]),
    "vela_share_hash": (I, [P, P, P]),
    "vela_gemm_w8a16": (I, [P, ctypes.POINTER(ASrc), I, I, P, I, I, I, I, P, ctypes.POINTER(AEpi)]),
    "vela_gemm_w8a16_stalled": (I, [P, ctypes.POINTER(ASrc), I, I, P, I, I, I, I, P, ctypes.POINTER(AEpi), LL]),
    "vela_gemm_hl": (I, [P, P, P, I, I, I, P, I, I, I, I, P, P, P, I, P, I, I, P, P, P]),
    "vela_conv_e": (I, [P, P, I, I, I, I, P]),
    "vela_quant_rows": (I, [P, P, I, I, I, P, P, P, I]),
    "vela_quant_rows_rm": (I, [P, P, P, I, I, I, P, P, P, I, I]),
    "vela_pixmax": (I, [P, P, I, I, P]),
    "vela_im2col3": (I, [P, P, P, I, I, I, I, I, P, P, P, I]),
    "vela_gn_stats": (I, [P, P, I, I, I, I, LL, P]),
    "vela_gn_apply_row": (I, [P, P, I, I, I, I, P, P, P, P, P, P, P, P, P, I]),
    "vela_lnorm_q": (I, [P, P, I, I, P, P, LL, P, P, P, I]),
    "vela_lnorm": (I, [P, P, I, I, P, P, LL, P]),
    "vela_act": (I, [P, P, SZ, P]),
    "vela_geglu": (I, [P, P, P, SZ, P]),
    "vela_add": (I, [P, P, P, SZ]),
    "vela_concat": (I, [P, P, I, P, I, I, P]),
    "vela_upsample2": (I, [P, P, I, I, I, I, P]),
    "vela_noise": (I, [P, P, I, P, LL, P, P]),
    "vela_finalize": (I, [P, P, P, I, LL, P]),
    "vela_text_embed": (I, [P, P, I, I, P, P, P, P, I, P]),
    "vela_quant_heads": (I, [P, P, I, I, I, I, I, P, P, P, P, P, P]),
    "vela_quant_heads_pad": (I, [P, I, I, I, P, P, P, P, P, P]),
    "vela_quant_v": (I, [P, P, I, I, I, I, I, P, P, P, P, P]),
    "vela_quant_v_static": (I, [P, P, I, I, I, I, I, P, P, P, P]),
    "vela_fused_attention": (I, [P] + [P] * 13 + [I] * 7 + [P, I, P, P, P, P]),
    "vela_fused_attention_stalled": (I, [P] + [P] * 13 + [I] * 7 + [P, I, P, P, LL]),
    "vela_model_load": (P, [I, ctypes.c_char_p]),
    "vela_model_load_memory": (P, [I, P, SZ]),
    "vela_model_free": (None, [P]),
    "vela_model_bytes": (SZ, [P]),
    "vela_engine_create": (P, [P, P]),
    "vela_engine_destroy": (None, [P]),
    "vela_engine_set_prompt": (I, [P, P, I]),
    "vela_engine_context": (I, [P, P]),
    "vela_engine_run": (I, [P, P, P]),
    "vela_engine_submit": (I, [P, P]),
    "vela_engine_collect": (I, [P, P]),
    "vela_engine_step_taps": (I, [P, P, P, P, P]),
    "vela_engine_launch_device": (I, [P, P, P]),
    "vela_engine_graph_kernels": (I, [P]),
    "vela_engine_device_error": (U, [P, I]),
    "vela_engine_test_attention": (LL, [P, I, I, I, I, I, I]),
    "vela_engine_in_flight": (I, [P]),
    "vela_engine_batch": (I, [P]),
    "vela_engine_arena_peak": (SZ, [P]),
    "vela_engine_stream": (P, [P]),
    "vela_engine_last_ms": (ctypes.c_double, [P]),
}


class EngineConfig(ctypes.Structure):
    """vela_engine_config"""
    _fields_ = [("batch", I), ("graph", I), ("arena_bytes", SZ)]


def declare(L):
    for name, (res, args) in SIGNATURES.items():
        f = getattr(L, name)
        f.restype = res
        f.argtypes = args
