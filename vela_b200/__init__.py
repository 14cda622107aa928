"""vela_b200: B200-native (sm_100a) exact-integer UNet step of the Vela PoI v2 miner.

The product is the C ABI in include/vela_b200.h, implemented by
libvela_b200.so (built in-tree from vela_b200/csrc/ by vela_b200.build).
This module is a thin ctypes view of that ABI for Python callers, tests and
bench.py; it holds no compute of its own.  On a machine without a GPU the
library still loads (host entry points work); device entry points return
VELA_ERR_CUDA.
"""
import ctypes
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libvela_b200.so")
_lib = None


class VelaError(RuntimeError):
    def __init__(self, code, msg):
        super().__init__(f"vela_b200 error {code}: {msg}")
        self.code = code


def lib():
    """Load libvela_b200.so (it must have been built: python -m vela_b200.build)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(f"{LIB_PATH} is missing: build it with `python -m vela_b200.build`")
        L = ctypes.CDLL(LIB_PATH)
        from . import abi
        abi.declare(L)
        _lib = L
    return _lib


def check(rc):
    if rc != 0:
        raise VelaError(rc, lib().vela_last_error().decode())
    return rc


def synth_model_write(path, seed=1):
    """Write the seeded random-init POISD model (SD-2.1 UNet + text encoder shapes) to `path`."""
    check(lib().vela_synth_model_write(path.encode(), int(seed)))
    return path
