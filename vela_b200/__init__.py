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


def _bytes_arg(b, n=None, what="buffer"):
    b = bytes(memoryview(b).cast("B")) if not isinstance(b, (bytes, bytearray)) else bytes(b)
    if n is not None and len(b) != n:
        raise ValueError(f"{what}: {n} bytes expected, got {len(b)}")
    return b


def sha256d(data):
    """SHA-256(SHA-256(data)) on the host (vela_sha256d)."""
    d = _bytes_arg(data)
    out = ctypes.create_string_buffer(32)
    check(lib().vela_sha256d(d, len(d), out))
    return out.raw


def poi_out(seed, x0):
    """The proof-of-inference hash of one inference: tagged SHA-256 "POI/out" over seed (32 bytes) and x0
    (32768 bytes, int16 little-endian), as the reference's miner computes it (vela_poi_out)."""
    out = ctypes.create_string_buffer(32)
    check(lib().vela_poi_out(_bytes_arg(seed, 32, "seed"), _bytes_arg(x0, 32768, "x0"), out))
    return out.raw


def poi_out_batch(seeds, x0, threads=4):
    """poi_out of every inference of a batch: seeds [batch][32] and x0 [batch][32768] (e.g. Engine.run's output),
    hashed on up to `threads` host threads; returns a list of 32-byte digests."""
    s, x = _bytes_arg(seeds), _bytes_arg(x0)
    batch = len(s) // 32
    if batch == 0 or len(s) != 32 * batch or len(x) != 32768 * batch:
        raise ValueError("poi_out_batch: seeds must be batch x 32 bytes and x0 batch x 32768 bytes")
    out = ctypes.create_string_buffer(32 * batch)
    check(lib().vela_poi_out_batch(s, x, batch, int(threads), out))
    return [out.raw[32 * b:32 * b + 32] for b in range(batch)]


def share_hash(header80, poi32):
    """The share hash sha256d(header[80] || poi[32]) the reference's miner compares with the pool target."""
    out = ctypes.create_string_buffer(32)
    check(lib().vela_share_hash(_bytes_arg(header80, 80, "header"), _bytes_arg(poi32, 32, "poi"), out))
    return out.raw


class Model:
    """Weights of one GPU (vela_model_load): a POISD file prepared for the tcgen05 kernels."""

    def __init__(self, path, device=0):
        self.h = lib().vela_model_load(int(device), path.encode())
        if not self.h:
            raise VelaError(-5, lib().vela_last_error().decode())
        self.device = device

    @property
    def bytes(self):
        return lib().vela_model_bytes(self.h)

    def close(self):
        if getattr(self, "h", None):
            lib().vela_model_free(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class Engine:
    """One lane: stream + arena + two graph slots (vela_engine_*).  Host numpy buffers in and out."""

    def __init__(self, model, batch=8, graph=True, arena_bytes=0):
        from .abi import EngineConfig
        import numpy as np
        self._np = np
        cfg = EngineConfig(int(batch), int(bool(graph)), int(arena_bytes))
        self.model = model
        self.h = lib().vela_engine_create(model.h, ctypes.byref(cfg))
        if not self.h:
            raise VelaError(-1, lib().vela_last_error().decode())
        self.batch = batch

    def set_prompt(self, tokens):
        t = self._np.ascontiguousarray(tokens, self._np.int32)
        check(lib().vela_engine_set_prompt(self.h, t.ctypes.data_as(ctypes.c_void_p), len(t)))

    def context(self):
        out = self._np.zeros((77, 1024), self._np.int32)
        check(lib().vela_engine_context(self.h, out.ctypes.data_as(ctypes.c_void_p)))
        return out

    def _seeds(self, seeds):
        s = self._np.ascontiguousarray(seeds, self._np.uint8)
        assert s.size == 32 * self.batch, "seeds must be [batch, 32] bytes"
        return s

    def run(self, seeds):
        s = self._seeds(seeds)
        x0 = self._np.zeros((self.batch, 32768), self._np.uint8)
        check(lib().vela_engine_run(self.h, s.ctypes.data_as(ctypes.c_void_p), x0.ctypes.data_as(ctypes.c_void_p)))
        return x0

    def submit(self, seeds):
        s = self._seeds(seeds)
        check(lib().vela_engine_submit(self.h, s.ctypes.data_as(ctypes.c_void_p)))

    def collect(self, out=None):
        x0 = out if out is not None else self._np.zeros((self.batch, 32768), self._np.uint8)
        check(lib().vela_engine_collect(self.h, x0.ctypes.data_as(ctypes.c_void_p)))
        return x0

    def step_taps(self, seeds, tap):
        """one eager step; tap(name, int32 numpy array) for every block output"""
        s = self._seeds(seeds)
        x0 = self._np.zeros((self.batch, 32768), self._np.uint8)
        TAP = ctypes.CFUNCTYPE(None, ctypes.c_void_p, ctypes.c_char_p, ctypes.POINTER(ctypes.c_int32), ctypes.c_size_t)
        cb = TAP(lambda u, name, data, n: tap(name.decode(), self._np.ctypeslib.as_array(data, shape=(n,))))
        check(lib().vela_engine_step_taps(self.h, s.ctypes.data_as(ctypes.c_void_p), x0.ctypes.data_as(ctypes.c_void_p),
                                          ctypes.cast(cb, ctypes.c_void_p), None))
        return x0

    def launch_device(self, d_seeds, d_x0):
        """enqueue one step on device-resident seeds / x0 (device addresses as ints); returns without waiting"""
        check(lib().vela_engine_launch_device(self.h, ctypes.c_void_p(d_seeds), ctypes.c_void_p(d_x0)))

    @property
    def stream(self):
        """the engine's cudaStream_t, as an int"""
        return lib().vela_engine_stream(self.h) or 0

    @property
    def graph_kernels(self):
        return lib().vela_engine_graph_kernels(self.h)

    def device_error(self, clear=True):
        """the engine's device error word (non-zero: one of its kernels gave up a bounded wait); clear resets it"""
        return lib().vela_engine_device_error(self.h, int(bool(clear)))

    @property
    def last_ms(self):
        return lib().vela_engine_last_ms(self.h)

    @property
    def arena_peak(self):
        return lib().vela_engine_arena_peak(self.h)

    def close(self):
        if getattr(self, "h", None):
            lib().vela_engine_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
