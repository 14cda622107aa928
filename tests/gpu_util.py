"""Helpers for the -m gpu tests: device buffers through torch (plumbing only), pointers for the C ABI."""
import ctypes

import numpy as np

try:
    import torch
except ImportError:  # pragma: no cover
    torch = None


class Dev:
    """Keeps every device buffer of a test alive until the test ends."""

    def __init__(self):
        self.keep = []

    def __call__(self, a):
        t = torch.from_numpy(np.ascontiguousarray(a)).cuda()
        self.keep.append(t)
        return t

    def empty(self, shape, dtype, fill=None):
        t = torch.empty(shape, dtype=dtype, device="cuda")
        if fill is not None:
            t.view(torch.uint8).fill_(fill)
        self.keep.append(t)
        return t

    def zeros(self, shape, dtype):
        t = torch.zeros(shape, dtype=dtype, device="cuda")
        self.keep.append(t)
        return t


def P(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


def A(t):
    """int value of a device pointer for ctypes Structure fields"""
    return None if t is None else t.data_ptr()


def H(t):
    torch.cuda.synchronize()
    return t.cpu().numpy()


def rbits(rng, shape, maxbits=31):
    bits = rng.integers(1, maxbits + 1, size=shape).astype(np.int64)
    x = rng.integers(0, 2**62, size=shape, dtype=np.int64)
    return ((x & ((np.int64(1) << bits) - 1)) - (np.int64(1) << (bits - 1))).astype(np.int32)


def cst_for(rng, W, N, Np):
    c = np.zeros((Np, 4), np.int32)
    c[:N, 0] = rng.integers(16384, 32768, N)
    c[:N, 1] = rng.integers(20, 30, N)
    c[:N, 2] = rng.integers(-50000, 50000, N)
    c[:N, 3] = W[:N, :].astype(np.int64).sum(1)
    return c
