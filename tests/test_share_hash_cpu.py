"""Host share hashing through the C ABI (CPU only) against Python's hashlib, on the reference's definitions:
poi_out = the tagged hash "POI/out" over seed[32] || x0[32768] (src/main.cpp:79, src/sha256.h:86-91) and the
share hash = sha256d(header[80] || poi_out) (src/main.cpp:263-264); sha256d at padding and block boundaries
(the sizes of the reference's src/test_sha256.cpp)."""
import ctypes
import hashlib
import os

import numpy as np
import pytest

import vela_b200 as V

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def sha256(b):
    return hashlib.sha256(b).digest()


def tagged(tag, msg):
    t = sha256(tag)
    return sha256(t + t + msg)


def buf(b):
    return ctypes.c_char_p(bytes(b))


@pytest.fixture(scope="module")
def L():
    return V.lib()


def test_sha256d_boundaries(L):
    rng = np.random.default_rng(2917)
    data = rng.integers(0, 256, 131072, dtype=np.uint8).tobytes()
    sizes = [0, 1, 31, 32, 55, 56, 63, 64, 65, 80, 112, 127, 128, 129, 32768, 32864, 131072] + list(rng.integers(0, 131072, 40))
    out = ctypes.create_string_buffer(32)
    for n in sizes:
        n = int(n)
        assert L.vela_sha256d(buf(data[:n]), n, out) == 0
        assert out.raw == sha256(sha256(data[:n])), n
    assert sha256(b"abc").hex() == "ba7816bf8f01cfea414140de5dae2223b00361a396177a9cb410ff61f20015ad"


def test_poi_out_and_share_hash(L):
    rng = np.random.default_rng(7)
    B = 5
    seeds = rng.integers(0, 256, (B, 32), dtype=np.uint8)
    x0 = rng.integers(0, 256, (B, 32768), dtype=np.uint8)
    want = [tagged(b"POI/out", seeds[b].tobytes() + x0[b].tobytes()) for b in range(B)]
    one = ctypes.create_string_buffer(32)
    for b in range(B):
        assert L.vela_poi_out(buf(seeds[b]), buf(x0[b]), one) == 0
        assert one.raw == want[b]
    for threads in (1, 3, 8):
        outb = ctypes.create_string_buffer(32 * B)
        assert L.vela_poi_out_batch(buf(seeds), buf(x0), B, threads, outb) == 0
        assert [outb.raw[32 * b:32 * b + 32] for b in range(B)] == want
    header = rng.integers(0, 256, 80, dtype=np.uint8).tobytes()
    sh = ctypes.create_string_buffer(32)
    assert L.vela_share_hash(buf(header), buf(want[0]), sh) == 0
    assert sh.raw == sha256(sha256(header + want[0]))


def test_null_pointers_are_errors(L):
    out = ctypes.create_string_buffer(32)
    assert L.vela_poi_out(None, None, out) != 0
    assert b"poi_out" in L.vela_last_error()
    assert L.vela_share_hash(None, None, None) != 0


def test_reference_digests(L, golden):
    """tests/golden/share_hash.npz: the reference's own hashing (src/sha256.h) on the reference engine's golden x0
    and on seeded inputs (tests/golden/make_share_hash.py)."""
    g = golden("share_hash")
    B = g["seeds"].shape[0]
    outb = ctypes.create_string_buffer(32 * B)
    assert L.vela_poi_out_batch(buf(g["seeds"]), buf(g["x0"]), B, 4, outb) == 0
    assert np.array_equal(np.frombuffer(outb.raw, np.uint8).reshape(B, 32), g["poi"])
    sh = ctypes.create_string_buffer(32)
    for b in range(B):
        assert L.vela_share_hash(buf(g["headers"][b]), buf(g["poi"][b]), sh) == 0
        assert np.array_equal(np.frombuffer(sh.raw, np.uint8), g["share"][b])


def test_python_helpers(golden):
    """vela_b200.poi_out / poi_out_batch / share_hash / sha256d (the Python view of the same entry points)"""
    g = golden("share_hash")
    B = g["seeds"].shape[0]
    assert V.poi_out(g["seeds"][0], g["x0"][0]) == g["poi"][0].tobytes()
    assert V.poi_out_batch(g["seeds"], g["x0"], threads=2) == [g["poi"][b].tobytes() for b in range(B)]
    assert V.share_hash(g["headers"][1], g["poi"][1]) == g["share"][1].tobytes()
    assert V.sha256d(b"abc") == sha256(sha256(b"abc"))
    with pytest.raises(ValueError):
        V.poi_out(b"short", g["x0"][0])
