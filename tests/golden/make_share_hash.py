"""Fixture for the host share hashing: digests computed by the REFERENCE's own hashing (src/sha256.h through
oracle/_ref/ref_share_hash, built by `make -C oracle ref`) on the reference engine's golden x0 (engine.npz) and on
seeded random inputs.  Run here (it needs the reference checkout's build); writes tests/golden/share_hash.npz."""
import os
import subprocess
import tempfile

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
EXE = os.path.join(ROOT, "oracle", "_ref", "ref_share_hash")


def main():
    e = np.load(os.path.join(HERE, "engine.npz"))
    rng = np.random.default_rng(31)
    seeds = np.concatenate([e["seeds"].reshape(-1, 32), rng.integers(0, 256, (3, 32), dtype=np.uint8)]).astype(np.uint8)
    x0 = np.concatenate([e["x0"].reshape(-1, 32768), rng.integers(0, 256, (3, 32768), dtype=np.uint8)]).astype(np.uint8)
    B = seeds.shape[0]
    headers = rng.integers(0, 256, (B, 80), dtype=np.uint8)
    with tempfile.TemporaryDirectory() as td:
        fi, fo = os.path.join(td, "in.bin"), os.path.join(td, "out.bin")
        with open(fi, "wb") as f:
            f.write(np.uint32(B).tobytes()); f.write(seeds.tobytes()); f.write(x0.tobytes()); f.write(headers.tobytes())
        subprocess.run([EXE, fi, fo], check=True)
        out = np.frombuffer(open(fo, "rb").read(), np.uint8).reshape(2, B, 32)
    np.savez_compressed(os.path.join(HERE, "share_hash.npz"), seeds=seeds, x0=x0, headers=headers, poi=out[0], share=out[1])


if __name__ == "__main__":
    main()
