"""The two writers of the seeded synthetic model give the same file.

The product writes the model its tests and bench load with vela_synth_model_write
(vela_b200/csrc/synth_model.cpp); the bench's reference arm writes its copy with the test
side's writer (oracle/synth_model.c) so that the reference process loads nothing of the
product.  Parity between the two engines rests on both reading the same bytes, so the whole
1.2 GB file is compared, for the bench's seed.
"""
import hashlib

import pytest

import vela_b200 as V
from oracle import pyoracle as O


def digest(path):
    h = hashlib.sha256()
    with open(path, "rb") as f:
        while True:
            b = f.read(1 << 24)
            if not b:
                return h.hexdigest()
            h.update(b)


@pytest.mark.parametrize("seed", [1])
def test_writers_agree(tmp_path, seed):
    a, b = str(tmp_path / "product.poisd"), str(tmp_path / "oracle.poisd")
    V.synth_model_write(a, seed)
    O.synth_model_write(b, seed)
    assert digest(a) == digest(b)
