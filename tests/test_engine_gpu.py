"""The whole UNet step on the B200 (vela_engine_* through the C ABI) vs the REFERENCE engine.

tests/golden/engine.npz and engine_taps.json hold, for the synthetic model of seed 1 and the
prompt {320, 736, 3240}: the reference engine's text-encoder context, the sha256 of every block
output of its UNet (src/engine.cu:455-490 order) and its x0 bytes for two seeds, eager and from
its CUDA graph.  Our engine must reproduce all of them bit for bit, through the graph and the
two-slot submit / collect pipeline too.
"""
import hashlib
import json
import os

import numpy as np
import pytest

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")
if not torch.cuda.is_available():
    pytest.skip("no CUDA device", allow_module_level=True)

import vela_b200 as V  # noqa: E402

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


@pytest.fixture(scope="module")
def model(synth_model_path):
    m = V.Model(synth_model_path)
    yield m
    m.close()


def test_engine_matches_reference_engine(model):
    e = np.load(os.path.join(GOLDEN, "engine.npz"))
    taps = json.load(open(os.path.join(GOLDEN, "engine_taps.json")))
    eng = V.Engine(model, batch=2, graph=True)
    eng.set_prompt([320, 736, 3240])
    assert np.array_equal(eng.context(), e["ctx"]), "text encoder context"
    got = {}
    x0 = eng.step_taps(e["seeds"], lambda n, a: got.__setitem__(n, hashlib.sha256(a.tobytes()).hexdigest()))
    assert list(got) == list(taps)
    bad = [k for k in taps if got[k] != taps[k]]
    assert not bad, f"first differing block: {bad[0]} ({len(bad)} differ)"
    assert np.array_equal(x0, e["x0"])
    assert np.array_equal(eng.run(e["seeds"]), e["x0"]), "graph replay"
    eng.submit(e["seeds"]); eng.submit(e["seeds"][::-1].copy())
    a, b = eng.collect(), eng.collect()
    assert np.array_equal(a, e["x0"]) and np.array_equal(b, e["x0"][::-1]), "submit/collect pipeline"
    assert V.lib().vela_device_error(1) == 0
    eng.close()


def test_batch_lanes_agree(model):
    """every batch lane computes the same x0 for the same seed (the reference's --check property)"""
    e = np.load(os.path.join(GOLDEN, "engine.npz"))
    eng = V.Engine(model, batch=8, graph=True)
    eng.set_prompt([320, 736, 3240])
    seeds = np.repeat(e["seeds"][:1], 8, axis=0)
    x0 = eng.run(seeds)
    for b in range(8):
        assert np.array_equal(x0[b], e["x0"][0]), b
    eng.close()
