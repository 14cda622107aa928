"""The reference's own host program running on vela_b200 (the drop-in at the engine API).

oracle/_ref/meow_host is the reference's src/main.cpp, unmodified, with its poisd / stratum / httpd / device
sources, built against include/vela_b200_engine.hpp and linked to libvela_b200.so (oracle/Makefile, target
_ref/meow_host; it is built where the reference checkout is present and travels prebuilt).  Its own modes run here:
--seed (one inference through runSingle: DevModel::load with the parsed model, setPrompt, run), --test-attn (its
attention checks through Engine::testAttention) and --bench (runBench: lanes of submit / collect).  The x0 of the
golden seed must be the reference engine's x0 byte for byte.
"""
import os
import re
import subprocess

import numpy as np
import pytest

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")
if not torch.cuda.is_available():
    pytest.skip("no CUDA device", allow_module_level=True)

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HOST = os.path.join(ROOT, "oracle", "_ref", "meow_host")
GOLDEN = os.path.join(ROOT, "tests", "golden")
if not os.path.exists(HOST):
    pytest.skip("oracle/_ref/meow_host is not built (make -C oracle ref where the reference checkout is present)", allow_module_level=True)


def host(args, timeout=600):
    r = subprocess.run([HOST] + args, capture_output=True, text=True, timeout=timeout)
    return r.returncode, r.stdout + r.stderr


def test_seed_run_matches_reference_engine(synth_model_path, tmp_path):
    g = np.load(os.path.join(GOLDEN, "engine.npz"))
    out = tmp_path / "x0.hex"
    rc, log = host(["--model", synth_model_path, "--devices", "0", "--batch", "2", "--tokens", "320,736,3240",
                    "--seed", bytes(g["seeds"][0]).hex(), "--x0-out", str(out)])
    assert rc == 0, log
    x0 = bytes.fromhex(out.read_text())
    assert x0 == bytes(g["x0"][0]), "the reference host's x0 on vela_b200 differs from the reference engine's"
    assert "sha256(x0)" in log


def test_attention_self_checks(synth_model_path):
    rc, log = host(["--model", synth_model_path, "--devices", "0", "--test-attn"])
    lines = [ln for ln in log.splitlines() if "test-attn" in ln]
    assert len(lines) == 17, log
    assert all(ln.endswith(": OK") for ln in lines), "\n".join(lines)
    assert rc == 0, log


def test_bench_mode(synth_model_path):
    rc, log = host(["--model", synth_model_path, "--devices", "0", "--batch", "8", "--lanes", "2", "--bench", "5"])
    assert rc == 0, log
    m = re.search(r"GPU 0: (\d+) inferences in ([0-9.]+) s = ([0-9.]+) inf/s", log)
    assert m, log
    assert int(m.group(1)) == 5 * 8 * 2 and float(m.group(3)) > 0
