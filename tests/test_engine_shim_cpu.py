"""The C++ engine API (include/vela_b200_engine.hpp) compiles against the C ABI header, links against the built
libvela_b200.so and reports failures as exceptions, like the reference's engine classes (CPU only)."""
import os
import shutil
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
LIBDIR = os.path.join(ROOT, "vela_b200")


@pytest.mark.skipif(shutil.which("g++") is None, reason="no C++ compiler")
def test_engine_shim_builds_and_reports_errors(tmp_path):
    if not os.path.exists(os.path.join(LIBDIR, "libvela_b200.so")):
        pytest.skip("libvela_b200.so not built")
    exe = str(tmp_path / "engine_shim_check")
    cmd = ["g++", "-std=c++17", "-O1", "-Wall", "-Werror", "-I", os.path.join(ROOT, "include"),
           os.path.join(ROOT, "tests", "host", "engine_shim_check.cpp"), "-o", exe,
           "-L", LIBDIR, "-lvela_b200", "-Wl,-rpath," + LIBDIR]
    r = subprocess.run(cmd, capture_output=True, text=True)
    assert r.returncode == 0, r.stdout + r.stderr
    r = subprocess.run([exe, str(tmp_path / "missing.poisd")], capture_output=True, text=True, timeout=120)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "image load refused" in r.stdout and "load refused" in r.stdout and "engine refused" in r.stdout


REF = os.path.abspath(os.path.join(ROOT, "..", "reference"))


@pytest.mark.skipif(not os.path.exists(os.path.join(REF, "src", "main.cpp")), reason="the reference checkout is not present")
@pytest.mark.skipif(shutil.which("g++") is None, reason="no C++ compiler")
def test_reference_host_builds_on_the_header():
    """the reference's own src/main.cpp, unmodified, with its poisd / stratum / httpd / device sources, compiles against
    include/reference_host/engine.h (-> vela_b200_engine.hpp) and links libvela_b200.so, with no cuBLASLt"""
    if not os.path.exists(os.path.join(LIBDIR, "libvela_b200.so")):
        pytest.skip("libvela_b200.so not built")
    r = subprocess.run(["make", "-s", "-C", os.path.join(ROOT, "oracle"), "_ref/meow_host", f"REF={REF}"], capture_output=True, text=True)
    assert r.returncode == 0, r.stdout + r.stderr
    exe = os.path.join(ROOT, "oracle", "_ref", "meow_host")
    deps = subprocess.run(["ldd", exe], capture_output=True, text=True).stdout
    assert "libvela_b200.so" in deps and "cublas" not in deps, deps
    r = subprocess.run([exe, "--help"], capture_output=True, text=True, timeout=60)
    assert r.returncode == 0 and "supr-meow-vela" in r.stdout
