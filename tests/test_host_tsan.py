"""ThreadSanitizer run of the C++ host control plane (CPU only).

Builds csrc/host/*.cc with -fsanitize=thread together with a native driver
(csrc/host/tests/tsan_driver.cc) that runs in-process clusters on threads:
collectives over plain TCP and over TLS, concurrent non-blocking all-reduces,
point-to-point traffic, and a rank failure handled by automatic recovery.
Any ThreadSanitizer report fails the test."""
import glob
import os
import shutil
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.mark.skipif(shutil.which("g++") is None, reason="needs g++")
def test_host_control_plane_has_no_data_races(tmp_path):
    srcs = [s for s in sorted(glob.glob(os.path.join(ROOT, "csrc", "host", "*.cc"))) if not s.endswith("bindings.cc")]
    exe = str(tmp_path / "tsan_driver")
    cmd = ["g++", "-std=c++17", "-O1", "-g", "-fsanitize=thread", "-I", os.path.join(ROOT, "csrc", "host"), *srcs,
           os.path.join(ROOT, "csrc", "host", "tests", "tsan_driver.cc"), "-lssl", "-lcrypto", "-pthread", "-o", exe]
    b = subprocess.run(cmd, capture_output=True, text=True, timeout=600)
    if b.returncode != 0 and "tsan" in (b.stderr or "").lower():
        pytest.skip("ThreadSanitizer runtime not available: " + b.stderr[-300:])
    assert b.returncode == 0, b.stderr[-2000:]
    r = subprocess.run([exe], capture_output=True, text=True, timeout=600)
    out = (r.stdout or "") + (r.stderr or "")
    assert "WARNING: ThreadSanitizer" not in out, out[-6000:]
    assert r.returncode == 0 and "tsan driver: ok" in out, out[-3000:]
