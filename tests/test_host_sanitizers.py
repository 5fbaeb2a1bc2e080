"""The C++ host cores under AddressSanitizer + UndefinedBehaviorSanitizer.

Reference: scripts/validate-*-sanitizer.sh run each native C translation unit
under ASan/UBSan through standalone probes.  Here the header-only cores of
csrc/host/ are compiled with the sanitizers into a standalone self-test
(csrc/host/selftest/host_selftest.cpp) and run; any report fails the test.
"""
import os
import shutil
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.mark.skipif(shutil.which("g++") is None, reason="needs g++")
def test_host_cores_under_asan_ubsan(tmp_path):
    exe = tmp_path / "host_selftest"
    cmd = ["g++", "-std=c++20", "-O1", "-g", "-fsanitize=address,undefined", "-fno-sanitize-recover=all",
           "-fno-omit-frame-pointer", "-I", os.path.join(ROOT, "csrc", "host"),
           os.path.join(ROOT, "csrc", "host", "selftest", "host_selftest.cpp"), "-o", str(exe)]
    b = subprocess.run(cmd, capture_output=True, text=True, timeout=300)
    assert b.returncode == 0, b.stderr[-3000:]
    scratch = tmp_path / "root"
    scratch.mkdir()
    env = dict(os.environ, ASAN_OPTIONS="detect_leaks=1:abort_on_error=0", UBSAN_OPTIONS="print_stacktrace=1")
    r = subprocess.run([str(exe), str(scratch)], capture_output=True, text=True, timeout=300, env=env)
    assert r.returncode == 0, (r.stdout + r.stderr)[-3000:]
    assert "host selftest ok" in r.stdout
