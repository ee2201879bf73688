"""The CUDA-free core under AddressSanitizer and UndefinedBehaviorSanitizer:
`make sanitize` builds the core sources with a randomized self-test
(src/selftest/core_selftest.cc: plans simulated against their oracle for
every route, group-machine scripts, host folds, gates, fault policy,
summary, calibration JSON), which must finish with no sanitizer report and
every plan matching. This replaces compute-sanitizer for the host-side
layers."""
import os
import subprocess

import pytest

from conftest import REPO


def test_core_under_asan_ubsan():
    b = subprocess.run(["make", "-s", "sanitize"], cwd=REPO, capture_output=True, text=True, timeout=600)
    if b.returncode != 0 and ("lasan" in b.stderr or "asan_preinit" in b.stderr):
        pytest.skip("no AddressSanitizer runtime for this compiler")
    assert b.returncode == 0, b.stderr[-3000:]
    env = dict(os.environ, ASAN_OPTIONS="detect_leaks=1:abort_on_error=0",
               UBSAN_OPTIONS="print_stacktrace=1:halt_on_error=1")
    env.pop("LD_PRELOAD", None)
    r = subprocess.run([os.path.join(REPO, "_build", "core_selftest_san"), "3"], cwd=REPO, env=env,
                       capture_output=True, text=True, timeout=600)
    out = r.stdout + r.stderr
    assert r.returncode == 0, out[-4000:]
    assert "ERROR: AddressSanitizer" not in out and "runtime error" not in out, out[-4000:]
    assert "plans:" in out and " 0 failed" in out and out.strip().endswith("OK"), out[-2000:]
