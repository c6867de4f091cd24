"""The C++ runtime (HTTP server, codecs, data loader) under AddressSanitizer + UndefinedBehaviorSanitizer
and under ThreadSanitizer: csrc/runtime/tests/selftest.cpp built with the runtime sources and run with
concurrent HTTP clients, the loader's prefetch thread and the codecs' round trips. Any sanitizer report
makes the executable fail."""
import os
import subprocess

import pytest


@pytest.mark.parametrize("sanitize,tag", [("address,undefined", "asan"), ("thread", "tsan")])
def test_runtime_selftest_under_sanitizer(tmp_path, sanitize, tag):
    from distrain_b200._build import build_runtime_selftest, sanitizer_cxx
    if sanitizer_cxx(sanitize) is None:
        pytest.skip(f"-fsanitize={sanitize} not available")
    exe = build_runtime_selftest(sanitize, tag)
    env = dict(os.environ)
    env["ASAN_OPTIONS"] = "detect_leaks=1:abort_on_error=0:halt_on_error=1:exitcode=23"
    env["UBSAN_OPTIONS"] = "halt_on_error=1:print_stacktrace=1:exitcode=24"
    env["TSAN_OPTIONS"] = "halt_on_error=1:exitcode=25:second_deadlock_stack=1"
    r = subprocess.run([exe, str(tmp_path)], capture_output=True, text=True, timeout=600, env=env)
    assert r.returncode == 0, f"exit {r.returncode}\n{r.stdout[-3000:]}\n{r.stderr[-6000:]}"
    assert "runtime selftest ok" in r.stdout
