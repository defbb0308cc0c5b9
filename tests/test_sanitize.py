"""The host side of the C ABI under AddressSanitizer + UndefinedBehaviorSanitizer:
tests/sanitize/Makefile builds the library with both in its host code and
links tests/sanitize/abi_host.cpp, which drives a host-only context (page and
sequence bookkeeping, decode protocol, prefix rule and table, argument
errors).  compute-sanitizer is closed on the GPU pool; this covers the host
code, and the device code's bounds are checked by its error word instead."""
import os
import subprocess

import pytest

HERE = os.path.join(os.path.dirname(os.path.abspath(__file__)), "sanitize")


def test_host_abi_under_asan_ubsan():
    if not os.path.exists("/usr/bin/g++"):
        pytest.skip("no system g++ with sanitizer runtimes")
    b = subprocess.run(["make", "-s", "-j8", "-C", HERE], capture_output=True, text=True)
    if b.returncode != 0 and "cannot find -lasan" in (b.stdout + b.stderr):
        pytest.skip("the sanitizer runtime is not installed")
    assert b.returncode == 0, b.stdout[-2000:] + b.stderr[-2000:]
    r = subprocess.run([os.path.join(HERE, "_build", "abi_host")], capture_output=True, text=True,
                       env=dict(os.environ, ASAN_OPTIONS="detect_leaks=1:halt_on_error=1",
                                UBSAN_OPTIONS="print_stacktrace=1:halt_on_error=1"))
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    assert "ok" in r.stdout
