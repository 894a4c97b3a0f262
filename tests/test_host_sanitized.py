"""The host C code (the reference API: loader, JSON reader, tokenizer, sampler stream, tensor helpers)
built under AddressSanitizer and UndefinedBehaviorSanitizer and driven through its CPU paths
(tests/host_sanitized_driver.py) in a child process that preloads the gcc sanitizer runtimes.  No GPU:
no path the driver takes initialises CUDA."""
import os
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_host_code_under_asan_and_ubsan(tmp_path):
    from diolkos_b200 import build as B

    runtimes = B.sanitizer_runtimes()
    if not runtimes:
        pytest.skip("this gcc has no ASan / UBSan runtime")
    lib = B.build_sanitized()
    env = {
        **os.environ,
        "LD_PRELOAD": ":".join(runtimes),
        # leaks: Python's own allocations at exit; odr / mismatch: the uninstrumented libraries around it
        "ASAN_OPTIONS": "detect_leaks=0:protect_shadow_gap=0:detect_odr_violation=0:alloc_dealloc_mismatch=0:halt_on_error=1",
        "UBSAN_OPTIONS": "halt_on_error=1:print_stacktrace=1",
        "PYTHONPATH": ROOT,
    }
    r = subprocess.run([sys.executable, os.path.join(ROOT, "tests", "host_sanitized_driver.py"), lib, str(tmp_path)],
                       env=env, capture_output=True, text=True, timeout=900)
    tail = (r.stdout[-2000:] + r.stderr[-6000:])
    assert "AddressSanitizer" not in r.stderr and "runtime error" not in r.stderr, tail
    assert r.returncode == 0 and "host code ok" in r.stdout, tail
