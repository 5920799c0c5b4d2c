"""The host side of the library under AddressSanitizer and
UndefinedBehaviorSanitizer.

The reference has no sanitizer runs of its own (its pool's `unsafe` blocks
are argued in comments, `pool.rs:36-39`).  Here the C++ bookkeeping, the
scheduler driver and the ABI glue are rebuilt with -fsanitize=address,undefined
(liblt_kv_asan.so, `build.py` variant "asan") and the CPU bookkeeping suites
-- the reference's known-answer tests, error paths, random operation
sequences against the oracle (fixed seeds and a hypothesis state machine), the scheduler driver against its Python
restatement, the prefix cache with token-level admission, and the plain C
client of the ABI -- run against it in a child process with libasan
preloaded (the C client inherits the preload).
Any report aborts the child (halt_on_error), which fails this test.
"""
from __future__ import annotations

import os
import subprocess
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT))

from langtrain_studio_b200 import build  # noqa: E402

CHILD = r"""
import sys
import pytest
from langtrain_studio_b200 import _native
_native.lib()
maps = open("/proc/self/maps").read()
assert "liblt_kv_asan.so" in maps, "the sanitized library is not the one loaded"
assert "libasan" in maps and "libubsan" in maps, "sanitizer runtimes not loaded"
sys.exit(pytest.main(["-q", "-m", "not gpu", "-p", "no:cacheprovider", "tests/test_abi.py", "tests/test_sched.py",
                      "tests/test_prefix.py", "tests/test_c_client.py", "tests/test_abi_stateful.py",
                      "tests/test_prefix_stateful.py", "tests/test_sched_stateful.py",
                      "tests/test_sched_length_stateful.py"]))
"""


def _libasan() -> str | None:
    try:
        out = subprocess.run(["gcc", "-print-file-name=libasan.so"], capture_output=True, text=True, check=True)
    except (OSError, subprocess.CalledProcessError):
        return None
    path = out.stdout.strip()
    return path if os.path.isabs(path) and os.path.exists(path) else None


def test_bookkeeping_under_asan_and_ubsan():
    asan = _libasan()
    if asan is None:
        pytest.skip("gcc's libasan is not installed")
    lib = build.build(variant="asan")
    syms = subprocess.run(["nm", "-D", "--undefined-only", str(lib)], capture_output=True, text=True, check=True)
    assert "__asan_" in syms.stdout and "__ubsan_" in syms.stdout, "library is not instrumented"
    env = dict(os.environ, LT_KV_VARIANT="asan", LD_PRELOAD=asan,
               ASAN_OPTIONS="detect_leaks=0:halt_on_error=1:abort_on_error=1",
               UBSAN_OPTIONS="halt_on_error=1:print_stacktrace=1", PYTHONPATH=str(ROOT))
    r = subprocess.run([sys.executable, "-c", CHILD], cwd=ROOT, env=env, capture_output=True, text=True,
                       timeout=600)
    tail = (r.stdout + r.stderr)[-4000:]
    assert r.returncode == 0, tail
    assert " passed" in r.stdout and "failed" not in r.stdout, tail
