"""The C ABI from a plain C program: tests/c_client/kv_kat.c is compiled with
gcc against include/*.h, linked to liblt_kv.so as the engine's FFI would link
it, and runs the reference's KvCache and SlotCache known-answer tests and its
scheduler's tests of KV behaviour (through lt_sched) on a bookkeeping-only
handle (no GPU)."""
import subprocess
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]


def test_c_client_runs_reference_known_answer_tests(tmp_path, native):
    from langtrain_studio_b200 import _native

    lib = Path(_native.library_path())
    exe = tmp_path / "kv_kat"
    subprocess.run(["gcc", "-std=c99", "-Wall", "-Werror", "-I", str(ROOT / "include"),
                    str(ROOT / "tests" / "c_client" / "kv_kat.c"), "-o", str(exe), str(lib),
                    f"-Wl,-rpath,{lib.parent}"], check=True)
    r = subprocess.run([str(exe)], capture_output=True, text=True, timeout=60)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "known-answer tests passed" in r.stdout
