"""Failure paths on the GPU, made to happen without faulting or hanging it.

The reference's path has no device code, so its failure handling is host
errors only (`kv.rs:67-74`, `kv.rs:87-92`, ported in test_abi.py).  The
kernels add two device-side paths, both tested here:

- Bounded waits.  Every wait in the kernels (bulk-copy barriers, the
  stream-K merge's neighbour flags) gives up after its limit, raises the
  handle's error flag and returns.  `lt_kv_selftest_wait` runs that wait on
  a flag that nothing sets with a short limit; the test checks the status
  (LT_E_TIMEOUT), that it clears, and that the handle keeps working.
- Bounds checks (debug build liblt_kv_checked.so, -DLT_BOUNDS_CHECK).  Run
  in a child process: the parity suite against the checked build, then a
  block-table entry overwritten with an id past the layer's blocks (inside
  the two-layer allocation), which the checked kernel redirects to block 0
  and reports as LT_E_BOUNDS.  The child first
  asserts that the checked library is the one loaded.
"""
from __future__ import annotations

import os
import subprocess
import sys
import time
from pathlib import Path

import numpy as np
import pytest

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu

ROOT = Path(__file__).resolve().parents[1]
ATOL, RTOL = 2e-3, 1e-3  # north-star attention tolerance


@pytest.fixture(scope="module", autouse=True)
def _need_cuda():
    if not torch.cuda.is_available():
        pytest.fail("CUDA device required for -m gpu tests")


def _filled(oracle_mod, lens, hq=32, hkv=8, d=128, seed=0, n_layers=1):
    """A cache with `lens` tokens per sequence, rows written in layer 0."""
    from langtrain_studio_b200.kv import KvCache

    kv = KvCache(n_layers, hkv, d, 16 * 64, n_heads=hq, max_seqs=len(lens), max_batch=1024, device=0)
    ok = oracle_mod.OracleKv(n_layers, hkv * d, 16 * 64, max_seqs=len(lens))
    rng = np.random.default_rng(seed)
    for s, n in enumerate(lens):
        seqs, pos = np.full(n, s), np.arange(n)
        b, sl = kv.append_batch(seqs, pos)
        ok.append_batch(seqs, pos)
        k = rng.standard_normal((n, hkv * d)).astype(np.float32)
        v = rng.standard_normal((n, hkv * d)).astype(np.float32)
        kv.write(0, b, sl, torch.from_numpy(k).cuda(), torch.from_numpy(v).cuda())
        ok.write_batch(0, b, sl, k, v)
    return kv, ok, rng


def _attend_matches(kv, ok, rng, lens, hq=32, hkv=8, d=128):
    seqs, pos = np.arange(len(lens)), np.array(lens) - 1
    q = rng.standard_normal((len(lens), hq * d)).astype(np.float32)
    out = kv.attend(0, torch.from_numpy(q).cuda(), seqs, pos, out_dtype=torch.float32)
    kv.check()
    ref = ok.attend(0, q, seqs, pos, hq, hkv, d)
    np.testing.assert_allclose(out.cpu().numpy(), ref, rtol=1e-4, atol=2e-5)


def test_bounded_wait_runs_out_reports_timeout_and_handle_recovers(oracle_mod):
    from langtrain_studio_b200 import _native as N
    from langtrain_studio_b200.kv import KvError

    lens = [37, 300]
    kv, ok, rng = _filled(oracle_mod, lens)
    _attend_matches(kv, ok, rng, lens)
    for limit_us in (20_000, 5_000):
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        kv.selftest_wait(limit_us)
        with pytest.raises(KvError) as e:
            kv.check()
        waited = time.perf_counter() - t0
        assert e.value.code == N.LT_E_TIMEOUT, e.value
        assert "timed out" in str(e.value)
        assert waited >= limit_us * 1e-6, f"the wait gave up after {waited * 1e6:.0f} us < {limit_us} us"
        kv.check()  # the flag was cleared by the report
        _attend_matches(kv, ok, rng, lens)  # the context and the handle still work
    with pytest.raises(KvError) as e:
        kv.selftest_wait(0)
    assert e.value.code == N.LT_E_ARG
    kv.close()


CHILD = r"""
import sys
import numpy as np
import pytest
import torch
sys.path.insert(0, ".")
sys.path.insert(0, "tests")
from langtrain_studio_b200 import _native as N
from langtrain_studio_b200.kv import KvError
from oracle import oracle
import test_gpu_failure as T

L = N.lib()
assert "liblt_kv_checked.so" in open("/proc/self/maps").read(), "checked library not loaded"
assert L.lt_kv_build_features() & N.LT_FEATURE_BOUNDS_CHECK, "library built without bounds checks"

# 1) no false reports: parity suites on the checked build (every call checks the flag)
rc = pytest.main(["-q", "-x", "-m", "gpu", "-p", "no:cacheprovider", "tests/test_gpu_parity.py",
                  "-k", "random_ops or cascade or attention_matches_oracle or compaction or cow"])
if rc != 0:
    sys.exit(10 + int(rc))

# 2) a table entry past the pool is reported, not read
from cuda.bindings import runtime as rt
oracle.build()
lens = [40, 21]
# Two layers: an id just past layer 0's blocks is outside the pool the kernel
# is told about but still inside the allocation (it names layer 1's block 0),
# so even a regressed check could not read past the allocation.
kv, ok, rng = T._filled(oracle, lens, n_layers=2)
T._attend_matches(kv, ok, rng, lens)
import ctypes as C
mb = C.c_uint32(0)
tables = L.lt_kv_device_tables(kv._h, C.byref(mb))
good = int(kv.seq_blocks(0)[0])
n_blocks = int(L.lt_kv_n_blocks(kv._h))
torch.cuda.synchronize()
def put(val):
    a = np.array([val], np.int32)
    err, = rt.cudaMemcpy(tables, a.ctypes.data, 4, rt.cudaMemcpyKind.cudaMemcpyHostToDevice)
    assert err == rt.cudaError_t.cudaSuccess, err
put(n_blocks)  # seq 0, entry 0 (not the last block: the kernel reads it from the table)
q = torch.from_numpy(rng.standard_normal((2, 32 * 128)).astype(np.float32)).cuda()
kv.attend(0, q, np.arange(2), np.array(lens) - 1, out_dtype=torch.float32)
try:
    kv.check()
    raise SystemExit("no LT_E_BOUNDS for a table entry past the pool")
except KvError as e:
    assert e.code == N.LT_E_BOUNDS, e
put(good)
T._attend_matches(kv, ok, rng, lens)
kv.close()
print("CHECKED_BUILD_OK")
"""


def test_bounds_checked_build_passes_parity_and_reports_bad_table_entries():
    pytest.importorskip("cuda.bindings.runtime")
    from langtrain_studio_b200 import build

    build.build(variant="checked")  # nvcc; a no-op when liblt_kv_checked.so is current
    env = dict(os.environ, LT_KV_VARIANT="checked", PYTHONPATH=str(ROOT))
    r = subprocess.run([sys.executable, "-c", CHILD], cwd=ROOT, env=env, capture_output=True, text=True,
                       timeout=900)
    tail = (r.stdout + r.stderr)[-4000:]
    assert r.returncode == 0 and "CHECKED_BUILD_OK" in r.stdout, tail
