"""GPU test of lt_paged_attend_noalloc, the allocation-free attention entry point.

That entry point serves callers that cannot call cudaMalloc: hosts whose
device memory is wholly owned by their own allocator or fixed budget, and
hosts that cannot afford cudaMalloc's possible device-wide synchronisation on
their step path.  It takes the pool and block tables the caller already has
and keeps the kernel's scratch in a fixed static device array.  This file is
named so that pytest collects it last.

Checks, through the C ABI, against the oracle (the CPU restatement of the
reference's attention closure, model.rs:431-476) on the same cache contents:
two calls in a row each match within the suite's attention tolerance; so do
calls of alternating sizes (600 tokens run as two launches, then 8, then 600
again); the error word stays clear on good calls; a table entry outside the
pool the caller declares is reported as LT_E_BOUNDS by
lt_paged_attend_noalloc_check and cleared by it; oversized requests are
refused with LT_E_SCRATCH before any work.
"""
import ctypes as C

import numpy as np
import pytest

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu

ATOL, RTOL = 2e-3, 1e-3  # the attention tolerance of tests/test_gpu_parity.py


@pytest.fixture(scope="module", autouse=True)
def _need_cuda():
    if not torch.cuda.is_available():
        pytest.fail("CUDA device required for -m gpu tests")


def _stream():
    return C.c_void_p(torch.cuda.current_stream().cuda_stream)


def _noalloc(lib, kv, layer, q, out, seqs, pos, scale, n_blocks=None, kv_format=0):
    from langtrain_studio_b200 import _native as N

    pool = lib.lt_kv_device_pool(kv._h)
    mb = C.c_uint32()
    tables = lib.lt_kv_device_tables(kv._h, C.byref(mb))
    layer_halves = kv.n_blocks * kv.n_kv_heads * 2 * 16 * kv.head_dim
    pool_layer = C.c_void_p(pool + layer * layer_halves * 2)
    seqs = np.ascontiguousarray(seqs, np.uint32)
    pos = np.ascontiguousarray(pos, np.uint32)
    dt = {torch.float32: N.LT_F32, torch.float16: N.LT_F16}
    return lib.lt_paged_attend_noalloc(
        pool_layer, kv_format, kv.n_blocks if n_blocks is None else n_blocks, kv.n_kv_heads, kv.head_dim,
        kv.n_heads, C.c_void_p(tables), kv.max_seqs, mb.value,
        seqs.ctypes.data_as(C.c_void_p), pos.ctypes.data_as(C.c_void_p), seqs.size,
        C.c_void_p(q.data_ptr()), dt[q.dtype], C.c_void_p(out.data_ptr()), dt[out.dtype], C.c_float(scale),
        _stream())


def _twin(oracle_mod, n_layers, hq, hkv, d, lens, seed):
    """A GPU cache and the oracle with the same sequences and rows."""
    from langtrain_studio_b200.kv import KvCache

    nblk = sum((L + 16) // 16 for L in lens) + 8
    kv = KvCache(n_layers, hkv, d, 16 * nblk, n_heads=hq, max_seqs=len(lens), max_batch=4096, device=0)
    ok = oracle_mod.OracleKv(n_layers, hkv * d, 16 * nblk, max_seqs=len(lens))
    rng = np.random.default_rng(seed)
    for s, L in enumerate(lens):
        seqs, pos = np.full(L, s), np.arange(L)
        b, sl = kv.append_batch(seqs, pos)
        rc, _, bo, so = ok.append_batch(seqs, pos)
        assert rc == 0 and np.array_equal(b, bo) and np.array_equal(sl, so)
        for layer in range(n_layers):
            k = rng.standard_normal((L, hkv * d)).astype(np.float32)
            v = rng.standard_normal((L, hkv * d)).astype(np.float32)
            kv.write(layer, b, sl, torch.from_numpy(k).cuda(), torch.from_numpy(v).cuda())
            ok.write_batch(layer, b, sl, k, v)
    kv.flush()
    torch.cuda.synchronize()
    return kv, ok, rng


@pytest.mark.parametrize("q_dtype", [torch.float32, torch.float16])
def test_noalloc_matches_oracle_two_calls(oracle_mod, q_dtype):
    from langtrain_studio_b200 import _native as N

    lib = N.lib()
    hq, hkv, d = 32, 8, 128
    lens = [1, 17, 300, 700, 1600, 2100, 64, 999]
    kv, ok, rng = _twin(oracle_mod, 2, hq, hkv, d, lens, seed=5)
    seqs = np.arange(len(lens))
    pos = np.array(lens) - 1
    scale = float(np.float32(1.0) / np.float32(np.sqrt(d)))
    for layer in range(2):
        q = torch.from_numpy(rng.standard_normal((len(lens), hq * d)).astype(np.float32)).cuda().to(q_dtype)
        ref = ok.attend(layer, q.float().cpu().numpy(), seqs, pos, hq, hkv, d, scale=scale)
        for _ in range(2):  # two calls in a row share (and reuse) the static scratch
            out = torch.full((len(lens), hq * d), float("nan"), device="cuda")
            rc = _noalloc(lib, kv, layer, q, out, seqs, pos, scale)
            assert rc == N.LT_OK, rc
            assert lib.lt_paged_attend_noalloc_check(_stream()) == N.LT_OK
            np.testing.assert_allclose(out.cpu().numpy(), ref, rtol=RTOL, atol=ATOL)
    kv.close()


def test_noalloc_alternating_call_sizes(oracle_mod):
    """600 tokens (more than one launch carries, so the call runs as two
    launches), then 8, then 600 again: each call must match the oracle
    although the previous call left its partials and flags in the array."""
    from langtrain_studio_b200 import _native as N

    lib = N.lib()
    hq, hkv, d = 16, 4, 128
    lens = [900, 75, 1300, 260, 640, 33, 1024, 512]
    kv, ok, rng = _twin(oracle_mod, 1, hq, hkv, d, lens, seed=11)
    big_seqs = np.repeat(np.arange(len(lens)), 75)  # 600 tokens
    big_pos = np.array([rng.integers(0, lens[s]) for s in big_seqs])
    small_seqs = np.arange(len(lens))
    small_pos = np.array(lens) - 1
    scale = float(np.float32(1.0) / np.float32(np.sqrt(d)))
    for seqs, pos in ((big_seqs, big_pos), (small_seqs, small_pos), (big_seqs, big_pos)):
        q = rng.standard_normal((seqs.size, hq * d)).astype(np.float32)
        ref = ok.attend(0, q, seqs, pos, hq, hkv, d, scale=scale)
        out = torch.full((seqs.size, hq * d), float("nan"), device="cuda")
        rc = _noalloc(lib, kv, 0, torch.from_numpy(q).cuda(), out, seqs, pos, scale)
        assert rc == N.LT_OK, rc
        assert lib.lt_paged_attend_noalloc_check(_stream()) == N.LT_OK
        np.testing.assert_allclose(out.cpu().numpy(), ref, rtol=RTOL, atol=ATOL)
    kv.close()


def test_noalloc_reports_block_ids_outside_the_declared_pool(oracle_mod):
    """The caller declares a pool one block smaller than the handle's, so the
    highest block in use lies outside it (but inside the allocation: nothing
    is read past it even if the check failed).  The call reads block 0 in its
    place and the check reports LT_E_BOUNDS once, then the word is clear and
    a call over the true pool size matches the oracle again."""
    from langtrain_studio_b200 import _native as N

    lib = N.lib()
    hq, hkv, d = 8, 2, 64
    lens = [40, 100]
    kv, ok, rng = _twin(oracle_mod, 1, hq, hkv, d, lens, seed=3)
    used = np.concatenate([kv.seq_blocks(s) for s in range(len(lens))])
    declared = int(used.max())  # the highest id in use is now outside [0, declared)
    seqs, pos = np.arange(len(lens)), np.array(lens) - 1
    q = rng.standard_normal((len(lens), hq * d)).astype(np.float32)
    out = torch.zeros((len(lens), hq * d), device="cuda")
    assert _noalloc(lib, kv, 0, torch.from_numpy(q).cuda(), out, seqs, pos, 0.125, n_blocks=declared) == N.LT_OK
    assert lib.lt_paged_attend_noalloc_check(_stream()) == N.LT_E_BOUNDS
    assert lib.lt_paged_attend_noalloc_check(_stream()) == N.LT_OK  # read and cleared
    ref = ok.attend(0, q, seqs, pos, hq, hkv, d, scale=0.125)
    assert _noalloc(lib, kv, 0, torch.from_numpy(q).cuda(), out, seqs, pos, 0.125) == N.LT_OK
    assert lib.lt_paged_attend_noalloc_check(_stream()) == N.LT_OK
    np.testing.assert_allclose(out.cpu().numpy(), ref, rtol=RTOL, atol=ATOL)
    kv.close()


def test_noalloc_rejects_oversized_requests_and_q8_pools():
    from langtrain_studio_b200 import _native as N
    from langtrain_studio_b200.kv import KvCache

    lib = N.lib()
    kv = KvCache(1, 1, 64, 16 * 4, n_heads=2, max_seqs=1, max_batch=8, device=0)
    kv.append_batch([0], [0])
    n = N.LT_NOALLOC_MAX_TOKENS + 1
    q = torch.zeros((n, 128), device="cuda")
    out = torch.zeros((n, 128), device="cuda")
    assert _noalloc(lib, kv, 0, q, out, np.zeros(n), np.zeros(n), 0.125) == N.LT_E_SCRATCH
    assert _noalloc(lib, kv, 0, q[:1], out[:1], [0], [0], 0.125, kv_format=N.LT_KV_Q8_0) == N.LT_E_UNSUPPORTED
    assert lib.lt_paged_attend_noalloc_check(_stream()) == N.LT_OK
    kv.close()
