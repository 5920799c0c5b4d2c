"""GPU test of lt_paged_attend_noalloc, the allocation-free attention entry point.

That entry point serves callers that cannot call cudaMalloc: hosts whose
device memory is wholly owned by their own allocator or fixed budget, and
hosts that cannot afford cudaMalloc's possible device-wide synchronisation on
their step path.  It takes the pool and block tables the caller already has
and keeps the kernel's scratch in a fixed static device array.  This file is
named so that pytest collects it last.

Checks, through the C ABI: two calls in a row each match lt_kv_attend on the
same cache within the suite's attention tolerance; so do calls of alternating
sizes, whose work plans sit at different places in the shared array; and
oversized requests are refused with LT_E_SCRATCH before any work.
"""
import ctypes as C

import numpy as np
import pytest

torch = pytest.importorskip("torch")

pytestmark = pytest.mark.gpu

ATOL, RTOL = 2e-3, 1e-3  # the attention tolerance of tests/test_gpu_parity.py


def _noalloc(lib, kv, layer, q, out, seqs, pos, scale):
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
        pool_layer, kv.n_kv_heads, kv.head_dim, kv.n_heads, C.c_void_p(tables), mb.value,
        seqs.ctypes.data_as(C.c_void_p), pos.ctypes.data_as(C.c_void_p), seqs.size,
        C.c_void_p(q.data_ptr()), dt[q.dtype], C.c_void_p(out.data_ptr()), dt[out.dtype], C.c_float(scale),
        C.c_void_p(torch.cuda.current_stream().cuda_stream))


@pytest.mark.parametrize("q_dtype", [torch.float32, torch.float16])
def test_noalloc_matches_attend_two_calls(q_dtype):
    if not torch.cuda.is_available():
        pytest.fail("CUDA device required for -m gpu tests")
    from langtrain_studio_b200 import _native as N
    from langtrain_studio_b200.kv import KvCache

    lib = N.lib()
    hq, hkv, d = 32, 8, 128
    lens = [1, 17, 300, 700, 1600, 2100, 64, 999]
    nblk = sum((L + 16) // 16 for L in lens) + 8
    kv = KvCache(2, hkv, d, 16 * nblk, n_heads=hq, max_seqs=len(lens), max_batch=4096, device=0)
    g = torch.Generator(device="cuda")
    g.manual_seed(5)
    for s, L in enumerate(lens):
        b, sl = kv.append_batch(np.full(L, s), np.arange(L))
        for layer in range(2):
            k = torch.randn((L, hkv * d), generator=g, device="cuda")
            v = torch.randn((L, hkv * d), generator=g, device="cuda")
            kv.write(layer, b, sl, k, v)
    kv.flush()
    seqs = np.arange(len(lens))
    pos = np.array(lens) - 1
    scale = float(np.float32(1.0) / np.float32(np.sqrt(d)))
    for layer in range(2):
        q = torch.randn((len(lens), hq * d), generator=g, device="cuda").to(q_dtype)
        ref = kv.attend(layer, q, seqs, pos, out_dtype=torch.float32, scale=scale)
        for _ in range(2):  # two calls in a row share (and reuse) the static scratch
            out = torch.full((len(lens), hq * d), float("nan"), device="cuda")
            rc = _noalloc(lib, kv, layer, q, out, seqs, pos, scale)
            assert rc == N.LT_OK, rc
            torch.cuda.synchronize()
            np.testing.assert_allclose(out.cpu().numpy(), ref.cpu().numpy(), rtol=RTOL, atol=ATOL)
    kv.close()


def test_noalloc_alternating_call_sizes():
    """600 tokens (more than the launch parameters carry, so the work plan goes
    through the array), then 8, then 600 again: each call must match
    lt_kv_attend although the previous call left its plan and partials where
    this call's layout differs."""
    if not torch.cuda.is_available():
        pytest.fail("CUDA device required for -m gpu tests")
    from langtrain_studio_b200 import _native as N
    from langtrain_studio_b200.kv import KvCache

    lib = N.lib()
    hq, hkv, d = 16, 4, 128
    lens = [900, 75, 1300, 260, 640, 33, 1024, 512]
    nblk = sum((L + 16) // 16 for L in lens) + 8
    kv = KvCache(1, hkv, d, 16 * nblk, n_heads=hq, max_seqs=len(lens), max_batch=4096, device=0)
    g = torch.Generator(device="cuda")
    g.manual_seed(11)
    for s, L in enumerate(lens):
        b, sl = kv.append_batch(np.full(L, s), np.arange(L))
        kv.write(0, b, sl, torch.randn((L, hkv * d), generator=g, device="cuda"),
                 torch.randn((L, hkv * d), generator=g, device="cuda"))
    kv.flush()
    rng = np.random.default_rng(11)
    big_seqs = np.repeat(np.arange(len(lens)), 75)  # 600 tokens
    big_pos = np.array([rng.integers(0, lens[s]) for s in big_seqs])
    small_seqs = np.arange(len(lens))
    small_pos = np.array(lens) - 1
    scale = float(np.float32(1.0) / np.float32(np.sqrt(d)))
    for seqs, pos in ((big_seqs, big_pos), (small_seqs, small_pos), (big_seqs, big_pos)):
        q = torch.randn((seqs.size, hq * d), generator=g, device="cuda")
        ref = kv.attend(0, q, seqs, pos, out_dtype=torch.float32, scale=scale)
        out = torch.full((seqs.size, hq * d), float("nan"), device="cuda")
        rc = _noalloc(lib, kv, 0, q, out, seqs, pos, scale)
        assert rc == N.LT_OK, rc
        torch.cuda.synchronize()
        np.testing.assert_allclose(out.cpu().numpy(), ref.cpu().numpy(), rtol=RTOL, atol=ATOL)
    kv.close()


def test_noalloc_rejects_oversized_requests():
    if not torch.cuda.is_available():
        pytest.fail("CUDA device required for -m gpu tests")
    from langtrain_studio_b200 import _native as N
    from langtrain_studio_b200.kv import KvCache

    lib = N.lib()
    kv = KvCache(1, 1, 64, 16 * 4, n_heads=2, max_seqs=1, max_batch=8, device=0)
    kv.append_batch([0], [0])
    n = N.LT_NOALLOC_MAX_TOKENS + 1
    q = torch.zeros((n, 128), device="cuda")
    out = torch.zeros((n, 128), device="cuda")
    rc = _noalloc(lib, kv, 0, q, out, np.zeros(n), np.zeros(n), 0.125)
    assert rc == N.LT_E_SCRATCH
    kv.close()
