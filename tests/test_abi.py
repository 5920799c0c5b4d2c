"""CPU tests of the C ABI: the library loads, exports every function that
include/lt_kv.h declares, and its host bookkeeping (a device = -1 handle)
is bit-identical to the oracle's restatement of engine/crates/native/src/kv.rs
under the reference's known-answer tests and long random operation mixes.
"""
import re
import subprocess
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parent.parent


def declared_functions():
    names = set()
    for h in (ROOT / "include").glob("*.h"):
        text = re.sub(r"/\*.*?\*/", "", h.read_text(), flags=re.S)
        names |= set(re.findall(r"\b(lt_[a-z0-9_]+)\s*\(", text))
    return sorted(names)


def test_header_declares_and_library_exports_everything(native):
    from langtrain_studio_b200 import _native

    decl = declared_functions()
    assert decl, "no declarations found"
    assert set(decl) == set(_native.EXPORTS), set(decl) ^ set(_native.EXPORTS)
    out = subprocess.run(["nm", "-D", "--defined-only", _native.library_path()], capture_output=True, text=True,
                         check=True).stdout
    exported = set(re.findall(r"\sT\s+(lt_\w+)", out))
    missing = set(decl) - exported
    assert not missing, missing
    for name in decl:
        assert hasattr(native, name)


def test_header_compiles_as_c():
    src = ('#include "lt_kv.h"\n#include "lt_llama.h"\n#include "lt_sched.h"\n#include "lt_prefix.h"\n'
           'int main(void){ lt_kv_config c = {0}; lt_llama_config m = {0}; (void)c; (void)m; return LT_OK; }\n')
    subprocess.run(["gcc", "-std=c99", "-Wall", "-Werror", "-I", str(ROOT / "include"), "-x", "c", "-", "-o",
                    "/dev/null"], input=src, text=True, check=True)


def host_kv(n_layers, kv_dim_heads, head_dim, n_tokens, max_seqs=16):
    from langtrain_studio_b200.kv import KvCache

    return KvCache(n_layers, kv_dim_heads, head_dim, n_tokens, max_seqs=max_seqs, device=-1)


def test_create_rejects_bad_configs(native):
    from langtrain_studio_b200.kv import KvCache, KvError

    with pytest.raises(KvError):
        KvCache(1, 2, 96, 64, device=-1)  # head_dim must be 64 or 128
    with pytest.raises(KvError):
        KvCache(1, 2, 64, 64, n_heads=3, device=-1)  # n_heads % n_kv_heads
    with pytest.raises(KvError):
        KvCache(1, 1, 64, 64, n_heads=16, device=-1)  # group > 8


def test_known_answer_share_then_diverge_bookkeeping():
    """kv.rs:202-217 (bookkeeping half; the data half runs on the GPU)."""
    kv = host_kv(1, 1, 64, 256)
    for p in range(20):
        kv.append(0, p)
    kv.share(0, 1, 20)
    free_before = kv.free_blocks()
    b, s = kv.append(1, 20)
    assert kv.free_blocks() == free_before - 1
    assert s == 4 and b not in kv.seq_blocks(0)
    assert list(kv.seq_blocks(1))[:1] == list(kv.seq_blocks(0))[:1]
    assert kv.len(0) == 20 and kv.len(1) == 21


def test_known_answer_truncate_frees_blocks():
    """kv.rs:219-229."""
    from langtrain_studio_b200.kv import KvNonContiguous

    kv = host_kv(1, 1, 64, 64)
    for p in range(40):
        kv.append(3, p)
    assert kv.free_blocks() == 1
    kv.truncate(3, 10)
    assert kv.free_blocks() == 3
    kv.truncate(3, 0)
    assert kv.free_blocks() == 4
    with pytest.raises(KvNonContiguous):
        kv.append(3, 5)


def test_errors_leave_state_like_reference(oracle_mod):
    from langtrain_studio_b200.kv import KvCacheFull, KvError

    kv = host_kv(1, 1, 64, 48, max_seqs=4)
    ok = oracle_mod.OracleKv(1, 64, 48, max_seqs=4)
    # batch: seq0 pos0, seq1 pos0, seq2 pos0, seq3 pos0 -> the 4th fails: full
    with pytest.raises(KvCacheFull) as e:
        kv.append_batch([0, 1, 2, 3], [0, 0, 0, 0])
    assert e.value.n_done == 3
    rc, done, _, _ = ok.append_batch([0, 1, 2, 3], [0, 0, 0, 0])
    assert rc == oracle_mod.FULL and done == 3
    assert kv.len(3) == 0 and ok.len(3) == 0
    with pytest.raises(KvError):
        kv.append(99, 0)  # seq id beyond max_seqs


def compare_state(kv, ok, max_seqs):
    assert kv.free_blocks() == ok.free_blocks()
    assert np.array_equal(kv.free_list(), ok.free_list())
    assert np.array_equal(kv.refs(), ok.refs())
    for s in range(max_seqs):
        assert kv.len(s) == ok.len(s), s
        assert np.array_equal(kv.seq_blocks(s), ok.seq_blocks(s)), s


def random_ops(seed, kv, ok, max_seqs, n_ops, compact_every=0):
    """Random mix of batched append / truncate / share / compact, the calls the
    scheduler makes through Backend::{decode, kv_remove, kv_copy}."""
    from langtrain_studio_b200.kv import KvError

    rng = np.random.default_rng(seed)
    for step in range(n_ops):
        r = rng.random()
        if r < 0.55:
            n = int(rng.integers(1, 12))
            seqs = rng.integers(0, max_seqs, n)
            pos = []
            lens = {}
            for s in seqs:
                cur = lens.get(int(s), kv.len(int(s)))
                # mostly contiguous, sometimes a deliberate gap
                p = cur if rng.random() < 0.95 else cur + int(rng.integers(1, 3))
                pos.append(p)
                lens[int(s)] = p + 1
            rc, done, blocks_o, slots_o = ok.append_batch(seqs, pos)
            try:
                blocks, slots = kv.append_batch(seqs, pos)
                assert rc == 0
                n_done = len(seqs)
            except KvError as e:
                assert e.code == rc, (e.code, rc, str(e))
                n_done = e.n_done
                blocks = slots = None
            assert n_done == done
            if blocks is not None:
                assert np.array_equal(blocks, blocks_o) and np.array_equal(slots, slots_o)
        elif r < 0.75:
            s = int(rng.integers(0, max_seqs))
            frm = int(rng.integers(0, max(kv.len(s), 1) + 3))
            kv.truncate(s, frm)
            ok.truncate(s, frm)
        elif r < 0.95:
            src, dst = (int(x) for x in rng.integers(0, max_seqs, 2))
            length = int(rng.integers(0, max(kv.len(src), 1) + 5))
            kv.share(src, dst, length)
            ok.share(src, dst, length)
        elif compact_every:
            assert kv.compact() == len(ok.compact())
        compare_state(kv, ok, max_seqs)


@pytest.mark.parametrize("seed", range(6))
def test_random_ops_match_oracle(oracle_mod, seed):
    max_seqs = 12
    kv = host_kv(2, 1, 64, 16 * 40, max_seqs=max_seqs)
    ok = oracle_mod.OracleKv(2, 64, 16 * 40, max_seqs=max_seqs)
    random_ops(seed, kv, ok, max_seqs, 400, compact_every=seed % 2)


def test_compaction_bookkeeping_matches_oracle(oracle_mod):
    max_seqs = 10
    kv = host_kv(1, 1, 64, 16 * 64, max_seqs=max_seqs)
    ok = oracle_mod.OracleKv(1, 64, 16 * 64, max_seqs=max_seqs)
    random_ops(11, kv, ok, max_seqs, 300)
    for s in range(0, max_seqs, 3):
        kv.truncate(s, 0)
        ok.truncate(s, 0)
    assert kv.compact() == len(ok.compact())
    compare_state(kv, ok, max_seqs)
    live = np.nonzero(kv.refs())[0]
    assert list(live) == list(range(live.size))


@pytest.mark.parametrize("share_rate", [0.0, 0.03])
def test_compaction_paths_match_oracle(oracle_mod, share_rate):
    """Compaction after every few operations, over a larger pool: with no
    sharing every moved block is rewritten through its owner entry; with
    occasional kv_copy some moves fall back to scanning every table.  The
    moves, tables, refcounts and free list must equal the oracle's full scan."""
    from langtrain_studio_b200.kv import KvError

    max_seqs, pool = 24, 16 * 300
    kv = host_kv(1, 1, 64, pool, max_seqs=max_seqs)
    ok = oracle_mod.OracleKv(1, 64, pool, max_seqs=max_seqs)
    rng = np.random.default_rng(int(share_rate * 1000) + 5)
    for step in range(1500):
        r = rng.random()
        if r < 0.6:
            s = int(rng.integers(0, max_seqs))
            n = int(rng.integers(1, 40))
            seqs, pos = np.full(n, s), np.arange(kv.len(s), kv.len(s) + n)
            rc, done, bo, so = ok.append_batch(seqs, pos)
            try:
                b, sl = kv.append_batch(seqs, pos)
                assert rc == 0 and np.array_equal(b, bo) and np.array_equal(sl, so)
            except KvError as e:
                assert e.code == rc and e.n_done == done
        elif r < 0.8:
            s = int(rng.integers(0, max_seqs))
            frm = int(rng.integers(0, kv.len(s) + 1))
            kv.truncate(s, frm)
            ok.truncate(s, frm)
        elif r < 0.8 + share_rate:
            src, dst = (int(x) for x in rng.integers(0, max_seqs, 2))
            n = int(rng.integers(0, kv.len(src) + 1))
            kv.share(src, dst, n)
            ok.share(src, dst, n)
        else:
            assert kv.compact() == len(ok.compact()), step
        compare_state(kv, ok, max_seqs)


def test_dtype_arguments_outside_the_enum_are_refused(native):
    """A dtype that is neither LT_F32 nor LT_F16 is refused (LT_E_ARG) before
    any other check or device work, on every entry point that takes one;
    nothing is dereferenced (the pointers here are placeholders)."""
    import ctypes as C

    from langtrain_studio_b200 import _native as N

    lib = native
    kv = host_kv(1, 1, 64, 64)
    h = kv._h
    p = C.c_void_p(256)  # 16-byte aligned placeholder, never dereferenced
    one = np.zeros(1, np.uint32)
    cell = np.zeros(1, np.int32)
    addr = lambda a: C.c_void_p(a.ctypes.data)  # noqa: E731
    bad, f32, f16 = 7, N.LT_F32, N.LT_F16
    calls = {
        "lt_kv_write": lambda d: lib.lt_kv_write(h, 0, addr(cell), addr(cell), 1, p, p, d, None),
        "lt_kv_attend q": lambda d: lib.lt_kv_attend(h, 0, p, d, addr(one), addr(one), 1, p, f32, 0.125, None),
        "lt_kv_attend out": lambda d: lib.lt_kv_attend(h, 0, p, f16, addr(one), addr(one), 1, p, d, 0.125, None),
        "lt_kv_write_attend": lambda d: lib.lt_kv_write_attend(h, 0, addr(cell), addr(cell), p, p, d, p, f16,
                                                               addr(one), addr(one), 1, p, f32, 0.125, None),
        "lt_kv_attend_gather": lambda d: lib.lt_kv_attend_gather(h, 0, p, f16, addr(one), addr(one), 1, p, d, 0.125,
                                                                 None),
    }
    for name, call in calls.items():
        assert call(bad) == N.LT_E_ARG, name
        assert "neither LT_F32 nor LT_F16" in lib.lt_kv_last_error(h).decode(), name
        assert call(f32 if "out" not in name else f16) == N.LT_E_ARG  # valid dtype: refused for having no device
        assert "without a device" in lib.lt_kv_last_error(h).decode(), name
    assert lib.lt_kv_gather_heads(h, p, p, p, 1, bad, p, 2, None) == N.LT_E_ARG
    assert lib.lt_paged_attend_noalloc(p, N.LT_KV_F16, 4, 1, 64, 1, p, 1, 4, addr(one), addr(one), 1, p, bad, p,
                                       f32, C.c_float(0.125), None) == N.LT_E_ARG
    assert lib.lt_paged_attend_noalloc(p, N.LT_KV_F16, 4, 1, 64, 1, p, 1, 4, addr(one), addr(one), 1, p, f32, p,
                                       bad, C.c_float(0.125), None) == N.LT_E_ARG
    kv.close()


def test_noalloc_refuses_what_would_index_outside_the_callers_buffers(native):
    """lt_paged_attend_noalloc takes its pool and tables from the caller, so
    every argument the kernel would index with is checked on the host before
    any device work; these calls return before touching a GPU (the pointers
    are placeholders, never dereferenced)."""
    import ctypes as C

    from langtrain_studio_b200 import _native as N

    lib = native
    p = C.c_void_p(256)  # 16-byte aligned placeholder
    f32 = N.LT_F32

    def call(pos=0, seq=0, pool=p, tables=p, kv_format=N.LT_KV_F16, n_blocks=4, rows=2, max_blocks=4,
             n=1, q=p, out=p):
        s = np.full(max(n, 1), seq, np.uint32)
        ps = np.full(max(n, 1), pos, np.uint32)
        return lib.lt_paged_attend_noalloc(pool, kv_format, n_blocks, 1, 64, 1, tables, rows, max_blocks,
                                           C.c_void_p(s.ctypes.data), C.c_void_p(ps.ctypes.data), n, q, f32, out,
                                           f32, C.c_float(0.125), None)

    # positions: past the row, and the uint32 values whose (pos + 16) / 16 wraps to 0
    assert call(pos=4 * 16) == N.LT_E_ARG
    for pos in (0xFFFFFFF0, 0xFFFFFFFF, 0x7FFFFFFF, 0x80000000):
        assert call(pos=pos, max_blocks=0x7FFFFFFF) == N.LT_E_ARG, hex(pos)
    # sequence ids past the caller's table rows
    assert call(seq=2) == N.LT_E_ARG
    assert call(seq=0xFFFFFFFF) == N.LT_E_ARG
    # sizes the kernel carries as int32, and empty pools or tables
    assert call(max_blocks=0x80000000) == N.LT_E_ARG
    assert call(n_blocks=0x80000000) == N.LT_E_ARG
    assert call(n_blocks=0) == N.LT_E_ARG
    assert call(rows=0) == N.LT_E_ARG
    assert call(max_blocks=0) == N.LT_E_ARG
    # bulk copies start at 16-byte boundaries; table entries are int32
    assert call(pool=C.c_void_p(256 + 8)) == N.LT_E_ARG
    assert call(tables=C.c_void_p(256 + 2)) == N.LT_E_ARG
    assert call(q=C.c_void_p(256 + 4)) == N.LT_E_ARG
    assert call(out=C.c_void_p(256 + 4)) == N.LT_E_ARG
    # the pool's format: f16 only
    assert call(kv_format=N.LT_KV_Q8_0) == N.LT_E_UNSUPPORTED
    assert call(kv_format=7) == N.LT_E_ARG
    # too many tokens for the fixed scratch
    assert call(n=N.LT_NOALLOC_MAX_TOKENS + 1) == N.LT_E_SCRATCH
    assert call(n=0) == N.LT_OK  # nothing to do, nothing touched


def test_accessors_of_a_null_handle_return_zero(native):
    lib = native
    assert lib.lt_kv_capacity(None) == 0
    assert lib.lt_kv_bytes(None) == 0
    assert lib.lt_kv_len(None, 0) == 0
    assert lib.lt_kv_free_blocks(None) == 0
    assert lib.lt_kv_n_blocks(None) == 0
    assert lib.lt_kv_refs(None, None, 0) == 0
    assert lib.lt_kv_free_list(None, None, 0) == 0
    assert lib.lt_kv_seq_blocks(None, 0, None, 0) == 0
