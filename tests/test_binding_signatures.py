"""The ctypes binding (langtrain_studio_b200/_native.py) against the C headers.

A ctypes declaration that disagrees with the C prototype does not fail to
load: an argument of the wrong width is silently truncated or reads a
neighbour's register, and a struct field at the wrong offset reads another
field.  So the prototypes are taken from the compiler itself (gcc -aux-info
over include/*.h) and every binding is compared with them argument by
argument: same count, same integer width and signedness, float for float,
pointer for pointer (and the pointee where the binding names one).  Every
struct the binding mirrors is compared field by field with offsetof/sizeof
from a compiled C program.  CPU only; the library is not loaded.
"""
from __future__ import annotations

import ctypes as C
import re
import sys
import types
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT))
sys.path.insert(0, str(ROOT / "tests"))

import _headers as H  # noqa: E402

from langtrain_studio_b200 import _native as N  # noqa: E402

STRUCTS = (N.lt_kv_config, N.lt_llama_config, N.lt_sched_config, N.lt_placement, N.lt_sched_stats)
OPAQUE = {"lt_kv", "lt_llama", "lt_sched", "lt_slot_cache"}
ENUMS = {"lt_status", "lt_dtype", "lt_kv_format", "lt_tensor"}
SCALARS = {
    "uint32_t": C.c_uint32, "int32_t": C.c_int32, "uint64_t": C.c_uint64, "int64_t": C.c_int64,
    "int": C.c_int, "unsigned int": C.c_uint, "float": C.c_float, "double": C.c_double, "size_t": C.c_size_t,
    **{e: C.c_int for e in ENUMS},
}
POINTERS = (C.c_void_p, C.c_char_p)

pytestmark = pytest.mark.skipif(not H.have_gcc(), reason="gcc is not installed")


@pytest.fixture(scope="module")
def prototypes():
    return H.prototypes()


def _declared():
    """name -> (restype, argtypes) exactly as _native._declare sets them."""
    funcs = {}

    class Recorder:
        def __getattr__(self, name):
            return funcs.setdefault(name, types.SimpleNamespace())

    N._declare(Recorder())
    return {k: (v.restype, list(v.argtypes)) for k, v in funcs.items()}


def _norm(t: str) -> str:
    t = re.sub(r"\bconst\b", "", t)
    t = re.sub(r"\bstruct\b", "", t)
    return re.sub(r"\s+", " ", t).replace(" *", "*").strip()


def _is_pointer_type(ct) -> bool:
    return ct in POINTERS or (isinstance(ct, type) and issubclass(ct, C._Pointer))


def _check(ctype: str, bound, where: str):
    t = _norm(ctype)
    if t == "void":
        assert bound is None, f"{where}: C returns void, binding says {bound}"
        return
    if t.endswith("*"):
        assert _is_pointer_type(bound), f"{where}: C type {ctype!r} is a pointer, binding says {bound}"
        if t == "char*":
            return
        if bound in POINTERS:
            return
        pointee = t[:-1]
        want = None
        if pointee.endswith("*") or pointee in OPAQUE or pointee == "void":
            want = C.c_void_p
        elif pointee in SCALARS:
            want = SCALARS[pointee]
        else:
            want = next((s for s in STRUCTS if s.__name__ == pointee), None)
        assert want is not None, f"{where}: no ctypes mapping for pointee {pointee!r}"
        assert bound._type_ is want, f"{where}: C pointee {pointee!r}, binding points at {bound._type_}"
        return
    assert t in SCALARS, f"{where}: no ctypes mapping for C type {ctype!r}"
    want = SCALARS[t]
    assert bound is not None and not _is_pointer_type(bound), f"{where}: C type {ctype!r}, binding says {bound}"
    assert C.sizeof(bound) == C.sizeof(want), f"{where}: C type {ctype!r} is {C.sizeof(want)} bytes, " \
                                              f"binding {bound} is {C.sizeof(bound)}"
    floating = want in (C.c_float, C.c_double)
    assert (bound in (C.c_float, C.c_double)) == floating, f"{where}: C type {ctype!r}, binding {bound}"
    if not floating and t not in ENUMS:
        signed = want(-1).value < 0
        assert (bound(-1).value < 0) == signed, f"{where}: signedness of {ctype!r} differs from {bound}"


def test_every_header_function_is_bound_and_exported(prototypes):
    declared = _declared()
    assert set(prototypes) == set(declared), (sorted(set(prototypes) - set(declared)),
                                              sorted(set(declared) - set(prototypes)))
    assert set(prototypes) == set(N.EXPORTS), (sorted(set(prototypes) - set(N.EXPORTS)),
                                               sorted(set(N.EXPORTS) - set(prototypes)))


def test_binding_signatures_match_the_prototypes(prototypes):
    declared = _declared()
    for name, (ret, args) in sorted(prototypes.items()):
        res, argtypes = declared[name]
        _check(ret, res, f"{name} return")
        assert len(args) == len(argtypes), f"{name}: C has {len(args)} arguments, binding {len(argtypes)}"
        for i, (a, b) in enumerate(zip(args, argtypes)):
            _check(a, b, f"{name} argument {i} ({a})")


def test_struct_layouts_match_the_compiler():
    got = H.layouts({st.__name__: [f for f, _ in st._fields_] for st in STRUCTS})
    for st in STRUCTS:
        lay = got[st.__name__]
        assert lay["sizeof"] == C.sizeof(st), f"{st.__name__}: sizeof differs"
        for f, ft in st._fields_:
            off, size = lay[f]
            assert getattr(st, f).offset == off, f"{st.__name__}.{f}: offset {getattr(st, f).offset} vs C {off}"
            assert C.sizeof(ft) == size, f"{st.__name__}.{f}: {C.sizeof(ft)} bytes vs C {size}"


def test_binding_constants_match_the_headers():
    names = ["LT_OK", "LT_E_FULL", "LT_E_NONCONTIG", "LT_E_ARG", "LT_E_CUDA", "LT_E_NCCL", "LT_E_TIMEOUT",
             "LT_E_UNSUPPORTED", "LT_E_SCRATCH", "LT_E_BOUNDS", "LT_F32", "LT_F16", "LT_KV_F16", "LT_KV_Q8_0",
             "LT_FEATURE_BOUNDS_CHECK", "LT_IPC_HANDLE_BYTES", "LT_NOALLOC_SCRATCH_BYTES", "LT_NOALLOC_MAX_TOKENS"]
    got = H.constants(names)
    for n in names:
        assert getattr(N, n) == got[n], f"{n}: binding {getattr(N, n)} vs header {got[n]}"
