"""The Rust binding include/lt_kv_sys.rs against the C headers.

Its `extern "C"` blocks are what the reference's engine would add to bind
liblt_kv.so (its native crate is Rust).  No Rust toolchain is installed here,
so the declarations cannot be compiled; instead every one is compared with
the prototype gcc reports for include/*.h: argument count, integer width and
signedness, f32/f64, pointer depth, const-ness and pointee.  `#[repr(C)]`
structs are laid out by the repr(C) rule and compared with offsetof/sizeof of
the C struct, field names included, and `pub const` values with the header's.
Every Rust excerpt that INTEGRATION.md quotes must appear in the file verbatim.
"""
from __future__ import annotations

import re
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT / "tests"))

import _headers as H  # noqa: E402

pytestmark = pytest.mark.skipif(not H.have_gcc(), reason="gcc is not installed")

# Rust scalar -> (size, signed, float)
RUST = {"u8": (1, False, False), "i8": (1, True, False), "u32": (4, False, False), "i32": (4, True, False),
        "u64": (8, False, False), "i64": (8, True, False), "usize": (8, False, False), "isize": (8, True, False),
        "f32": (4, True, True), "f64": (8, True, True)}
ENUMS = {"lt_status", "lt_dtype", "lt_kv_format", "lt_tensor"}
C_SCALAR = {"uint8_t": (1, False, False), "uint32_t": (4, False, False), "int32_t": (4, True, False),
            "int": (4, True, False), "uint64_t": (8, False, False), "int64_t": (8, True, False),
            "size_t": (8, False, False), "float": (4, True, True), "double": (8, True, True),
            **{e: (4, True, False) for e in ENUMS}}


def _snake(camel: str) -> str:
    return re.sub(r"(?<!^)([A-Z])", r"_\1", camel).lower()


RUST_FILE = ROOT / "include" / "lt_kv_sys.rs"


def _rust_blocks() -> str:
    code = RUST_FILE.read_text()
    code = re.sub(r"/\*.*?\*/", "", code, flags=re.S)
    return re.sub(r"//[^\n]*", "", code)


def test_integration_doc_quotes_the_binding_verbatim():
    text = (ROOT / "INTEGRATION.md").read_text()
    quotes = re.findall(r"```rust\n(.*?)```", text, flags=re.S)
    assert quotes, "INTEGRATION.md quotes no Rust"
    src = RUST_FILE.read_text()
    for q in quotes:
        for line in q.strip("\n").split("\n"):
            assert line.strip() in src, f"INTEGRATION.md quotes a line that lt_kv_sys.rs lacks: {line!r}"


def _extern_fns(code: str) -> dict[str, tuple[list[tuple[str, str]], str]]:
    fns = {}
    for block in re.findall(r'extern "C" \{(.*?)\n\s*\}', code, flags=re.S):
        for decl in block.split(";"):
            m = re.search(r"pub fn (\w+)\((.*?)\)\s*(?:->\s*(.+?))?\s*$", decl.strip(), flags=re.S)
            if not m:
                continue
            args = [a.strip() for a in m.group(2).split(",") if a.strip()]
            parsed = []
            for a in args:
                nm, ty = a.split(":", 1)
                parsed.append((nm.strip(), " ".join(ty.split())))
            assert m.group(1) not in fns, f"{m.group(1)} declared twice"
            fns[m.group(1)] = (parsed, " ".join((m.group(3) or "()").split()))
    return fns


def _structs(code: str) -> dict[str, list[tuple[str, str]]]:
    out = {}
    for name, body in re.findall(r"#\[repr\(C\)\]\s*pub struct (\w+)\s*\{(.*?)\}", code, flags=re.S):
        fields = re.findall(r"pub (\w+): ([\w\[\]; ]+)", body)
        if fields:  # opaque handles have only a private zero-sized field
            out[name] = fields
    return out


def _c_pointer(ct: str):
    """'const lt_kv *' -> (pointer depth, whether the outermost pointer's
    pointee is const, base type)."""
    t = " ".join(ct.replace("*", " * ").split())
    toks = t.split(" ")
    depth = toks.count("*")
    base = " ".join(x for x in toks if x not in ("*", "const", "struct"))
    # const-ness of the pointee the outermost pointer points at: 'const' right
    # before the last '*' (or leading, when depth is 1)
    if depth == 0:
        return 0, False, base
    last = len(toks) - 1 - toks[::-1].index("*")
    before = toks[:last]
    pointee_const = (before[-1] == "const") or (depth == 1 and toks[0] == "const")
    return depth, pointee_const, base


def _rust_pointer(rt: str):
    depth, consts = 0, []
    t = rt
    while t.startswith("*"):
        m = re.match(r"\*(const|mut) (.+)", t)
        assert m, rt
        consts.append(m.group(1) == "const")
        t = m.group(2).strip()
        depth += 1
    return depth, (consts[0] if consts else False), t


def _compare(ct: str, rt: str, where: str):
    ct_n = " ".join(ct.split())
    if ct_n == "void":
        assert rt == "()", f"{where}: C returns void, Rust {rt}"
        return
    cd, cconst, cbase = _c_pointer(ct_n)
    rd, rconst, rbase = _rust_pointer(rt)
    assert cd == rd, f"{where}: C {ct!r} has pointer depth {cd}, Rust {rt!r} {rd}"
    if cd:
        assert cconst == rconst, f"{where}: C {ct!r} vs Rust {rt!r}: const-ness of the pointee differs"
        if cbase == "void":
            assert rbase in ("c_void", "u8"), f"{where}: C void pointer, Rust points at {rbase}"
        elif cbase == "char":
            assert rbase == "c_char", f"{where}: C char pointer, Rust points at {rbase}"
        elif cbase in C_SCALAR:
            assert rbase in RUST and RUST[rbase] == C_SCALAR[cbase], f"{where}: C {cbase} vs Rust {rbase}"
        else:
            assert _snake(rbase) == cbase, f"{where}: C points at {cbase}, Rust at {rbase}"
        return
    assert cbase in C_SCALAR, f"{where}: unmapped C type {ct!r}"
    assert rbase in RUST, f"{where}: unmapped Rust type {rt!r}"
    assert RUST[rbase] == C_SCALAR[cbase], f"{where}: C {cbase} {C_SCALAR[cbase]} vs Rust {rbase} {RUST[rbase]}"


# What an engine host calls: the cache and attention (decode, gather over
# NCCL or NVLink, allocation-free), the model step, the scheduler driver and
# the prefix cache.  Parity, profiling and op-level test hooks are left to
# the Python binding.
ENGINE_FACING = {
    "lt_kv_create", "lt_kv_destroy", "lt_kv_last_error", "lt_kv_capacity", "lt_kv_bytes", "lt_kv_len",
    "lt_kv_free_blocks", "lt_kv_append", "lt_kv_write", "lt_kv_attend", "lt_kv_write_attend", "lt_kv_truncate",
    "lt_kv_share", "lt_kv_compact", "lt_kv_flush", "lt_kv_check", "lt_kv_selftest_wait", "lt_kv_build_features",
    "lt_kv_set_cascade", "lt_kv_set_min_tiles_per_warp", "lt_kv_nccl_unique_id", "lt_kv_nccl_init",
    "lt_kv_nccl_destroy", "lt_kv_gather_heads", "lt_kv_peer_export", "lt_kv_peer_import", "lt_kv_peer_close",
    "lt_kv_attend_gather", "lt_kv_write_attend_gather", "lt_paged_attend_noalloc", "lt_paged_attend_noalloc_check",
    "lt_llama_create", "lt_llama_destroy", "lt_llama_last_error", "lt_llama_set_tensor", "lt_llama_forward",
    "lt_llama_step_greedy",
    "lt_sched_create", "lt_sched_destroy", "lt_sched_last_error", "lt_sched_submit", "lt_sched_submit_tokens",
    "lt_sched_step", "lt_sched_get_stats",
    "lt_slot_cache_create", "lt_slot_cache_destroy", "lt_slot_cache_place", "lt_slot_cache_acquire",
    "lt_slot_cache_release", "lt_slot_cache_evict_lru", "lt_slot_cache_idle_cells",
}


def test_rust_extern_declarations_match_the_prototypes():
    protos = H.prototypes()
    fns = _extern_fns(_rust_blocks())
    assert ENGINE_FACING <= set(fns), sorted(ENGINE_FACING - set(fns))
    for name, (args, ret) in sorted(fns.items()):
        assert name in protos, f"{name} is declared in Rust but not in include/*.h"
        cret, cargs = protos[name]
        _compare(cret, ret, f"{name} return")
        assert len(args) == len(cargs), f"{name}: C has {len(cargs)} arguments, Rust {len(args)}"
        for (an, at), ca in zip(args, cargs):
            _compare(ca, at, f"{name}({an})")


def test_rust_repr_c_structs_match_the_c_layout():
    structs = _structs(_rust_blocks())
    assert {"LtKvConfig", "LtLlamaConfig", "LtPlacement"} <= set(structs), sorted(structs)
    got = H.layouts({_snake(s): [f for f, _ in fields] for s, fields in structs.items()})
    for s, fields in structs.items():
        off = 0
        for f, ty in fields:
            size = RUST[ty.strip()][0]
            off = (off + size - 1) // size * size  # repr(C): each scalar aligned to its size
            c_off, c_size = got[_snake(s)][f]
            assert (off, size) == (c_off, c_size), f"{s}.{f}: Rust ({off}, {size}) vs C ({c_off}, {c_size})"
            off += size
        align = max(RUST[ty.strip()][0] for _, ty in fields)
        assert (off + align - 1) // align * align == got[_snake(s)]["sizeof"], f"{s}: sizeof differs"


def test_rust_constants_match_the_headers():
    consts = re.findall(r"pub const (\w+): \w+ = (-?\d+);", _rust_blocks())
    assert consts
    got = H.constants([n for n, _ in consts])
    for n, v in consts:
        assert int(v) == got[n], f"{n}: Rust {v} vs header {got[n]}"
