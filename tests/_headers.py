"""The C headers as the compiler sees them, for tests that compare a binding
(ctypes, or the Rust declarations in the integration notes) with include/*.h.

prototypes() runs gcc -aux-info over the headers: name -> (return type,
[argument types]) in gcc's normalised spelling.  layouts() compiles a small
program printing sizeof/offsetof of the given struct fields.  Host gcc only.
"""
from __future__ import annotations

import re
import subprocess
import tempfile
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]
HEADERS = ("lt_kv.h", "lt_llama.h", "lt_sched.h", "lt_prefix.h")


def have_gcc() -> bool:
    try:
        subprocess.run(["gcc", "--version"], capture_output=True, check=True)
        return True
    except (OSError, subprocess.CalledProcessError):
        return False


def prototypes() -> dict[str, tuple[str, list[str]]]:
    with tempfile.TemporaryDirectory() as d:
        src = Path(d) / "hdr.c"
        src.write_text("".join(f'#include "{h}"\n' for h in HEADERS))
        aux = Path(d) / "aux.txt"
        subprocess.run(["gcc", "-I", str(ROOT / "include"), "-aux-info", str(aux), "-fsyntax-only", str(src)],
                       check=True, capture_output=True, text=True)
        text = aux.read_text()
    protos = {}
    pat = re.compile(r"^/\* (\S+?):\d+:\w+ \*/ extern (.+?)\s*\b(lt_\w+) \((.*)\);$")
    for line in text.splitlines():
        m = pat.match(line)
        if not m or Path(m.group(1)).name not in HEADERS:
            continue
        ret, name, args = m.group(2).strip(), m.group(3), m.group(4).strip()
        protos[name] = (ret, [] if args in ("", "void") else [a.strip() for a in args.split(",")])
    assert len(protos) > 50, "no prototypes parsed from gcc -aux-info"
    return protos


def _run_c(body: list[str]) -> str:
    lines = [f'#include "{h}"' for h in HEADERS] + ["#include <stddef.h>", "#include <stdio.h>", "int main(void) {"]
    lines += body + ["    return 0;", "}"]
    with tempfile.TemporaryDirectory() as d:
        src, exe = Path(d) / "probe.c", Path(d) / "probe"
        src.write_text("\n".join(lines) + "\n")
        r = subprocess.run(["gcc", "-I", str(ROOT / "include"), "-o", str(exe), str(src)], capture_output=True,
                           text=True)
        assert r.returncode == 0, r.stderr  # a name the binding uses that C lacks fails here
        return subprocess.run([str(exe)], capture_output=True, text=True, check=True).stdout


def layouts(structs: dict[str, list[str]]) -> dict[str, dict]:
    """struct -> {"sizeof": n, field: (offset, size)} for the named fields."""
    body = []
    for s, fields in structs.items():
        body.append(f'    printf("{s} sizeof %zu 0\\n", sizeof({s}));')
        body += [f'    printf("{s} {f} %zu %zu\\n", offsetof({s}, {f}), sizeof((({s}*)0)->{f}));' for f in fields]
    out: dict[str, dict] = {s: {} for s in structs}
    for line in _run_c(body).splitlines():
        s, f, a, b = line.split()
        out[s][f] = int(a) if f == "sizeof" else (int(a), int(b))
    return out


def constants(names: list[str]) -> dict[str, int]:
    body = [f'    printf("{n} %lld\\n", (long long)({n}));' for n in names]
    out = _run_c(body).split()
    return dict(zip(out[0::2], (int(x) for x in out[1::2])))
