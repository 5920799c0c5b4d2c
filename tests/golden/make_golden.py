"""Generate tests/golden/f16_convert.npz: f32 -> f16 known answers.

The reference converts K/V rows with `half::f16::from_f32` (half 2.7.1, call
sites engine/crates/native/src/kv.rs:126,129).  On x86-64 that crate uses the
F16C instruction VCVTPS2PH with round-to-nearest-even when the CPU has it,
so the answers here come from that instruction (a tiny C helper compiled
with gcc -mf16c and run on this host), cross-checked against numpy's
independent IEEE conversion for every non-NaN input.

Inputs cover every class: signed zeros, f32 subnormals, f16 subnormal range
and its underflow boundary, round-half-even ties at several exponents, the
overflow boundary (65504 / 65519.99 / 65520), infinities, quiet and
signalling NaNs with assorted payloads, plus 20k seeded random patterns.

Run:  python tests/golden/make_golden.py
"""
from __future__ import annotations

import os
import subprocess
import tempfile
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent

C_HELPER = r"""
#include <immintrin.h>
#include <stdint.h>
#include <stdio.h>
#include <string.h>
int main(int argc, char** argv) {
    FILE* in = fopen(argv[1], "rb");
    FILE* out = fopen(argv[2], "wb");
    uint32_t x;
    while (fread(&x, 4, 1, in) == 1) {
        float f; memcpy(&f, &x, 4);
        uint16_t h = _cvtss_sh(f, _MM_FROUND_TO_NEAREST_INT);
        fwrite(&h, 2, 1, out);
    }
    fclose(in); fclose(out);
    return 0;
}
"""


def inputs() -> np.ndarray:
    u = []
    f = lambda v: np.array([v], np.float32).view(np.uint32)[0]
    for s in (0, 0x80000000):
        u += [s | 0, s | 1, s | 0x7FFFFF, s | 0x00800000]  # zeros, f32 subnormals, min normal
        u += [s | 0x7F800000]  # inf
        for payload in (1, 2, 0x1000, 0x1FFF, 0x2000, 0x3FFFFF, 0x400000, 0x400001, 0x7FFFFF):
            u.append(s | 0x7F800000 | payload)  # NaNs: signalling (< 0x400000) and quiet
        for v in (65504.0, 65519.0, 65519.996, 65520.0, 65536.0, 1e10, 2.0 ** -24, 2.0 ** -25,
                  1.5 * 2.0 ** -25, 2.0 ** -26, 2.0 ** -14, 2.0 ** -15, 1.0, 1.0 + 2.0 ** -11,
                  1.0 + 3 * 2.0 ** -11, 1.0 + 2.0 ** -11 + 2.0 ** -20, 0.1, 3.14159265, 1000.0):
            u.append(s | (f(v) & 0x7FFFFFFF))
    # round-half-even ties and neighbours across the whole f16 exponent range
    for e in range(-24, 16):
        base = f(2.0 ** e) & 0x7F800000
        for m in (0x000000, 0x001000, 0x002000, 0x003000, 0x000FFF, 0x001001, 0x7FF000, 0x7FE000):
            u.append(base | m)
    rng = np.random.default_rng(0)
    u = np.array(u, dtype=np.uint32)
    rand = rng.integers(0, 2 ** 32, size=20000, dtype=np.uint64).astype(np.uint32)
    near = (rng.standard_normal(20000).astype(np.float32) * np.float32(3.0)).view(np.uint32)
    return np.concatenate([u, rand, near])


def f16c_convert(x: np.ndarray) -> np.ndarray:
    with tempfile.TemporaryDirectory() as d:
        src, exe = os.path.join(d, "cvt.c"), os.path.join(d, "cvt")
        Path(src).write_text(C_HELPER)
        subprocess.run(["gcc", "-O1", "-mf16c", "-o", exe, src], check=True)
        fin, fout = os.path.join(d, "in.bin"), os.path.join(d, "out.bin")
        x.astype(np.uint32).tofile(fin)
        subprocess.run([exe, fin, fout], check=True)
        return np.fromfile(fout, dtype=np.uint16)


def main():
    x = inputs()
    h = f16c_convert(x)
    f = x.view(np.float32)
    nan = np.isnan(f)
    with np.errstate(over="ignore"):
        ref = f.astype(np.float16).view(np.uint16)
    assert np.array_equal(ref[~nan], h[~nan]), "F16C and numpy disagree on a non-NaN input"
    np.savez_compressed(HERE / "f16_convert.npz", f32_bits=x, f16_bits=h)
    print(f"wrote {len(x)} vectors ({int(nan.sum())} NaN)")


if __name__ == "__main__":
    main()
