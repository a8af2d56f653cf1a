"""Builds oracle/_ref/libref.so: the reference's own pre-pass, dtype helpers, output relayout and h3s_rms_rope, cut out
of its kernels/h3sycl.cpp and compiled for the CPU with g++ around oracle/ref_pin.cpp and oracle/ref_shim.h.

TEST INFRASTRUCTURE ONLY. Runs where the reference's source is present (this build machine); the library it makes
travels with the repository's other built files, so the GPU tests can compare against it without the source. The cut
line ranges are checked against the text they must start and end with, so a changed reference fails here instead of
compiling something else.

    python oracle/ref_build.py [path/to/reference]
"""
from __future__ import annotations

import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
OUT = os.path.join(HERE, "_ref")
LIB = os.path.join(OUT, "libref.so")
DEFAULT_REF = "/root/reference"

# (file written into oracle/_ref, first line, last line (1-based, inclusive), text the first and the last line start with)
CUTS = [
    ("h3sycl_dtype.inc", 38, 63, "enum Dt : int { F32 = 0, F16 = 1, BF16 = 2 };", "}"),
    ("h3sycl_rms_rope.inc", 1276, 1376, "int h3s_rms_rope(void* ctx, void* x, int x_dt,",
     "} catch (const std::exception& e) { g_err = e.what(); return -1; }"),
    ("h3sycl_prepass.inc", 1733, 1764, "qu.parallel_for(sycl::range<1>((size_t) (H * D)), [=](sycl::id<1> id) {", "});"),
    ("h3sycl_out.inc", 1769, 1771, "qu.parallel_for(sycl::range<3>((size_t) S, (size_t) H, (size_t) D), [=](sycl::id<3> id) {",
     "});"),
]


def source(ref: str) -> str:
    return os.path.join(ref, "kernels", "h3sycl.cpp")


def available(ref: str = DEFAULT_REF) -> bool:
    return os.path.exists(source(ref))


def build(ref: str = DEFAULT_REF) -> str:
    """Cuts the line ranges into oracle/_ref and compiles libref.so (skipped when it is newer than its inputs)."""
    src = source(ref)
    inputs = [src, os.path.join(HERE, "ref_pin.cpp"), os.path.join(HERE, "ref_shim.h"), os.path.abspath(__file__)]
    if os.path.exists(LIB) and os.path.getmtime(LIB) >= max(os.path.getmtime(p) for p in inputs):
        return LIB
    with open(src) as f:
        lines = f.read().split("\n")
    os.makedirs(OUT, exist_ok=True)
    for name, a, b, first, last in CUTS:
        chunk = lines[a - 1:b]
        if not chunk[0].strip().startswith(first) or not chunk[-1].strip().startswith(last):
            raise RuntimeError(f"{src}:{a}-{b} no longer holds the expected code ({name}): "
                               f"{chunk[0].strip()[:60]!r} ... {chunk[-1].strip()[:60]!r}")
        with open(os.path.join(OUT, name), "w") as f:
            f.write(f"// cut from {src}:{a}-{b} by oracle/ref_build.py (not part of the repository)\n")
            f.write("\n".join(chunk) + "\n")
    cmd = ["g++", "-std=c++17", "-O2", "-ffp-contract=off", "-fno-fast-math", "-fopenmp", "-fPIC", "-shared",
           "-I", OUT, "-I", HERE, os.path.join(HERE, "ref_pin.cpp"), "-o", LIB]
    subprocess.run(cmd, check=True)
    return LIB


if __name__ == "__main__":
    print(build(sys.argv[1] if len(sys.argv) > 1 else DEFAULT_REF))
