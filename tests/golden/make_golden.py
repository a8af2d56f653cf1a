"""Writes the golden fixtures of tests/golden/ from the CPU oracle (oracle/sage_ref.cpp), and recomputes them for the
tests. Run from the repo root: ``python tests/golden/make_golden.py``.

Each fixture holds seeded inputs (q, k, v as the strided parts of one qkv buffer, in the stated element type) and what
the reference's attention path makes of them, as restated by the oracle: the Sage pre-pass (int8 q and k, the q and k
scales per 64-row block, k's channel mean; kernels/h3sycl.cpp:1733-1761) and the h3s_attention output through the Sage
path and through the fp16 SDPA path (kernels/h3sycl.cpp:1779-1798). The reference has no fixture of its own for this
path, so these pin the oracle against regressions and give the GPU tests exact expected int8 / scale bits. Where the
reference's source is present, its own pre-pass lines compiled for the CPU (oracle/_ref/libref.so) must give the same
int8 q / k, scales and mean before a fixture is written (tests/test_ref_pin.py checks the committed ones against it).
"""
from __future__ import annotations

import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))

# name: (S, H, D, dt, out_dt, seed)
CASES = {
    "s1_h1_f16": (1, 1, 128, 1, 1, 11),
    "s65_h2_f16": (65, 2, 128, 1, 1, 12),
    "s130_h1_bf16": (130, 1, 128, 2, 2, 13),
    "s64_h2_f32": (64, 2, 128, 0, 0, 14),
    "s200_h2_f16": (200, 2, 128, 1, 1, 15),
}


def make_inputs(orc, S, H, D, dt, seed):
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((S, 3 * H * D)).astype(np.float32)
    x[:, H * D:2 * H * D] += (rng.standard_normal(H * D) * 2.0).astype(np.float32)
    if dt == orc.F16:
        return orc.f32_to_f16(x)
    if dt == orc.BF16:
        return orc.f32_to_bf16(x)
    return x


def compute(orc, f) -> dict:
    S, H, D, dt, out_dt = (int(f[k]) for k in ("S", "H", "D", "dt", "out_dt"))
    qkv = np.ascontiguousarray(f["qkv"])
    st = 3 * H * D
    iq, ik, qs, ks, km, _ = orc.sage_prepass(qkv, (qkv, H * D), (qkv, 2 * H * D), dt, S, H, D, st)
    if orc.ref_available():
        ref = orc.ref_sage_prepass(qkv, (qkv, H * D), (qkv, 2 * H * D), dt, S, H, D, st)[:5]
        for name, a, b in zip(("iq", "ik", "qs", "ks", "kmean"), (iq, ik, qs, ks, km), ref):
            assert np.array_equal(np.asarray(a).view(np.uint8), np.asarray(b).view(np.uint8)), \
                f"the oracle's {name} differs from the reference's own pre-pass"
    args = (qkv, (qkv, H * D), (qkv, 2 * H * D), dt, S, H, D, st)
    return {
        "iq": iq, "ik": ik, "qs": qs, "ks": ks, "kmean": km,
        "out_sage": orc.attention(*args, out_dt=out_dt, sage_min_s=0),
        "out_sdpa": orc.attention(*args, out_dt=out_dt, sage_min_s=1 << 30),
    }


def main() -> None:
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle as orc

    orc.build()
    for name, (S, H, D, dt, out_dt, seed) in CASES.items():
        f = {"S": S, "H": H, "D": D, "dt": dt, "out_dt": out_dt, "qkv": make_inputs(orc, S, H, D, dt, seed)}
        f.update(compute(orc, f))
        np.savez_compressed(os.path.join(HERE, f"{name}.npz"), **f)
        print(name, {k: getattr(v, "shape", v) for k, v in f.items()})


if __name__ == "__main__":
    main()
