"""The oracle pinned to the reference itself: the reference's own kernels/h3sycl.cpp lines for the attention pre-pass
(:1733-1764), the dtype helpers (:38-63), the output relayout (:1769-1771) and h3s_rms_rope (:1276-1376), compiled for
the CPU from its source (oracle/ref_build.py -> oracle/_ref/libref.so), against the oracle's restatement
(oracle/sage_ref.cpp) and the committed golden fixtures, bit for bit.

This makes "bit-exact with the reference quantiser" a comparison with the reference's code, compiled with strict IEEE
arithmetic (the reference's own binary is built by icpx -O3 for an Intel GPU, which cannot run here). rsqrt is the one
choice the shim makes (SYCL leaves its accuracy to the implementation): correctly rounded, as the GPU kernel."""
import glob
import os

import numpy as np
import pytest

import oracle
from sycl_minimax_h3_b200.workloads import bits, make_qkv

pytestmark = pytest.mark.skipif(not oracle.ref_available(),
                                reason="oracle/_ref/libref.so is not built (needs the reference's source)")

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")


def same(a, b) -> bool:
    a, b = np.asarray(a), np.asarray(b)
    return a.shape == b.shape and np.array_equal(a.view(np.uint8), b.view(np.uint8))


def inputs(S, H, D, dt, seed, extra=0):
    """q | k | v rows (k with per-channel offsets) of element stride 3*H*D + extra, as element bits."""
    rng = np.random.default_rng(seed)
    st = 3 * H * D + extra
    x = rng.standard_normal((S, st)).astype(np.float32)
    x[:, H * D:2 * H * D] += (rng.standard_normal(H * D) * 2.0).astype(np.float32)
    if dt == oracle.F16:
        return oracle.f32_to_f16(x), st
    if dt == oracle.BF16:
        return oracle.f32_to_bf16(x), st
    return x, st


def both(x, dt, S, H, D, st):
    args = (x, (x, H * D), (x, 2 * H * D), dt, S, H, D, st)
    return oracle.sage_prepass(*args), oracle.ref_sage_prepass(*args)


@pytest.mark.parametrize("dt", [oracle.F16, oracle.BF16, oracle.F32])
@pytest.mark.parametrize("S", [1, 2, 63, 64, 65, 127, 130, 200])
@pytest.mark.parametrize("D", [64, 128])
def test_prepass_matches_reference_source(S, D, dt):
    x, st = inputs(S, 2, D, dt, seed=S * 7 + D + dt)
    mine, ref = both(x, dt, S, 2, D, st)
    for name, a, b in zip(("iq", "ik", "qs", "ks", "kmean", "hv"), mine, ref):
        assert same(a, b), f"{name} differs from the reference's own pre-pass (S={S}, D={D}, dt={dt})"


def test_prepass_odd_stride_and_heads():
    """A row stride that is no multiple of anything (3*H*D + 5) and 3 heads."""
    x, st = inputs(150, 3, 128, oracle.F16, seed=3, extra=5)
    mine, ref = both(x, oracle.F16, 150, 3, 128, st)
    assert all(same(a, b) for a, b in zip(mine, ref))


def test_prepass_edge_values():
    """Zero blocks (scale 0, codes 0), one huge value per block, values on rounding ties of the quantiser, and the
    largest half values: the reference's handling of each, bit for bit."""
    S, H, D = 192, 2, 128
    x = np.zeros((S, 3 * H * D), np.float32)
    rng = np.random.default_rng(9)
    x[64:128] = rng.standard_normal((64, 3 * H * D)).astype(np.float32)
    x[64, 5] = 6.0e4                                   # one huge q value: the rest of its block rounds to 0
    x[128:192, :H * D] = (rng.integers(-254, 255, (64, H * D)) / 2.0).astype(np.float32)   # halves: x*inv ties
    x[128, 0] = 127.0                                  # m = 127, inv = 1: the halves are exact ties
    x[128:192, H * D:2 * H * D] = 65504.0 * np.sign(rng.standard_normal((64, H * D))).astype(np.float32)
    h = oracle.f32_to_f16(x)
    mine, ref = both(h, oracle.F16, S, H, D, 3 * H * D)
    assert all(same(a, b) for a, b in zip(mine, ref))


@pytest.mark.parametrize("dt", [oracle.F16, oracle.BF16])
@pytest.mark.parametrize("D", [64, 128])
def test_prepass_nan_inf_values(dt, D):
    """NaN, +-inf, -0, subnormals and an all-NaN channel in a block (the inputs of the GPU edge test): the oracle's
    pre-pass has the reference's bits."""
    import torch
    from _util import edge_qkv
    S, H = 200, 2
    t = edge_qkv(S, H, D, torch.float16 if dt == oracle.F16 else torch.bfloat16, seed=D)
    x = bits(t)
    mine, ref = both(x, dt, S, H, D, 3 * H * D)
    for name, a, b in zip(("iq", "ik", "qs", "ks", "kmean", "hv"), mine, ref):
        assert same(a, b), f"{name} differs from the reference's own pre-pass"


def test_prepass_c0():
    """8 heads x 2,048 tokens, fp16."""
    S, H, D = 2048, 8, 128
    host = bits(make_qkv(S, H, D, seed=0))
    mine, ref = both(host, oracle.F16, S, H, D, 3 * H * D)
    assert all(same(a, b) for a, b in zip(mine, ref))


def test_prepass_c2_full():
    """32 heads x 16,848 tokens (the last block of 16 rows), fp16, whole tensors."""
    S, H, D = 16848, 32, 128
    host = bits(make_qkv(S, H, D, seed=S))
    mine, ref = both(host, oracle.F16, S, H, D, 3 * H * D)
    for name, a, b in zip(("iq", "ik", "qs", "ks", "kmean", "hv"), mine, ref):
        assert same(a, b), name


def test_golden_fixtures_are_the_reference_s():
    """Every committed fixture's int8 q / k, scales and mean are what the reference's own pre-pass makes."""
    paths = sorted(glob.glob(os.path.join(GOLDEN, "*.npz")))
    assert paths
    for path in paths:
        f = np.load(path)
        S, H, D, dt = (int(f[k]) for k in ("S", "H", "D", "dt"))
        x = np.ascontiguousarray(f["qkv"])
        iq, ik, qs, ks, km, _ = oracle.ref_sage_prepass(x, (x, H * D), (x, 2 * H * D), dt, S, H, D, 3 * H * D)
        for name, got in (("iq", iq), ("ik", ik), ("qs", qs), ("ks", ks), ("kmean", km)):
            assert same(got, f[name]), f"{os.path.basename(path)}: {name}"


@pytest.mark.parametrize("out_dt", [oracle.F16, oracle.BF16, oracle.F32])
def test_out_relayout(out_dt):
    """kernels/h3sycl.cpp:1769-1771: half [H, S, D] -> out_dt rows, against the oracle's conversions."""
    S, H, D = 70, 3, 64
    rng = np.random.default_rng(out_dt)
    ao = oracle.f32_to_f16((rng.standard_normal((H, S, D)) * 100).astype(np.float32))
    got = oracle.ref_out_relayout(ao, out_dt, S, H, D)
    f = oracle.f16_to_f32(ao).transpose(1, 0, 2).reshape(S, H * D)
    want = {oracle.F16: lambda v: oracle.f32_to_f16(v), oracle.BF16: lambda v: oracle.f32_to_bf16(v),
            oracle.F32: lambda v: v.astype(np.float32)}[out_dt](np.ascontiguousarray(f))
    assert same(got, want)


def test_dtype_helpers():
    """kernels/h3sycl.cpp:42-63 against the oracle's conversions: round-to-nearest-even ties, subnormals, overflow,
    infinities and NaN."""
    specials = np.array([0.0, -0.0, 1.0, -2.5, 65504.0, 65520.0, 1e-8, 6.1e-5, 3.0e38, np.inf, -np.inf, np.nan,
                         1.00390625, 1.01171875, 0.1, 1.0 + 2 ** -8, 1.0 + 3 * 2 ** -8], np.float32)
    vals = np.concatenate([specials, np.random.default_rng(1).standard_normal(500).astype(np.float32) * 1e3])
    assert same(oracle.ref_store(vals, oracle.BF16), oracle.f32_to_bf16(vals))
    assert same(oracle.ref_store(vals, oracle.F16), oracle.f32_to_f16(vals))
    allb = np.arange(0, 65536, 7, dtype=np.uint16)
    a, b = oracle.ref_load(allb, oracle.BF16), oracle.bf16_to_f32(allb)
    assert same(np.where(np.isnan(a), np.float32(0), a), np.where(np.isnan(b), np.float32(0), b))
    a, b = oracle.ref_load(allb, oracle.F16), oracle.f16_to_f32(allb)
    assert same(np.where(np.isnan(a), np.float32(0), a), np.where(np.isnan(b), np.float32(0), b))


@pytest.mark.parametrize("dt", [oracle.F16, oracle.BF16, oracle.F32])
@pytest.mark.parametrize("D,rot", [(128, 128), (128, 96), (128, 0), (64, 64), (128, 120), (96, 30), (100, 20)])
def test_rms_rope_matches_reference_source(dt, D, rot):
    """The oracle's h3s_rms_rope against the reference's, both of its kernels (the 16-byte one for aligned 16-bit rows,
    the element one otherwise), rows inside a qkv buffer."""
    for M, offset in ((1, 0), (129, 0), (60, 3)):
        rng = np.random.default_rng(M + D + rot + dt)
        H = 3
        stride = 3 * H * D + offset
        x = (rng.standard_normal(M * stride + offset) * 3).astype(np.float32)
        host = x if dt == oracle.F32 else (oracle.f32_to_f16(x) if dt == oracle.F16 else oracle.f32_to_bf16(x))
        w = (1 + 0.2 * rng.standard_normal(D)).astype(np.float32)
        ang = rng.random((M, rot // 2)) * 14 - 7
        cs = np.stack([np.cos(ang), np.sin(ang)], -1).astype(np.float32)
        sub = np.ascontiguousarray(host[offset:])
        want = oracle.ref_rms_rope(sub, dt, M, H, D, stride, w, 1e-5, cs, rot)
        got = oracle.rms_rope(sub, dt, M, H, D, stride, w, 1e-5, cs, rot)
        assert same(got, want), f"M={M}, offset={offset}: {np.count_nonzero(got != want)} differ"


def test_rms_rope_refusals_match():
    x = np.zeros(4 * 128, np.float32)
    w = np.ones(128, np.float32)
    cs = np.zeros((4, 64, 2), np.float32)
    for rot in (3, 130):
        with pytest.raises(ValueError):
            oracle.ref_rms_rope(x, oracle.F32, 4, 1, 128, 128, w, 1e-5, cs, rot)
        with pytest.raises(ValueError):
            oracle.rms_rope(x, oracle.F32, 4, 1, 128, 128, w, 1e-5, cs, rot)
