"""The CPU oracle pinned: against the reference's own known-answer tests (dtype conversions, engine/h3-core/src/dtype.rs
:137-155), against an independent numpy restatement of the reference quantiser (kernels/h3sycl.cpp:1733-1761), against
float64 softmax attention, and against the committed golden fixtures (tests/golden/)."""
import glob
import os

import numpy as np
import pytest

import oracle

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def f32(bits_u32):
    return np.array(bits_u32, np.uint32).view(np.float32)


# ---- dtype helpers: the reference's own known answers --------------------------------------------------------------
def test_bf16_known_answers(orc):
    # engine/h3-core/src/dtype.rs:145-147: ties go to even
    assert orc.f32_to_bf16(f32([0x3F808000]))[0] == 0x3F80
    assert orc.f32_to_bf16(f32([0x3F818000]))[0] == 0x3F82
    # dtype.rs:139-143: round trip within 0.4 %
    v = np.array([0.0, 1.0, -1.0, 0.5, 3.140625, -1234.0, 1e-20], np.float32)
    r = orc.bf16_to_f32(orc.f32_to_bf16(v))
    assert np.all(np.abs(r - v) <= np.abs(v) * 0.004)


def test_f16_known_answers(orc):
    # engine/h3-core/src/dtype.rs:149-155
    got = orc.f16_to_f32(np.array([0x3C00, 0xC000, 0x0001, 0x7C00, 0x0000], np.uint16))
    assert got[0] == 1.0 and got[1] == -2.0 and got[2] == np.float32(5.9604645e-8) and np.isinf(got[3]) and got[4] == 0.0


def test_f16_matches_ieee(orc):
    h = np.arange(65536, dtype=np.uint16)
    ref = h.view(np.float16).astype(np.float32)
    got = orc.f16_to_f32(h)
    ok = ~np.isnan(ref)
    assert np.array_equal(got.view(np.uint32)[ok], ref.view(np.uint32)[ok]) and np.all(np.isnan(got[~ok]))
    rng = np.random.default_rng(0)
    x = (rng.standard_normal(1 << 18) * np.exp(rng.uniform(-25, 12, 1 << 18))).astype(np.float32)
    x = np.concatenate([x, np.array([65504, 65519.99, 65520, 2.98e-8, 2.9802322e-8, 5.96e-8, -0.0], np.float32)])
    with np.errstate(over="ignore"):
        assert np.array_equal(orc.f32_to_f16(x), x.astype(np.float16).view(np.uint16))


def test_bf16_matches_rne(orc):
    rng = np.random.default_rng(1)
    u = rng.integers(0, 1 << 32, 1 << 18, dtype=np.uint64).astype(np.uint32)
    u = u[(u & 0x7F800000) != 0x7F800000]
    got = orc.f32_to_bf16(u.view(np.float32))
    lsb = (u >> 16) & 1
    want = ((u.astype(np.uint64) + 0x7FFF + lsb) >> 16).astype(np.uint16)
    assert np.array_equal(got, want)


# ---- the quantiser against an independent numpy restatement ---------------------------------------------------------
def round_half_away(x):
    t = np.trunc(x)
    return t + np.where(np.abs(x - t) >= 0.5, np.sign(x), 0).astype(x.dtype)


def np_kmean(kf):
    return (np.add.accumulate(kf, axis=0, dtype=np.float32)[-1] / np.float32(kf.shape[0])).astype(np.float32)


def np_quant(xf, mean, S, H, D):
    nb = (S + 63) // 64
    dst = np.zeros((H, S, D), np.int8)
    sc = np.zeros((H, nb), np.float32)
    for h in range(H):
        for b in range(nb):
            blk = xf[b * 64:(b + 1) * 64, h * D:(h + 1) * D]
            y = (blk - (mean[h * D:(h + 1) * D] if mean is not None else np.float32(0))).astype(np.float32)
            m = np.float32(np.max(np.abs(y)))
            inv = np.float32(127) / m if m > 0 else np.float32(0)
            sc[h, b] = m / np.float32(127)
            dst[h, b * 64:b * 64 + blk.shape[0]] = np.clip(round_half_away((y * inv).astype(np.float32)), -127, 127)
    return dst, sc


def to_dt(orc, x, dt):
    if dt == orc.F16:
        return orc.f32_to_f16(x), orc.f16_to_f32(orc.f32_to_f16(x))
    if dt == orc.BF16:
        return orc.f32_to_bf16(x), orc.bf16_to_f32(orc.f32_to_bf16(x))
    return x.astype(np.float32), x.astype(np.float32)


@pytest.mark.parametrize("S", [1, 63, 64, 65, 200])
@pytest.mark.parametrize("dt", [1, 2, 0])
def test_quantiser_matches_numpy(orc, S, dt):
    H, D = 2, 128
    st = 3 * H * D + 8
    rng = np.random.default_rng(S * 10 + dt)
    x = rng.standard_normal((S, st)).astype(np.float32)
    x[:, H * D:2 * H * D] += (rng.standard_normal(H * D) * 2).astype(np.float32)
    raw, val = to_dt(orc, x, dt)
    kval = np.ascontiguousarray(val[:, H * D:2 * H * D])
    km = orc.kmean((raw, H * D), dt, S, H, D, st)
    assert np.array_equal(km.view(np.uint32), np_kmean(kval).view(np.uint32))
    iq, qs = orc.quant(raw, dt, S, H, D, st)
    wq, wqs = np_quant(np.ascontiguousarray(val[:, :H * D]), None, S, H, D)
    assert np.array_equal(iq, wq) and np.array_equal(qs.view(np.uint32), wqs.view(np.uint32))
    ik, ks = orc.quant((raw, H * D), dt, S, H, D, st, km)
    wk, wks = np_quant(kval, km, S, H, D)
    assert np.array_equal(ik, wk) and np.array_equal(ks.view(np.uint32), wks.view(np.uint32))


def test_quantiser_edges(orc):
    """round half away from zero, clamp at +-127 (never -128), an all-zero block gives scale 0 and zeros."""
    S, H, D = 128, 1, 128
    x = np.zeros((S, D), np.float32)
    x[0, 0] = 127.0                        # block 0: m = 127, inv = 1
    x[0, 1], x[0, 2], x[0, 3], x[0, 4] = 2.5, -2.5, 0.5, -127.0
    iq, qs = orc.quant(x, orc.F32, S, H, D, D)
    assert qs[0, 0] == np.float32(1.0) and qs[0, 1] == 0.0
    assert list(iq[0, 0, :5]) == [127, 3, -3, 1, -127]
    assert np.all(iq[0, 64:] == 0) and iq.min() >= -127


def test_prepass_layout(orc):
    """sc = q scales [H, nb] | k scales [H, nb] | k mean [H*D] (kernels/h3sycl.cpp:1716-1718)."""
    S, H, D = 130, 2, 128
    rng = np.random.default_rng(3)
    raw = orc.f32_to_f16(rng.standard_normal((S, 3 * H * D)).astype(np.float32))
    iq, ik, qs, ks, km, hv = orc.sage_prepass(raw, (raw, H * D), (raw, 2 * H * D), orc.F16, S, H, D, 3 * H * D)
    assert qs.shape == (H, 3) and ks.shape == (H, 3) and km.shape == (H * D,)
    assert np.array_equal(hv[1, 5], raw[5, 2 * H * D + D:2 * H * D + 2 * D])
    assert np.array_equal(km, orc.kmean((raw, H * D), orc.F16, S, H, D, 3 * H * D))


# ---- attention semantics against float64 ----------------------------------------------------------------------------
def _qkv(S, H, D, seed):
    from sycl_minimax_h3_b200.workloads import bits, make_qkv

    return bits(make_qkv(S, H, D, seed=seed))


@pytest.mark.parametrize("S", [1, 65, 384])
def test_sage_and_sdpa_semantics_vs_exact(orc, S):
    H, D = 2, 128
    host = _qkv(S, H, D, seed=S)
    st = 3 * H * D
    rh, rs = np.repeat(np.arange(H), S), np.tile(np.arange(S), H)
    exact = orc.exact_rows(host, (host, H * D), (host, 2 * H * D), orc.F16, S, H, D, st, rh, rs)
    iq, ik, qs, ks, km, hv = orc.sage_prepass(host, (host, H * D), (host, 2 * H * D), orc.F16, S, H, D, st)
    sage = orc.sage_rows(iq, ik, hv, qs, ks, S, H, D, rh, rs).view(np.float16).astype(np.float32)
    sdpa = orc.sdpa_rows(host, (host, H * D), (host, 2 * H * D), orc.F16, S, H, D, st, rh, rs).view(np.float16).astype(np.float32)
    assert orc.row_cosines(sage, exact).min() >= 0.999
    assert orc.row_cosines(sdpa, exact).min() >= 0.9999
    rel, cos = orc.compare(sdpa, exact)
    assert rel < 1e-2 and cos > 0.9999


def test_dispatch_threshold(orc):
    """h3s_attention: Sage at S >= sage_min_s, fp16 SDPA below (kernels/h3sycl.cpp:1784)."""
    S, H, D = 96, 2, 128
    host = _qkv(S, H, D, seed=11)
    st = 3 * H * D
    rh, rs = np.repeat(np.arange(H), S), np.tile(np.arange(S), H)
    a_sdpa = orc.attention(host, (host, H * D), (host, 2 * H * D), orc.F16, S, H, D, st, orc.F16, sage_min_s=S + 1)
    a_sage = orc.attention(host, (host, H * D), (host, 2 * H * D), orc.F16, S, H, D, st, orc.F16, sage_min_s=S)
    want_sdpa = orc.sdpa_rows(host, (host, H * D), (host, 2 * H * D), orc.F16, S, H, D, st, rh, rs)
    assert np.array_equal(a_sdpa.reshape(S, H, D).transpose(1, 0, 2).reshape(H * S, D), want_sdpa)
    assert not np.array_equal(a_sage, a_sdpa)
    with pytest.raises(ValueError):
        orc.attention(host, host, host, orc.F16, S, H, D, H * D - 1)


def test_out_dtypes_round_through_half(orc):
    S, H, D = 40, 1, 128
    host = _qkv(S, H, D, seed=2)
    args = (host, (host, H * D), (host, 2 * H * D), orc.F16, S, H, D, 3 * H * D)
    o16 = orc.attention(*args, out_dt=orc.F16, sage_min_s=1 << 30)
    o32 = orc.attention(*args, out_dt=orc.F32, sage_min_s=1 << 30)
    obf = orc.attention(*args, out_dt=orc.BF16, sage_min_s=1 << 30)
    assert np.array_equal(o32, o16.view(np.float16).astype(np.float32))
    assert np.array_equal(obf, orc.f32_to_bf16(o16.view(np.float16).astype(np.float32)))


# ---- golden fixtures --------------------------------------------------------------------------------------------------
FIXTURES = sorted(glob.glob(os.path.join(GOLDEN, "*.npz")))


def test_golden_fixtures_exist():
    assert FIXTURES, "tests/golden/*.npz missing (tests/golden/make_golden.py writes them)"


@pytest.mark.parametrize("path", FIXTURES, ids=[os.path.basename(p) for p in FIXTURES])
def test_golden_fixture(orc, path):
    import sys

    sys.path.insert(0, GOLDEN)
    import make_golden

    f = np.load(path)
    got = make_golden.compute(orc, f)
    for key, want in got.items():
        assert np.array_equal(np.asarray(f[key]).view(np.uint8), np.asarray(want).view(np.uint8)), f"{path}: {key} differs"


# ---- RMS norm + RoPE (kernels/h3sycl.cpp:1276-1376) against an independent numpy restatement -------------------------
def numpy_rms_rope(x: np.ndarray, M: int, H: int, D: int, w: np.ndarray, eps: float, cs: np.ndarray, rot: int,
                   narrow) -> np.ndarray:
    """float32 [M, H, D] values -> results rounded by `narrow`; the same operation order, float32 throughout."""
    v = x.astype(np.float32)
    s = np.add.accumulate(v * v, axis=-1, dtype=np.float32)[..., -1]          # feature order, every step rounded
    arg = (s / np.float32(D) + np.float32(eps)).astype(np.float32)
    inv = (1.0 / np.sqrt(arg.astype(np.float64))).astype(np.float32)[..., None]
    half = rot // 2
    y = (v * inv * w).astype(np.float32)
    a, b = y[..., :half].copy(), y[..., half:rot].copy()
    co, si = cs[:, None, :, 0], cs[:, None, :, 1]
    y[..., :half] = a * co - b * si
    y[..., half:rot] = b * co + a * si
    return narrow(y)


@pytest.mark.parametrize("D,rot", [(128, 128), (128, 96), (128, 0), (64, 64), (96, 30)])
@pytest.mark.parametrize("dt", ["f16", "bf16", "f32"])
def test_rms_rope_matches_numpy(orc, D, rot, dt):
    rng = np.random.default_rng(D + rot)
    M, H = 37, 3
    stride = 3 * H * D
    vals = (rng.standard_normal((M, stride)) * 3).astype(np.float32)
    w = (1 + 0.2 * rng.standard_normal(D)).astype(np.float32)
    ang = rng.uniform(-7, 7, (M, rot // 2)).astype(np.float32)
    cs = np.ascontiguousarray(np.stack([np.cos(ang), np.sin(ang)], -1).astype(np.float32))
    if dt == "f16":
        code, x = orc.F16, vals.astype(np.float16).view(np.uint16)
        widen, narrow = (lambda b: b.view(np.float16).astype(np.float32)), (lambda y: y.astype(np.float16).view(np.uint16))
    elif dt == "bf16":
        code, x = orc.BF16, orc.f32_to_bf16(vals)
        widen, narrow = orc.bf16_to_f32, (lambda y: orc.f32_to_bf16(np.ascontiguousarray(y)).reshape(y.shape))
    else:
        code, x = orc.F32, vals
        widen, narrow = (lambda b: b), (lambda y: y)
    got = orc.rms_rope(x, code, M, H, D, stride, w, 1e-5, cs, rot)
    part = widen(np.ascontiguousarray(x[:, :H * D]).reshape(-1)).reshape(M, H, D)
    want = numpy_rms_rope(part, M, H, D, w, 1e-5, cs, rot, narrow)
    assert np.array_equal(np.asarray(got[:, :H * D]).reshape(M, H, D), np.asarray(want).reshape(M, H, D))
    assert np.array_equal(got[:, H * D:], x[:, H * D:])          # the rest of each row untouched


def test_rms_rope_refusals(orc):
    x = np.zeros((2, 128), np.float32)
    w = np.ones(128, np.float32)
    cs = np.zeros(2 * 128, np.float32)
    for rot in (3, 130, -2):
        with pytest.raises(ValueError):
            orc.rms_rope(x, orc.F32, 2, 1, 128, 128, w, 1e-5, cs, rot)
    with pytest.raises(ValueError):
        orc.rms_rope(x, orc.F32, 1, 2, 128, 128, w, 1e-5, cs, 128)     # stride < H * D


# ---- causal attention with grouped heads (kernels/h3sycl.cpp:870-898) against float64 numpy ---------------------------
def numpy_causal(q, k, v, L, Hq, Hkv, D):
    """float64 causal softmax attention; q [L, Hq, D], k, v [L, Hkv, D] as float64."""
    out = np.zeros((L, Hq, D))
    grp = Hq // Hkv
    mask = np.tril(np.ones((L, L), bool))
    for h in range(Hq):
        s = q[:, h, :] @ k[:, h // grp, :].T / np.sqrt(D)
        s = np.where(mask, s, -np.inf)
        p = np.exp(s - s.max(1, keepdims=True))
        out[:, h, :] = (p / p.sum(1, keepdims=True)) @ v[:, h // grp, :]
    return out


@pytest.mark.parametrize("L,Hq,Hkv,D", [(1, 2, 1, 128), (37, 4, 2, 128), (90, 3, 3, 64), (50, 4, 1, 96)])
def test_causal_matches_float64(orc, L, Hq, Hkv, D):
    rng = np.random.default_rng(L + D)
    q = rng.standard_normal((L, Hq * D)).astype(np.float32)
    k = rng.standard_normal((L, Hkv * D)).astype(np.float32)
    v = rng.standard_normal((L, Hkv * D)).astype(np.float32)
    got = orc.attention_causal(q, k, v, orc.F32, L, Hq, Hkv, D, Hq * D, Hkv * D)
    want = numpy_causal(q.reshape(L, Hq, D).astype(np.float64), k.reshape(L, Hkv, D).astype(np.float64),
                        v.reshape(L, Hkv, D).astype(np.float64), L, Hq, Hkv, D)
    assert np.max(np.abs(got.reshape(L, Hq, D) - want)) < 1e-5


def test_causal_refusals(orc):
    x = np.zeros((2, 512), np.float32)
    with pytest.raises(ValueError):
        orc.attention_causal(x, x, x, orc.F32, 2, 1, 1, 512, 512, 512)      # D > 256
    with pytest.raises(ValueError):
        orc.attention_causal(x, x, x, orc.F32, 2, 3, 2, 128, 512, 512)      # Hq not a multiple of Hkv


# ---- int8 ConvRot linear (kernels/h3sycl.cpp:404-652; engine/h3-core/src/reference.rs:37-132) ----------------------
def _hadamard(g):
    """The reference's normalised Hadamard matrix builder (kernels/h3sycl.cpp:185-200), in float64."""
    h4 = np.array([[1, 1, 1, -1], [1, 1, -1, 1], [1, -1, 1, 1], [-1, 1, 1, 1]])
    h = np.zeros((g, g))
    norm = 1.0
    s = 1
    while s < g:
        norm *= 0.5
        s *= 4
    for i in range(g):
        for j in range(g):
            sign, a, b, s = 1, i, j, 1
            while s < g:
                sign *= h4[a % 4][b % 4]
                a, b, s = a // 4, b // 4, s * 4
            h[i, j] = sign * norm
    return h


def _compare(a, b):
    """reference.rs:85-95: relative error and cosine."""
    a, b = a.astype(np.float64).ravel(), b.astype(np.float64).ravel()
    return np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-300), a @ b / max(np.linalg.norm(a) * np.linalg.norm(b), 1e-300)


@pytest.mark.parametrize("g", [4, 16, 64])
def test_hadamard_is_orthonormal(g):
    """reference.rs:105-113."""
    h = _hadamard(g)
    assert np.allclose(h @ h.T, np.eye(g), atol=1e-12)


def test_int8_linear_matches_a_plain_linear_within_quantization(orc):
    """reference.rs:115-127 on both restatements: weights exactly int8 * scale, no rotation."""
    m, k, n = 3, 64, 5
    rng = np.random.default_rng(7)
    x = rng.standard_normal((m, k)).astype(np.float32)
    w = rng.integers(-127, 128, (n, k)).astype(np.int8)
    ws = np.array([0.01], np.float32)
    want = (x.astype(np.float64) @ w.astype(np.float64).T) * 0.01
    for got in (orc.int8_linear_dense(x, m, k, w, n, ws, None, 0),
                orc.int8_linear(x, orc.F32, m, k, w, n, ws, None, orc.F32, 0)):
        rel, cos = _compare(got, want)
        assert rel < 0.02 and cos > 0.999, (rel, cos)


@pytest.mark.parametrize("g", [2, 4, 8, 16, 32, 64, 128, 256])
def test_butterfly_matches_the_dense_rotation(orc, g):
    """The butterfly (the fused kernel's order) against the dense rotation with the matrix the library builds
    (kernels/h3sycl.cpp:185-200), for every group the entry point accepts (2 * 4^n included, where that matrix is
    singular in its top digit and its norm is 1/2 per base-4 digit), and against reference.rs's dense product for the
    powers of 4 it is defined on (reference.rs:4-5; its norm 1/sqrt(g) is the library's there): the rotated values
    differ by float rounding only, so at most a few quantisation levels move, by one."""
    M, K, N = 16, 1024, 24
    rng = np.random.default_rng(g)
    x = (rng.standard_normal((M, K)) * 3).astype(np.float32)
    w = rng.integers(-127, 128, (N, K)).astype(np.int8)
    ws = (rng.random(N) * 0.01 + 1e-3).astype(np.float32)
    b = rng.standard_normal(N).astype(np.float32)
    a = orc.int8_linear(x, orc.F32, M, K, w, N, ws, b, orc.F32, g)
    if g in (4, 16, 64, 256):
        d = orc.int8_linear_dense(x, M, K, w, N, ws, b, g)
        rel, cos = _compare(a, d)
        assert rel < 2e-3 and cos > 0.99999, (rel, cos)
    # and the float64 rotation with the reference's matrix, quantised the same way, agrees as closely
    xr = (x.astype(np.float64).reshape(M, K // g, g) @ _hadamard(g)).reshape(M, K)
    s = np.maximum(np.abs(xr).max(1) / 127, 1e-30)
    q = np.clip(np.rint(xr / s[:, None]), -128, 127)
    exact = (q @ w.astype(np.float64).T) * s[:, None] * ws[None, :] + b[None, :]
    rel, _ = _compare(a, exact)
    assert rel < 2e-3, rel


def test_rotated_weights_recover_the_plain_linear(orc):
    """With W stored rotated (W . H per group, quantised per output row) the rotation cancels: the layer is within
    quantisation of x . W^T (what int8_convrot checkpoints rely on)."""
    M, K, N, g = 8, 512, 32, 256
    rng = np.random.default_rng(3)
    x = rng.standard_normal((M, K)).astype(np.float32)
    wf = rng.standard_normal((N, K)) / 16
    wr = (wf.reshape(N, K // g, g) @ _hadamard(g)).reshape(N, K)
    sc = np.abs(wr).max(1) / 127
    wq = np.clip(np.rint(wr / sc[:, None]), -127, 127).astype(np.int8)
    got = orc.int8_linear(x, orc.F32, M, K, wq, N, sc.astype(np.float32), None, orc.F32, g)
    rel, cos = _compare(got, x.astype(np.float64) @ wf.T)
    assert rel < 0.02 and cos > 0.999, (rel, cos)


def test_rotq_scale_and_clamp(orc):
    """Row scale = max(absmax / 127, 1e-30); the largest value of a row quantises to +-127; a zero row keeps the floor
    scale and all-zero codes."""
    x = np.zeros((3, 64), np.float32)
    x[1] = np.linspace(-5, 3, 64)
    x[2, 5] = 1e-20
    q, s = orc.rotq(x, orc.F32, 3, 64, 0)
    assert s[0] == np.float32(1e-30) and not q[0].any()
    assert s[1] == np.float32(np.float32(5) / np.float32(127)) and q[1, 0] == -127 and q[1].max() <= 127
    assert q[2, 5] == 127
