"""Helpers shared by the tests: running the product through its C ABI and checking it with the oracle."""
from __future__ import annotations

import os

import numpy as np
import torch

import oracle
from sycl_minimax_h3_b200 import native, ops
from sycl_minimax_h3_b200.workloads import bits, make_qkv

# Tolerances of the attention outputs: per-row cosine >= 0.999 against float64 softmax of
# the same inputs; max-abs error is measured and reported, and bounded loosely here (the outputs are O(0.1..1)).
MIN_ROW_COSINE = 0.999
MAX_ABS_VS_EXACT = 0.05
# Against the oracle's restatement of the same arithmetic (same quantised inputs, same rounding points; the GPU's
# online softmax rescales lazily and uses ex2.approx, so half-precision P can round differently).
MIN_ROW_COSINE_VS_SAME_SEMANTICS = 0.9999


def tok_rows_to_head_rows(out: np.ndarray, S: int, H: int, D: int) -> np.ndarray:
    """[S, H*D] -> [H*S, D] in (head, token) order, as the oracle's row lists."""
    return out.reshape(S, H, D).transpose(1, 0, 2).reshape(H * S, D)


def half_bits_to_f32(x: np.ndarray) -> np.ndarray:
    return x.view(np.float16).astype(np.float32)


def run_attention(qkv: torch.Tensor, H: int, D: int, out_dtype=torch.float16, min_s: int | None = None) -> torch.Tensor:
    """h3s_attention on q, k, v as the strided parts of a qkv buffer (the engine's layout)."""
    if min_s is not None:
        os.environ["H3S_SAGE_MIN_S"] = str(min_s)
    else:
        os.environ.pop("H3S_SAGE_MIN_S", None)
    ops._ctx.clear()
    try:
        q, k, v = ops.Rows.qkv(qkv, H, D)
        out = torch.empty(qkv.shape[0], H * D, dtype=out_dtype, device=qkv.device)
        ops.attention(q, k, v, out)
        ops.context(qkv.device).wait()
        return out
    finally:
        os.environ.pop("H3S_SAGE_MIN_S", None)
        ops._ctx.clear()


def sample_rows(S: int, H: int, n: int | None, seed: int = 0):
    """All (head, token) pairs, or n of them spread over heads and positions (first and last rows included)."""
    if n is None or n >= S * H:
        return np.repeat(np.arange(H), S), np.tile(np.arange(S), H)
    rng = np.random.default_rng(seed)
    rh = rng.permutation(np.arange(n) % H)          # every head, when n >= H
    rs = rng.integers(0, S, n)
    rh[:2] = [0, H - 1]
    rs[:2] = [0, S - 1]
    return rh, rs


def attention_stats(qkv_cpu: torch.Tensor, got: torch.Tensor, H: int, D: int, sage: bool, rows=None, dt=None) -> dict:
    """The GPU output against float64 softmax of the same inputs and against the oracle's restatement of the same
    arithmetic (Sage or SDPA semantics) on the chosen rows: min row cosine and max-abs error of each."""
    S = qkv_cpu.shape[0]
    host = bits(qkv_cpu)
    if dt is None:
        dt = {torch.float16: oracle.F16, torch.bfloat16: oracle.BF16, torch.float32: oracle.F32}[qkv_cpu.dtype]
    st = 3 * H * D
    rh, rs = rows if rows is not None else sample_rows(S, H, None)
    exact = oracle.exact_rows(host, (host, H * D), (host, 2 * H * D), dt, S, H, D, st, rh, rs)
    g = got.float().cpu().numpy().reshape(S, H, D)[rs, rh, :]
    if sage:
        iq, ik, qs, ks, km, hv = oracle.sage_prepass(host, (host, H * D), (host, 2 * H * D), dt, S, H, D, st)
        same = half_bits_to_f32(oracle.sage_rows(iq, ik, hv, qs, ks, S, H, D, rh, rs))
    else:
        same = half_bits_to_f32(oracle.sdpa_rows(host, (host, H * D), (host, 2 * H * D), dt, S, H, D, st, rh, rs))
    return {"rows": int(len(rh)), "min_cos_vs_exact": float(oracle.row_cosines(g, exact).min()),
            "max_abs_vs_exact": float(np.max(np.abs(g - exact))),
            "min_cos_vs_same_semantics": float(oracle.row_cosines(g, same).min()),
            "max_abs_vs_same_semantics": float(np.max(np.abs(g - same)))}


def check_attention(qkv_cpu: torch.Tensor, got: torch.Tensor, H: int, D: int, sage: bool, rows=None, dt=None):
    """Compares the GPU output with the oracle on the chosen rows; returns (min cosine vs exact, max-abs vs exact)."""
    S = qkv_cpu.shape[0]
    host = bits(qkv_cpu)
    if dt is None:
        dt = {torch.float16: oracle.F16, torch.bfloat16: oracle.BF16, torch.float32: oracle.F32}[qkv_cpu.dtype]
    st = 3 * H * D
    rh, rs = rows if rows is not None else sample_rows(S, H, None)
    exact = oracle.exact_rows(host, (host, H * D), (host, 2 * H * D), dt, S, H, D, st, rh, rs)
    g = got.float().cpu().numpy().reshape(S, H, D)[rs, rh, :]
    cos = oracle.row_cosines(g, exact)
    maxabs = float(np.max(np.abs(g - exact)))
    assert cos.min() >= MIN_ROW_COSINE, f"min row cosine vs exact {cos.min():.6f}"
    assert maxabs <= MAX_ABS_VS_EXACT, f"max-abs vs exact {maxabs:.4g}"
    if sage:
        iq, ik, qs, ks, km, hv = oracle.sage_prepass(host, (host, H * D), (host, 2 * H * D), dt, S, H, D, st)
        same = half_bits_to_f32(oracle.sage_rows(iq, ik, hv, qs, ks, S, H, D, rh, rs))
    else:
        same = half_bits_to_f32(oracle.sdpa_rows(host, (host, H * D), (host, 2 * H * D), dt, S, H, D, st, rh, rs))
    cs = oracle.row_cosines(g, same)
    assert cs.min() >= MIN_ROW_COSINE_VS_SAME_SEMANTICS, f"min row cosine vs the same-semantics oracle {cs.min():.6f}"
    return float(cos.min()), maxabs


def gpu_prepass(qkv: torch.Tensor, H: int, D: int, stride: int | None = None, dt=native.F16):
    """h3s_sage_prepass on q, k inside qkv; returns (iq, ik, qs, ks, kmean) as numpy."""
    S = qkv.shape[0]
    st = stride if stride is not None else qkv.shape[1]
    nb = (S + 63) // 64
    iq = torch.empty(H, S, D, dtype=torch.int8, device=qkv.device)
    ik = torch.empty_like(iq)
    sc = torch.empty(2 * H * nb + H * D, dtype=torch.float32, device=qkv.device)
    ctx = ops.context(qkv.device)
    es = qkv.element_size()
    ctx.sage_prepass(qkv.data_ptr(), qkv.data_ptr() + H * D * es, dt, S, H, D, st, iq.data_ptr(), ik.data_ptr(),
                     sc.data_ptr())
    ctx.wait()
    s = sc.cpu().numpy()
    return (iq.cpu().numpy(), ik.cpu().numpy(), s[:H * nb].reshape(H, nb), s[H * nb:2 * H * nb].reshape(H, nb),
            s[2 * H * nb:])


__all__ = ["make_qkv", "bits", "run_attention", "check_attention", "attention_stats", "gpu_prepass", "sample_rows", "tok_rows_to_head_rows",
           "half_bits_to_f32", "MIN_ROW_COSINE", "MAX_ABS_VS_EXACT"]


def edge_qkv(S: int, H: int, D: int, dtype: torch.dtype, seed: int = 0) -> torch.Tensor:
    """q | k | v rows with the values a quantiser's absmax can mishandle: NaN (scattered, and a whole channel of one
    64-row block), +-inf, -0, subnormals, the largest finite values, and blocks of zeros; S need not be a multiple of 64."""
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(S, 3 * H * D, generator=g) * 2
    big = 65504.0 if dtype == torch.float16 else 3.0e38
    tiny = 6.0e-8 if dtype == torch.float16 else 1.0e-39
    n = S * 3 * H * D
    idx = torch.randperm(n, generator=g)
    flat = x.view(-1)
    flat[idx[: n // 200]] = float("nan")
    flat[idx[n // 200: n // 100]] = float("inf")
    flat[idx[n // 100: n // 70]] = -float("inf")
    flat[idx[n // 70: n // 50]] = -0.0
    flat[idx[n // 50: n // 40]] = big * torch.sign(torch.randn(n // 40 - n // 50, generator=g))
    flat[idx[n // 40: n // 30]] = tiny
    x[:64, 5] = float("nan")                       # one q channel all NaN in the first block
    x[64:128, H * D + 7] = float("nan")            # one k channel all NaN in the second block
    if S > 128:
        x[128:min(S, 192), :H * D] = 0.0           # a block of zeros (scale 0, codes 0)
    return x.to(dtype)
