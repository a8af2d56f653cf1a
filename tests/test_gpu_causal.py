"""h3s_attention_causal on the GPU through the C ABI: the text encoder's causal attention with grouped heads
(kernels/h3sycl.cpp:870-898; engine/h3-core/src/te.rs:340-346), against the oracle's fp32 restatement of the reference
loop and against float64 causal softmax.

Tolerances (the same bar as the other attention paths): per-row cosine >= 0.9999 against the oracle (same arithmetic
up to the order of the dot-product sums and the exponential's last bits), per-row cosine >= 0.999 and max-abs <= 0.05
against float64 (f16 and bf16 outputs round at the end)."""
import numpy as np
import pytest
import torch

import oracle
from sycl_minimax_h3_b200 import native, ops

pytestmark = pytest.mark.gpu

CODE = {torch.float16: native.F16, torch.bfloat16: native.BF16, torch.float32: native.F32}


def bits(t: torch.Tensor) -> np.ndarray:
    c = t.cpu().contiguous()
    return c.view(torch.int16).numpy().view(np.uint16) if c.element_size() == 2 else c.numpy()


def f32(t: torch.Tensor) -> np.ndarray:
    return t.float().cpu().numpy()


def exact(q, k, v, L, Hq, Hkv, D):
    out = np.zeros((L, Hq, D))
    grp = Hq // Hkv
    qf = q.reshape(L, Hq, D).astype(np.float64)
    kf = k.reshape(L, Hkv, D).astype(np.float64)
    vf = v.reshape(L, Hkv, D).astype(np.float64)
    mask = np.tril(np.ones((L, L), bool))
    for h in range(Hq):
        s = np.where(mask, qf[:, h] @ kf[:, h // grp].T / np.sqrt(D), -np.inf)
        p = np.exp(s - s.max(1, keepdims=True))
        out[:, h] = (p / p.sum(1, keepdims=True)) @ vf[:, h // grp]
    return out.reshape(L, Hq * D)


def run(L, Hq, Hkv, D, dtype, cuda, seed=0):
    g = torch.Generator().manual_seed(seed)
    q = torch.randn(L, Hq * D, generator=g).to(dtype)
    k = (torch.randn(L, Hkv * D, generator=g) * 1.5).to(dtype)
    v = torch.randn(L, Hkv * D, generator=g).to(dtype)
    out = torch.empty(L, Hq * D, dtype=dtype, device=cuda)
    qd, kd, vd = q.to(cuda), k.to(cuda), v.to(cuda)
    ops.attention_causal(ops.Rows.packed(qd, Hq, D), ops.Rows.packed(kd, Hkv, D), ops.Rows.packed(vd, Hkv, D), out)
    ops.context(cuda).wait()
    want = oracle.attention_causal(bits(q), bits(k), bits(v), CODE[dtype], L, Hq, Hkv, D, Hq * D, Hkv * D)
    want = torch.from_numpy(want.view(np.int16)).view(dtype).float().numpy() if dtype != torch.float32 else want
    return f32(out), want, exact(f32(q), f32(k), f32(v), L, Hq, Hkv, D)


def cos_rows(a, b, D):
    a = a.reshape(-1, D).astype(np.float64)
    b = b.reshape(-1, D).astype(np.float64)
    return (a * b).sum(1) / np.maximum(np.linalg.norm(a, axis=1) * np.linalg.norm(b, axis=1), 1e-300)


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16, torch.float32])
@pytest.mark.parametrize("L,Hq,Hkv,D", [(1, 4, 2, 128), (5, 4, 4, 128), (77, 8, 2, 128), (300, 4, 1, 128),
                                        (130, 2, 2, 64), (61, 4, 2, 96), (40, 2, 1, 256)])
def test_against_oracle_and_float64(dtype, L, Hq, Hkv, D, cuda):
    got, want, ex = run(L, Hq, Hkv, D, dtype, cuda, seed=L + D + Hq)
    assert cos_rows(got, want, D).min() >= 0.9999
    assert cos_rows(got, ex, D).min() >= 0.999
    assert np.max(np.abs(got - ex)) <= 0.05


def test_first_query_sees_only_itself(cuda):
    """Row 0 attends to key 0 alone: its output is v_0 of its key/value head, exactly (weight 1)."""
    L, Hq, Hkv, D = 16, 4, 2, 128
    got, _, _ = run(L, Hq, Hkv, D, torch.float32, cuda, seed=3)
    g = torch.Generator().manual_seed(3)
    torch.randn(L, Hq * D, generator=g)
    torch.randn(L, Hkv * D, generator=g)
    v = torch.randn(L, Hkv * D, generator=g).numpy()
    for h in range(Hq):
        np.testing.assert_allclose(got[0, h * D:(h + 1) * D], v[0, (h // 2) * D:(h // 2 + 1) * D], rtol=1e-6)


def test_refusals_and_degenerate_sizes(cuda):
    ctx = ops.context(cuda)
    L_ = native.lib()
    assert L_.h3s_attention_causal(ctx.handle, 0, 0, 0, native.F16, 0, 4, 2, 128, 512, 256, 0) == 0
    assert L_.h3s_attention_causal(ctx.handle, 0, 0, 0, native.F16, 4, 4, 2, 512, 2048, 1024, 0) == -1
    assert "D <= 256" in native.last_error()
    assert L_.h3s_attention_causal(ctx.handle, 0, 0, 0, native.F16, 4, 3, 2, 128, 384, 256, 0) == -1
    assert L_.h3s_attention_causal(ctx.handle, 0, 0, 0, native.F16, 4, 4, 2, 128, 100, 256, 0) == -1
    assert "stride" in native.last_error()
