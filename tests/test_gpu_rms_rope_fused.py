"""The block's RMS norm + RoPE fused into the Sage pre-pass (h3s_sage_prepass_rope) and the block's three calls in one
(h3s_attention_rms_rope), through the C ABI: bit for bit what h3s_rms_rope on q, h3s_rms_rope on k and then
h3s_sage_prepass / h3s_attention make of the same rows (engine/h3-core/src/dit.rs:347-350), and the pre-pass against
the oracle's restatement of kernels/h3sycl.cpp:1276-1376 followed by :1733-1761. All three element types, both head
sizes, rotation widths with and without 16-byte chunks, odd strides (the unfused fallback), edge sequence lengths, and
configs[3] at full size."""
import numpy as np
import pytest
import torch

import oracle
from _util import bits as tbits
from sycl_minimax_h3_b200 import native, ops
from sycl_minimax_h3_b200.workloads import make_qkv

pytestmark = pytest.mark.gpu

CODE = {torch.float16: native.F16, torch.bfloat16: native.BF16, torch.float32: native.F32}


def _inputs(S, H, D, rot, dtype, cuda, extra=0, seed=0):
    g = torch.Generator().manual_seed(seed)
    st = 3 * H * D + extra
    buf = torch.zeros(S, st, dtype=dtype)
    buf[:, :3 * H * D] = make_qkv(S, H, D, seed=seed, dtype=dtype)
    wq = (1 + 0.2 * torch.randn(D, generator=g)).float()
    wk = (1 + 0.2 * torch.randn(D, generator=g)).float()
    ang = torch.rand(S, max(rot // 2, 1), generator=g) * 14 - 7
    cs = torch.stack([torch.cos(ang), torch.sin(ang)], -1).float().contiguous()
    return buf, st, wq.to(cuda), wk.to(cuda), cs.to(cuda)


def _prepass_buffers(S, H, D, cuda):
    nb = (S + 63) // 64
    iq = torch.empty(H, S, D, dtype=torch.int8, device=cuda)
    ik = torch.empty_like(iq)
    sc = torch.empty(2 * H * nb + H * D, dtype=torch.float32, device=cuda)
    return iq, ik, sc


def _both(buf, st, S, H, D, rot, dt, wq, wk, cs, cuda):
    """(fused results, separate-call results): rotated qkv rows, iq, ik, scales."""
    ctx = ops.context(cuda)
    es = buf.element_size()
    a = buf.to(cuda).clone()        # two copies, also when buf already lives on the GPU
    b = buf.to(cuda).clone()
    fa = _prepass_buffers(S, H, D, cuda)
    fb = _prepass_buffers(S, H, D, cuda)
    ctx.sage_prepass_rope(a.data_ptr(), a.data_ptr() + H * D * es, dt, S, H, D, st, wq.data_ptr(), wk.data_ptr(), 1e-5,
                          cs.data_ptr(), rot, *(t.data_ptr() for t in fa))
    ctx.rms_rope(b.data_ptr(), dt, S, H, D, st, wq.data_ptr(), 1e-5, cs.data_ptr(), rot)
    ctx.rms_rope(b.data_ptr() + H * D * es, dt, S, H, D, st, wk.data_ptr(), 1e-5, cs.data_ptr(), rot)
    ctx.sage_prepass(b.data_ptr(), b.data_ptr() + H * D * es, dt, S, H, D, st, *(t.data_ptr() for t in fb))
    ctx.wait()
    return (a, *fa), (b, *fb)


def _same(x: torch.Tensor, y: torch.Tensor) -> bool:
    return torch.equal(x.contiguous().view(torch.uint8), y.contiguous().view(torch.uint8))


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16, torch.float32])
@pytest.mark.parametrize("D,rot", [(128, 96), (128, 128), (128, 0), (64, 64), (128, 30), (64, 20)])
def test_prepass_rope_equals_separate_calls(dtype, D, rot, cuda):
    for S, H, extra in ((1, 2, 0), (65, 2, 0), (200, 3, 0), (130, 2, 3)):   # extra: an odd stride (unfused fallback)
        buf, st, wq, wk, cs = _inputs(S, H, D, rot, dtype, cuda, extra=extra, seed=S + D + rot)
        fused, sep = _both(buf, st, S, H, D, rot, CODE[dtype], wq, wk, cs, cuda)
        for name, x, y in zip(("q/k rows", "iq", "ik", "scales"), fused, sep):
            assert _same(x, y), f"{name} differ (S={S}, H={H}, stride {st})"


def test_prepass_rope_vs_oracle(cuda):
    """Against the CPU restatement: rms_rope of q and k, then the pre-pass of the rotated rows."""
    S, H, D, rot = 300, 2, 128, 96
    buf, st, wq, wk, cs = _inputs(S, H, D, rot, torch.float16, cuda, seed=11)
    fused, _ = _both(buf, st, S, H, D, rot, native.F16, wq, wk, cs, cuda)
    host = tbits(buf)
    rq = oracle.rms_rope(host, oracle.F16, S, H, D, st, wq.cpu().numpy(), 1e-5, cs.cpu().numpy(), rot).ravel()
    # k: the same rows from element H*D on
    rk = oracle.rms_rope(np.ascontiguousarray(rq[H * D:]), oracle.F16, S, H, D, st, wk.cpu().numpy(), 1e-5,
                         cs.cpu().numpy(), rot)
    rows = np.concatenate([rq[:H * D], rk]).reshape(S, st)
    assert np.array_equal(tbits(fused[0].cpu()), rows), "rotated rows"
    iq, ik, qs, ks, km, _ = oracle.sage_prepass(rows, (rows, H * D), (rows, 2 * H * D), oracle.F16, S, H, D, st)
    nb = (S + 63) // 64
    sc = fused[3].cpu().numpy()
    assert np.array_equal(fused[1].cpu().numpy(), iq) and np.array_equal(fused[2].cpu().numpy(), ik)
    assert np.array_equal(sc.view(np.uint32), np.concatenate([qs.ravel(), ks.ravel(), km]).view(np.uint32))
    assert sc.size == 2 * H * nb + H * D


def test_prepass_rope_c3_full(cuda):
    """configs[3] (32 heads x 47,232 tokens, fp16, rot_dim 96): the fused pre-pass equals the separate calls."""
    S, H, D, rot = 47232, 32, 128, 96
    g = torch.Generator(device=cuda)
    g.manual_seed(5)
    buf = make_qkv(S, H, D, seed=S, device=cuda)
    wq = (1 + 0.1 * torch.randn(D, generator=g, device=cuda)).float()
    wk = (1 + 0.1 * torch.randn(D, generator=g, device=cuda)).float()
    ang = torch.rand(S, rot // 2, generator=g, device=cuda) * 6.28
    cs = torch.stack([torch.cos(ang), torch.sin(ang)], -1).float().contiguous()
    fused, sep = _both(buf, 3 * H * D, S, H, D, rot, native.F16, wq, wk, cs, cuda)
    for name, x, y in zip(("q/k rows", "iq", "ik", "scales"), fused, sep):
        assert _same(x, y), name


@pytest.mark.parametrize("min_s", [0, 1 << 30])          # the Sage path, the fp16 SDPA path
@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_attention_rms_rope_equals_three_calls(min_s, dtype, cuda, monkeypatch):
    monkeypatch.setenv("H3S_SAGE_MIN_S", str(min_s))
    ops._ctx.clear()
    try:
        S, H, D, rot = 333, 2, 128, 96
        buf, st, wq, wk, cs = _inputs(S, H, D, rot, dtype, cuda, seed=7)
        a, b = buf.to(cuda).clone(), buf.to(cuda).clone()
        oa = torch.empty(S, H * D, dtype=dtype, device=cuda)
        ob = torch.empty_like(oa)
        qa, ka, va = ops.Rows.qkv(a, H, D)
        ops.attention_rms_rope(qa, ka, va, oa, wq, wk, 1e-5, cs, rot)
        qb, kb, vb = ops.Rows.qkv(b, H, D)
        ops.rms_rope(qb, wq, 1e-5, cs, rot)
        ops.rms_rope(kb, wk, 1e-5, cs, rot)
        ops.attention(qb, kb, vb, ob)
        ops.context(cuda).wait()
        assert _same(a, b), "q, k are left rotated in place as the separate calls leave them"
        assert _same(oa, ob), "the output"
    finally:
        ops._ctx.clear()


def test_refusals(cuda):
    ctx = ops.context(cuda)
    L = native.lib()
    x = torch.zeros(4, 3 * 128, dtype=torch.float16, device=cuda)
    w = torch.ones(128, device=cuda)
    for rot in (3, 130):
        assert L.h3s_attention_rms_rope(ctx.handle, x.data_ptr(), x.data_ptr(), x.data_ptr(), native.F16, 4, 1, 128,
                                        384, x.data_ptr(), native.F16, w.data_ptr(), w.data_ptr(), 1e-5, w.data_ptr(),
                                        rot) == -1
        assert "rot_dim" in native.last_error()
    assert L.h3s_sage_prepass_rope(ctx.handle, x.data_ptr(), x.data_ptr(), native.F16, 4, 1, 128, 100, w.data_ptr(),
                                   w.data_ptr(), 1e-5, w.data_ptr(), 96, x.data_ptr(), x.data_ptr(), x.data_ptr()) == -1
    assert "stride" in native.last_error()
