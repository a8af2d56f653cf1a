"""h3s_rms_rope on the GPU through the C ABI against the oracle: the per-head RMS norm + rotary rotation the denoiser
runs on q and k right before the attention (kernels/h3sycl.cpp:1276-1376; engine/h3-core/src/dit.rs:347-348).

The kernel and the oracle follow the same operation order with every step rounded, so the results must be bit-exact:
all three element types, rotation widths that do and do not fall on 16-byte chunks, head sizes 64 to 128, rows inside
a qkv buffer, rows the shared-memory staging cannot take (unaligned), and the reference's refusals."""
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


def case(M, H, D, rot, dtype, cuda, offset=0, seed=0):
    g = torch.Generator().manual_seed(seed)
    stride = 3 * H * D + offset
    buf = (torch.randn(M * stride + offset, generator=g) * 3).to(dtype)
    w = (1 + 0.2 * torch.randn(D, generator=g)).float()
    ang = (torch.rand(M, rot // 2, generator=g) * 14 - 7)
    cs = torch.stack([torch.cos(ang), torch.sin(ang)], -1).float().contiguous()
    host = bits(buf)
    want = oracle.rms_rope(host[offset:], CODE[dtype], M, H, D, stride, w.numpy(), 1e-5, cs.numpy(), rot)
    dev = buf.to(cuda)
    ctx = ops.context(cuda)
    wd, csd = w.to(cuda), cs.to(cuda)
    ctx.rms_rope(dev.data_ptr() + offset * dev.element_size(), CODE[dtype], M, H, D, stride, wd.data_ptr(), 1e-5,
                 csd.data_ptr(), rot)
    ctx.wait()
    got = bits(dev)[offset:]
    return got, want


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16, torch.float32])
@pytest.mark.parametrize("D,rot", [(128, 128), (128, 96), (128, 0), (64, 64), (128, 120), (96, 30), (100, 20)])
def test_bit_exact(dtype, D, rot, cuda):
    for M in (1, 129, 300):
        got, want = case(M, 3, D, rot, dtype, cuda, seed=M + D + rot)
        assert np.array_equal(got, want), f"M={M}: {np.count_nonzero(got != want)} of {got.size} differ"


@pytest.mark.parametrize("dtype", [torch.float16, torch.float32])
def test_unaligned_rows_take_the_plain_kernel(dtype, cuda):
    got, want = case(77, 2, 128, 96, dtype, cuda, offset=1, seed=5)
    assert np.array_equal(got, want)


def test_through_rows_and_the_qkv_layout(cuda):
    """ops.rms_rope on q and k as the strided parts of a qkv buffer (dit.rs:345-348); v is left alone."""
    S, H, D, rot = 200, 4, 128, 96
    g = torch.Generator().manual_seed(9)
    qkv = torch.randn(S, 3 * H * D, generator=g).half()
    w = (1 + 0.1 * torch.randn(D, generator=g)).float()
    ang = torch.rand(S, rot // 2, generator=g) * 6
    cs = torch.stack([torch.cos(ang), torch.sin(ang)], -1).float().contiguous()
    host = bits(qkv).reshape(-1)
    after_q = oracle.rms_rope(host, native.F16, S, H, D, 3 * H * D, w.numpy(), 1e-5, cs.numpy(), rot)
    # k starts H*D elements into the buffer, rows at the same stride
    k_done = oracle.rms_rope(after_q[H * D:], native.F16, S, H, D, 3 * H * D, w.numpy(), 1e-5, cs.numpy(), rot)
    want = np.concatenate([after_q[:H * D], k_done]).reshape(S, 3 * H * D)
    dev = qkv.to(cuda)
    q, k, v = ops.Rows.qkv(dev, H, D)
    ops.rms_rope(q, w.to(cuda), 1e-5, cs.to(cuda), rot)
    ops.rms_rope(k, w.to(cuda), 1e-5, cs.to(cuda), rot)
    ops.context(cuda).wait()
    got = bits(dev)
    assert np.array_equal(got, want)
    assert np.array_equal(got[:, 2 * H * D:], bits(qkv)[:, 2 * H * D:])     # v untouched


def test_refusals_and_degenerate_sizes(cuda):
    ctx = ops.context(cuda)
    L = native.lib()
    assert L.h3s_rms_rope(ctx.handle, 0, native.F16, 0, 2, 128, 256, 0, 1e-5, 0, 128) == 0
    for rot in (3, 130, -2):
        assert L.h3s_rms_rope(ctx.handle, 0, native.F16, 4, 1, 128, 128, 0, 1e-5, 0, rot) == -1
        assert "rot_dim" in native.last_error()
    assert L.h3s_rms_rope(ctx.handle, 0, native.F16, 4, 2, 128, 128, 0, 1e-5, 0, 128) == -1
    assert "stride" in native.last_error()
    with pytest.raises(native.H3Error):
        x = torch.zeros(4, 128, dtype=torch.float16, device=cuda)
        ops.rms_rope(ops.Rows.packed(x, 1, 128), torch.ones(64, device=cuda), 1e-5, torch.zeros(4 * 128, device=cuda), 128)


@pytest.mark.skipif(not oracle.ref_available(), reason="oracle/_ref/libref.so is not built")
@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16, torch.float32])
@pytest.mark.parametrize("D,rot", [(128, 96), (128, 128), (64, 64), (100, 20)])
def test_vs_reference_source(dtype, D, rot, cuda):
    """The GPU kernel against h3s_rms_rope compiled from the reference's own source (its rsqrt correctly rounded)."""
    for M, offset in ((257, 0), (64, 3)):
        g = torch.Generator().manual_seed(M + D + rot)
        H = 3
        stride = 3 * H * D + offset
        buf = (torch.randn(M * stride + offset, generator=g) * 3).to(dtype)
        w = (1 + 0.2 * torch.randn(D, generator=g)).float()
        ang = torch.rand(M, rot // 2, generator=g) * 14 - 7
        cs = torch.stack([torch.cos(ang), torch.sin(ang)], -1).float().contiguous()
        want = oracle.ref_rms_rope(np.ascontiguousarray(bits(buf)[offset:]), CODE[dtype], M, H, D, stride, w.numpy(),
                                   1e-5, cs.numpy(), rot)
        dev = buf.to(cuda)
        ctx = ops.context(cuda)
        wd, csd = w.to(cuda), cs.to(cuda)
        ctx.rms_rope(dev.data_ptr() + offset * dev.element_size(), CODE[dtype], M, H, D, stride, wd.data_ptr(), 1e-5,
                     csd.data_ptr(), rot)
        ctx.wait()
        got = bits(dev)[offset:]
        assert np.array_equal(got, want), f"M={M}: {np.count_nonzero(got != want)} of {got.size} differ"
