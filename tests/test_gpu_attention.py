"""Attention on the GPU through the C ABI against the oracle: the int8 Sage path and the fp16 SDPA path, edge sizes,
element types, the batch entry point, the plugin ABI called directly, and error behaviour.

Tolerance: per-row cosine >= 0.999 against float64 softmax of the same inputs, max-abs error
measured and bounded by 0.05; and per-row cosine >= 0.9999 against the oracle's restatement of the same arithmetic."""
import ctypes

import numpy as np
import pytest
import torch

import oracle
from _util import check_attention, half_bits_to_f32, run_attention
from sycl_minimax_h3_b200 import native, ops
from sycl_minimax_h3_b200.workloads import bits, make_qkv

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("S", [1, 63, 64, 65, 127, 128, 129, 300, 1000])
def test_sage_path_sizes(S, cuda):
    H, D = 2, 128
    qkv = make_qkv(S, H, D, seed=S)
    out = run_attention(qkv.to(cuda), H, D, min_s=0)
    check_attention(qkv, out, H, D, sage=True)


@pytest.mark.parametrize("S", [1, 65, 200, 777])
def test_sdpa_path_sizes(S, cuda):
    H, D = 2, 128
    qkv = make_qkv(S, H, D, seed=100 + S)
    out = run_attention(qkv.to(cuda), H, D, min_s=1 << 30)
    check_attention(qkv, out, H, D, sage=False)


def test_c0_both_paths(cuda):
    """8 heads x 2,048 tokens, forced Sage and fp16 SDPA."""
    S, H, D = 2048, 8, 128
    qkv = make_qkv(S, H, D, seed=0)
    rows = (np.repeat(np.arange(H), 64), np.tile(np.linspace(0, S - 1, 64).astype(np.int64), H))
    for min_s, sage in ((0, True), (1 << 30, False)):
        out = run_attention(qkv.to(cuda), H, D, min_s=min_s)
        check_attention(qkv, out, H, D, sage=sage, rows=rows)


def test_default_threshold_picks_sdpa_below_8192(cuda):
    S, H, D = 500, 2, 128
    qkv = make_qkv(S, H, D, seed=3)
    out = run_attention(qkv.to(cuda), H, D, min_s=None)
    host = bits(qkv)
    want = oracle.attention(host, (host, H * D), (host, 2 * H * D), oracle.F16, S, H, D, 3 * H * D, oracle.F16,
                            sage_min_s=8192)
    g = out.float().cpu().numpy()
    assert oracle.row_cosines(g.reshape(-1, D), half_bits_to_f32(want).reshape(-1, D)).min() >= 0.9999


@pytest.mark.parametrize("dtype,out_dtype", [(torch.bfloat16, torch.bfloat16), (torch.float32, torch.float32),
                                             (torch.float16, torch.float32), (torch.float16, torch.bfloat16)])
@pytest.mark.parametrize("min_s", [0, 1 << 30])
def test_element_types(dtype, out_dtype, min_s, cuda):
    S, H, D = 260, 2, 128
    qkv = make_qkv(S, H, D, seed=21, dtype=dtype)
    out = run_attention(qkv.to(cuda), H, D, out_dtype=out_dtype, min_s=min_s)
    assert out.dtype == out_dtype
    check_attention(qkv, out, H, D, sage=min_s == 0)
    # the output went through half (kernels/h3sycl.cpp:1769-1771)
    o = out.float()
    assert torch.equal(o, o.half().float())


def test_packed_rows_and_unaligned_stride(cuda):
    S, H, D = 190, 2, 128
    for st in (H * D, 3 * H * D + 4):
        x = torch.zeros(S, st, dtype=torch.float16)
        full = make_qkv(S, H, D, seed=st)
        for min_s in (0, 1 << 30):
            # q, k, v in three separate buffers of row stride st
            parts = []
            for i in range(3):
                t = x.clone()
                t[:, :H * D] = full[:, i * H * D:(i + 1) * H * D]
                parts.append(t.to(cuda))
            out = torch.empty(S, H * D, dtype=torch.float16, device=cuda)
            import os

            os.environ["H3S_SAGE_MIN_S"] = str(min_s)
            ops._ctx.clear()
            rows = [ops.Rows(p, 0, st, S, H, D) for p in parts]
            ops.attention(*rows, out)
            ops.context(cuda).wait()
            os.environ.pop("H3S_SAGE_MIN_S")
            ops._ctx.clear()
            check_attention(full, out, H, D, sage=min_s == 0)


def test_attention_batch(cuda):
    B, S, H, D = 3, 150, 2, 128
    qkv = torch.cat([make_qkv(S, H, D, seed=40 + b) for b in range(B)])
    q, k, v = ops.Rows.qkv(qkv.to(cuda), H, D)
    out = torch.empty(B * S, H * D, dtype=torch.float16, device=cuda)
    ops._ctx.clear()
    ops.attention_batch(q, k, v, B, out)
    ops.context(cuda).wait()
    for b in range(B):
        check_attention(qkv[b * S:(b + 1) * S], out[b * S:(b + 1) * S], H, D, sage=False)


def test_plugin_abi_direct(cuda):
    """h3sage_attention with the reference plugin's layouts: int8 q, k and half v, out [H, S, D] (kernels/sage.cpp:31)."""
    S, H, D = 333, 2, 128
    qkv = make_qkv(S, H, D, seed=8)
    host = bits(qkv)
    iq, ik, qs, ks, km, hv = oracle.sage_prepass(host, (host, H * D), (host, 2 * H * D), oracle.F16, S, H, D, 3 * H * D)
    d = {n: torch.from_numpy(np.ascontiguousarray(a)).to(cuda) for n, a in
         (("iq", iq), ("ik", ik), ("qs", qs), ("ks", ks), ("hv", hv.view(np.int16)))}
    out = torch.empty(H, S, D, dtype=torch.float16, device=cuda)
    sage = native.sage_lib()
    st = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    rc = sage.h3sage_attention(ctypes.byref(st), d["iq"].data_ptr(), d["ik"].data_ptr(), d["hv"].data_ptr(),
                               out.data_ptr(), d["qs"].data_ptr(), d["ks"].data_ptr(), 64, S, H, D, 1.0 / D ** 0.5)
    assert rc == 0, sage.h3sage_error()
    assert sage.h3sage_check(ctypes.byref(st)) == 0, sage.h3sage_error()
    rh, rs = np.repeat(np.arange(H), S), np.tile(np.arange(S), H)
    want = half_bits_to_f32(oracle.sage_rows(iq, ik, hv, qs, ks, S, H, D, rh, rs))
    got = out.float().cpu().numpy().reshape(H * S, D)
    assert oracle.row_cosines(got, want).min() >= 0.9999
    # the plugin's refusals (kernels/sage.cpp:33-35)
    assert sage.h3sage_attention(ctypes.byref(st), 0, 0, 0, 0, 0, 0, 64, S, H, 96, 0.1) == -1
    assert b"head size" in sage.h3sage_error()
    assert sage.h3sage_attention(ctypes.byref(st), 0, 0, 0, 0, 0, 0, 32, S, H, D, 0.1) == -1
    assert b"multiple of 64" in sage.h3sage_error()
    assert sage.h3sage_attention(ctypes.byref(st), 0, 0, 0, 0, 0, 0, 64, 1 << 30, H, D, 0.1) == -1


def test_plugin_block_128(cuda):
    """A scale block of 128 rows (any multiple of 64 is accepted, kernels/sage.cpp:34)."""
    S, H, D = 300, 1, 128
    qkv = make_qkv(S, H, D, seed=31)
    host = bits(qkv)
    # quantise with 128-row blocks: two 64-row blocks' data under one scale, restated here
    qf = half_bits_to_f32(np.ascontiguousarray(host[:, :D]))
    kf = half_bits_to_f32(np.ascontiguousarray(host[:, D:2 * D]))
    vf = np.ascontiguousarray(host[:, 2 * D:3 * D])
    km = oracle.kmean((host, D), oracle.F16, S, H, D, 3 * D)

    def q128(x, mean):
        nb = (S + 127) // 128
        out = np.zeros((1, S, D), np.int8)
        sc = np.zeros((1, nb), np.float32)
        for b in range(nb):
            y = (x[b * 128:(b + 1) * 128] - mean).astype(np.float32)
            m = np.float32(np.abs(y).max())
            inv = np.float32(127) / m
            sc[0, b] = m / np.float32(127)
            t = (y * inv).astype(np.float32)
            r = np.trunc(t) + np.where(np.abs(t - np.trunc(t)) >= 0.5, np.sign(t), 0)
            out[0, b * 128:b * 128 + y.shape[0]] = np.clip(r, -127, 127)
        return out, sc

    iq, qs = q128(qf, np.float32(0))
    ik, ks = q128(kf, km)
    d = [torch.from_numpy(a).to(cuda) for a in (iq, ik, qs, ks, vf.view(np.int16))]
    out = torch.empty(1, S, D, dtype=torch.float16, device=cuda)
    sage = native.sage_lib()
    st = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    assert sage.h3sage_attention(ctypes.byref(st), d[0].data_ptr(), d[1].data_ptr(), d[4].data_ptr(), out.data_ptr(),
                                 d[2].data_ptr(), d[3].data_ptr(), 128, S, H, D, 1.0 / D ** 0.5) == 0
    assert sage.h3sage_check(ctypes.byref(st)) == 0
    # reference: float64 softmax over the dequantised int8 values
    qd = iq[0].astype(np.float64) * np.repeat(qs[0], 128)[:S, None]
    kd = ik[0].astype(np.float64) * np.repeat(ks[0], 128)[:S, None]
    s = qd @ kd.T / np.sqrt(D)
    p = np.exp(s - s.max(1, keepdims=True))
    want = (p / p.sum(1, keepdims=True)) @ vf.view(np.float16).astype(np.float64)
    got = out[0].float().cpu().numpy()
    assert oracle.row_cosines(got, want).min() >= 0.9999


def test_error_behaviour(cuda):
    ctx = ops.context(cuda)
    L = native.lib()
    # degenerate sizes: nothing to do (kernels/h3sycl.cpp:1782)
    assert L.h3s_attention(ctx.handle, 0, 0, 0, native.F16, 0, 2, 128, 256, 0, native.F16) == 0
    assert L.h3s_attention(ctx.handle, 0, 0, 0, native.F16, 10, 2, 128, 255, 0, native.F16) == -1
    assert "stride" in native.last_error()
    x = torch.zeros(10, 512, dtype=torch.float16, device=cuda)
    # heads wider than the kernel's 128 features (a stated narrowing: the reference's fused path takes any D)
    assert L.h3s_attention(ctx.handle, x.data_ptr(), x.data_ptr(), x.data_ptr(), native.F16, 10, 1, 160, 512,
                           x.data_ptr(), native.F16) == -1
    assert "head size" in native.last_error()
    assert L.h3s_attention(ctx.handle, x.data_ptr(), x.data_ptr(), x.data_ptr(), 7, 10, 1, 128, 256, x.data_ptr(),
                           native.F16) == -1
    # the allocation cap is a refusal, not an allocation (kernels/h3sycl.h:43-52)
    assert L.h3s_alloc(ctx.handle, ctx.mem_cap() + 1) is None
    assert "cap" in native.last_error()
    p = ctx.alloc(1 << 20)
    assert ctx.mem_used() >= 1 << 20
    ctx.free(p)


def test_wait_limit_reports_and_recovers(cuda):
    """A kernel wait that runs out (an mbarrier nothing arrives at) makes h3s_wait fail with a message; the context
    stays usable for the next call."""
    ctx = native.Context.open_gpu(0)
    try:
        ctx.selftest_wait_timeout(2_000_000)      # 2 ms
        with pytest.raises(native.H3Error, match="gave up"):
            ctx.wait()
        ctx.wait()                                 # the error word was cleared
        S, H, D = 100, 1, 128
        qkv = make_qkv(S, H, D, seed=1).to(cuda)
        out = torch.empty(S, H * D, dtype=torch.float16, device=cuda)
        torch.cuda.synchronize()
        ctx.attention(qkv.data_ptr(), qkv.data_ptr() + H * D * 2, qkv.data_ptr() + 2 * H * D * 2, native.F16, S, H, D,
                      3 * H * D, out.data_ptr(), native.F16)
        ctx.wait()
        check_attention(qkv.cpu(), out, H, D, sage=False)
    finally:
        ctx.close()


def test_context_memory_and_copies(cuda):
    ctx = native.Context.open_gpu(0)
    try:
        assert "B200" in ctx.device_name or ctx.device_name
        n = 1 << 16
        a = np.arange(n, dtype=np.uint8)
        p = ctx.alloc(n)
        ctx.write(p, a.ctypes.data, n)
        q = ctx.alloc(n)
        L = native.lib()
        assert L.h3s_copy(ctx.handle, q, p, n) == 0
        b = np.zeros(n, np.uint8)
        ctx.read(b.ctypes.data, q, n)
        assert np.array_equal(a, b)
        h = L.h3s_alloc_host(ctx.handle, n)
        ctypes.memmove(h, a.ctypes.data, n)
        assert L.h3s_upload(ctx.handle, p, h, n) == 0
        assert L.h3s_upload_wait(ctx.handle) == 0
        assert L.h3s_upload(ctx.handle, p, a.ctypes.data, n) == -1     # pageable source: refused
        L.h3s_free_host(ctx.handle, h)
        ctx.free(p)
        ctx.free(q)
        info = native.gpu_info(0)
        assert info["mem_bytes"] > 0 and ":" in info["pci"]
    finally:
        ctx.close()


@pytest.mark.parametrize("D", [8, 12, 32, 48, 80, 96, 100, 120])
@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_other_head_sizes(D, dtype, cuda):
    """Head sizes other than 64 and 128 (kernels/h3sycl.cpp:1464-1573 takes any D; the Sage plugin only 64 and 128,
    kernels/sage.cpp:33, so these run on the fp16 SDPA at every length): heads whose rows are not 16-byte multiples go
    through the padded half copy, the others are read in place; the output's last chunk of features is partial."""
    for S, min_s in ((300, None), (200, 0)):          # the default threshold, and a forced Sage request that falls back
        H = 3
        qkv = make_qkv(S, H, D, seed=S + D, dtype=dtype)
        out = run_attention(qkv.to(cuda), H, D, min_s=min_s)
        check_attention(qkv, out, H, D, sage=False)
