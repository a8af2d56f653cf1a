"""Head size 64 on the GPU through the C ABI against the oracle: the reference plugin takes D in {64, 128}
(kernels/sage.cpp:33) and the fp16 path serves the VAE's 64-wide heads (kernels/h3sycl.cpp:1581-1674).

The Sage kernel runs 128 wide and reads a 64-wide head as zeros in features 64-127 (TMA fills outside the tensor with
zeros); the fp16 SDPA runs a 64-wide instantiation (K = 64 Q.K^T, N = 64 P.V, 64 TMEM columns of O per tile). Both
are held to the same tolerances as D = 128 (per-row cosine >= 0.999 and max-abs <= 0.05 against float64 softmax;
>= 0.9999 against the oracle's restatement of the same arithmetic), and the pre-pass is bit-exact."""
import ctypes

import numpy as np
import pytest
import torch

import oracle
from _util import check_attention, gpu_prepass, half_bits_to_f32, run_attention
from sycl_minimax_h3_b200 import native, ops
from sycl_minimax_h3_b200.workloads import bits, make_qkv

pytestmark = pytest.mark.gpu

D = 64


@pytest.mark.parametrize("S", [1, 65, 300, 1000])
def test_sage_path_d64(S, cuda):
    H = 2
    qkv = make_qkv(S, H, D, seed=640 + S)
    out = run_attention(qkv.to(cuda), H, D, min_s=0)
    check_attention(qkv, out, H, D, sage=True)


@pytest.mark.parametrize("S", [1, 200, 777])
def test_sdpa_path_d64(S, cuda):
    H = 3
    qkv = make_qkv(S, H, D, seed=650 + S)
    out = run_attention(qkv.to(cuda), H, D, min_s=1 << 30)
    check_attention(qkv, out, H, D, sage=False)


@pytest.mark.parametrize("dtype,out_dtype", [(torch.bfloat16, torch.bfloat16), (torch.float32, torch.float32),
                                             (torch.float16, torch.float32), (torch.float16, torch.bfloat16)])
@pytest.mark.parametrize("min_s", [0, 1 << 30])
def test_element_types_d64(dtype, out_dtype, min_s, cuda):
    """Every input and output type on both paths; the output rounded through half first (kernels/h3sycl.cpp:1769-1771)."""
    S, H = 333, 2
    qkv = make_qkv(S, H, D, seed=67, dtype=dtype)
    out = run_attention(qkv.to(cuda), H, D, out_dtype=out_dtype, min_s=min_s)
    assert out.dtype == out_dtype
    check_attention(qkv, out, H, D, sage=min_s == 0)
    o = out.float()
    assert torch.equal(o, o.half().float())


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_sage_path_d64_other_types(dtype, cuda):
    S, H = 257, 2
    qkv = make_qkv(S, H, D, seed=66, dtype=dtype)
    out = run_attention(qkv.to(cuda), H, D, min_s=0)
    check_attention(qkv, out, H, D, sage=True)


def test_prepass_bit_exact_d64(cuda):
    S, H = 300, 3
    qkv = make_qkv(S, H, D, seed=67)
    got = gpu_prepass(qkv.to(cuda), H, D)
    host = bits(qkv)
    want = oracle.sage_prepass(host, (host, H * D), (host, 2 * H * D), oracle.F16, S, H, D, 3 * H * D)[:5]
    for g, w, name in zip(got, want, ("iq", "ik", "qs", "ks", "kmean")):
        assert np.array_equal(np.asarray(g).reshape(-1).view(np.uint8), np.asarray(w).reshape(-1).view(np.uint8)), name


def test_plugin_abi_direct_d64(cuda):
    """h3sage_attention with the plugin's layouts at D = 64: int8 q, k [H, S, 64], half v and out [H, S, 64]."""
    S, H = 333, 2
    qkv = make_qkv(S, H, D, seed=68)
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


def test_attention_batch_d64(cuda):
    """The VAE's shape class: B sequences of 64-wide heads in one fp16 call (kernels/h3sycl.cpp:1800-1816)."""
    B, S, H = 3, 190, 2
    qkv = torch.cat([make_qkv(S, H, D, seed=69 + b) for b in range(B)])
    g = qkv.to(cuda)
    q, k, v = ops.Rows.qkv(g, H, D)
    out = torch.empty(B * S, H * D, dtype=torch.float16, device=cuda)
    ops._ctx.clear()
    ops.attention_batch(q, k, v, B, out)
    ops.context(cuda).wait()
    for b in range(B):
        check_attention(qkv[b * S:(b + 1) * S], out[b * S:(b + 1) * S], H, D, sage=False)
