"""The Sage pre-pass on the GPU (K channel mean, int8 Q / K-mean quantiser) bit for bit against the oracle's
restatement of kernels/h3sycl.cpp:1733-1761, through h3s_sage_prepass of the C ABI, and against the reference's own
pre-pass compiled from its source (oracle/_ref/libref.so) at configs[0], [2] and [3]."""
import numpy as np
import pytest
import torch

import oracle
from _util import edge_qkv, gpu_prepass
from sycl_minimax_h3_b200 import native
from sycl_minimax_h3_b200.workloads import bits, make_qkv

pytestmark = pytest.mark.gpu

DT = {torch.float16: native.F16, torch.bfloat16: native.BF16, torch.float32: native.F32}


def check(qkv_cpu: torch.Tensor, H: int, D: int, stride: int, cuda):
    S = qkv_cpu.shape[0]
    dt = DT[qkv_cpu.dtype]
    got = gpu_prepass(qkv_cpu.to(cuda), H, D, stride=stride, dt=dt)
    host = bits(qkv_cpu)
    want = oracle.sage_prepass(host, (host, H * D), (host, 2 * H * D), dt, S, H, D, stride)[:5]
    for name, g, w in zip(("iq", "ik", "qs", "ks", "kmean"), got, want):
        g, w = np.asarray(g), np.asarray(w)
        if g.dtype == np.float32:
            # bit for bit, except that any NaN equals any NaN: NaN's bits are the hardware's (x86 keeps an operand's
            # payload and makes inf - inf negative; the GPU returns one canonical NaN), not the algorithm's
            both_nan = np.isnan(g) & np.isnan(w)
            bad = (g.view(np.uint32) != w.view(np.uint32)) & ~both_nan
            assert not bad.any(), f"{name} differs at {np.flatnonzero(bad)[:5]} (S={S}, H={H})"
        else:
            assert np.array_equal(g.view(np.uint8), w.view(np.uint8)), f"{name} differs (S={S}, H={H})"


@pytest.mark.parametrize("S", [1, 63, 64, 65, 127, 200, 1000])
def test_prepass_bit_exact_f16(S, cuda):
    H, D = 2, 128
    check(make_qkv(S, H, D, seed=S), H, D, 3 * H * D, cuda)


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_prepass_bit_exact_other_types(dtype, cuda):
    H, D, S = 3, 128, 300
    check(make_qkv(S, H, D, seed=5, dtype=dtype), H, D, 3 * H * D, cuda)


@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("D", [64, 128])
def test_prepass_edge_values(dtype, D, cuda):
    """NaN, +-inf, -0, subnormals, the largest finite values, an all-NaN channel in a block, zero blocks and a partial
    last block: the GPU's absmax (taken at each channel's extremes) and codes have the oracle's bits."""
    S, H = 200, 2
    check(edge_qkv(S, H, D, dtype, seed=D), H, D, 3 * H * D, cuda)


def test_prepass_unaligned_stride(cuda):
    """A row stride TMA cannot take (not a multiple of 16 bytes): the plain-load kernels, same bits."""
    S, H, D = 150, 2, 128
    st = 3 * H * D + 3
    x = torch.zeros(S, st, dtype=torch.float16)
    x[:, :3 * H * D] = make_qkv(S, H, D, seed=9)
    check(x, H, D, st, cuda)


def test_prepass_c0(cuda):
    """8 heads x 2,048 tokens."""
    check(make_qkv(2048, 8, 128, seed=0), 8, 128, 3 * 8 * 128, cuda)


def test_prepass_golden(cuda):
    import glob
    import os

    for path in sorted(glob.glob(os.path.join(os.path.dirname(__file__), "golden", "*.npz"))):
        f = np.load(path)
        S, H, D, dt = (int(f[k]) for k in ("S", "H", "D", "dt"))
        tdt = {native.F16: torch.float16, native.BF16: torch.bfloat16, native.F32: torch.float32}[dt]
        raw = np.ascontiguousarray(f["qkv"])
        t = torch.from_numpy(raw) if dt == native.F32 else torch.from_numpy(raw.view(np.int16)).view(tdt)
        iq, ik, qs, ks, km = gpu_prepass(t.to(cuda), H, D, stride=3 * H * D, dt=dt)
        assert np.array_equal(iq, f["iq"]) and np.array_equal(ik, f["ik"]), path
        assert np.array_equal(qs.view(np.uint32), f["qs"].view(np.uint32)), path
        assert np.array_equal(ks.view(np.uint32), f["ks"].view(np.uint32)), path
        assert np.array_equal(km.view(np.uint32), f["kmean"].view(np.uint32)), path


@pytest.mark.skipif(not oracle.ref_available(), reason="oracle/_ref/libref.so is not built")
@pytest.mark.parametrize("S,H", [(2048, 8), (16848, 32), (47232, 32)])
def test_prepass_vs_reference_source(S, H, cuda):
    """configs[0], [2], [3] at full size: the GPU's int8 q / k, scales and K mean are the bits the reference's own
    kernels/h3sycl.cpp:1733-1761 make of the same inputs (compiled for the CPU from its source)."""
    D = 128
    qkv = make_qkv(S, H, D, seed=S + 1)
    got = gpu_prepass(qkv.to(cuda), H, D)
    host = bits(qkv)
    want = oracle.ref_sage_prepass(host, (host, H * D), (host, 2 * H * D), native.F16, S, H, D, 3 * H * D)[:5]
    for name, g, w in zip(("iq", "ik", "qs", "ks", "kmean"), got, want):
        assert np.array_equal(np.asarray(g).view(np.uint8), np.asarray(w).view(np.uint8)), f"{name} (S={S}, H={H})"
