"""h3s_attention_sage_static, the allocation-free entry point, against h3s_attention on the same inputs.

It serves callers that cannot allocate device memory when they call (a path that must not synchronise the device, or a
host whose device memory is owned and budgeted by another allocator): its scratch is a fixed array inside libh3cuda.so
instead of memory allocated per call. This file is named so that pytest collects it last: a run that stops at the
first failure has run every other test before it."""
import ctypes

import numpy as np
import pytest
import torch

import oracle
from _util import MIN_ROW_COSINE_VS_SAME_SEMANTICS, check_attention, run_attention
from sycl_minimax_h3_b200 import native
from sycl_minimax_h3_b200.workloads import make_qkv

pytestmark = pytest.mark.gpu


def call_static(qkv: torch.Tensor, H: int, D: int, out: torch.Tensor, err: torch.Tensor) -> int:
    """One call through the C ABI on PyTorch's current stream; q, k, v are the strided parts of qkv."""
    st = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    base = qkv.data_ptr()
    return native.lib().h3s_attention_sage_static(ctypes.byref(st), base, base + H * D * 2, base + 2 * H * D * 2,
                                                  qkv.shape[0], H, D, 3 * H * D, out.data_ptr(), native.F16,
                                                  err.data_ptr())


def test_two_calls_match_h3s_attention(cuda):
    H, D = 8, 128
    err = torch.full((1,), 7, dtype=torch.int32, device=cuda)      # each call sets it to 0 first
    for S, seed in ((2048, 11), (700, 12)):                          # two calls in a row, the array reused
        qkv_cpu = make_qkv(S, H, D, seed=seed)
        qkv = qkv_cpu.to(cuda)
        out = torch.empty(S, H * D, dtype=torch.float16, device=cuda)
        assert call_static(qkv, H, D, out, err) == 0, native.last_error()
        torch.cuda.synchronize()
        assert int(err.item()) == 0, "a wait inside the kernels gave up"
        ref = run_attention(qkv, H, D, min_s=0)                     # the existing entry point, its Sage path
        got = out.float().cpu().numpy().reshape(-1, D)
        want = ref.float().cpu().numpy().reshape(-1, D)
        # the tolerance the attention tests use between two runs of the same arithmetic
        assert oracle.row_cosines(got, want).min() >= MIN_ROW_COSINE_VS_SAME_SEMANTICS
        assert float(np.max(np.abs(got - want))) <= 1e-3
        check_attention(qkv_cpu, out, H, D, sage=True)              # and the oracle's bounds against float64


def test_sizes_beyond_the_array_are_refused(cuda):
    H, D, S = 32, 128, 1025                                          # S*H*D = 4,198,400 > 4,194,304
    qkv = torch.zeros(S, 3 * H * D, dtype=torch.float16, device=cuda)
    out = torch.empty(S, H * D, dtype=torch.float16, device=cuda)
    err = torch.zeros(1, dtype=torch.int32, device=cuda)
    assert call_static(qkv, H, D, out, err) == -1
    assert "beyond the fixed scratch" in native.last_error()
