"""The benchmark configurations at full size (BASELINE.json configs[1..3]): the int8 q/k and scales bit for bit over
the whole tensors, and the outputs on 4,096 rows spread over every head and over positions (first and last included)
against float64 softmax (cosine >= 0.999) and the oracle's Sage / SDPA restatement."""
import numpy as np
import pytest
import torch

import oracle
from _util import check_attention, gpu_prepass, run_attention, sample_rows
from sycl_minimax_h3_b200.workloads import bits, make_qkv

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("S", [16848, 47232])
def test_sage_full_size(S, cuda):
    H, D = 32, 128
    qkv = make_qkv(S, H, D, seed=S)
    dq = qkv.to(cuda)
    got = gpu_prepass(dq, H, D)
    host = bits(qkv)
    want = oracle.sage_prepass(host, (host, H * D), (host, 2 * H * D), oracle.F16, S, H, D, 3 * H * D)[:5]
    for name, g, w in zip(("iq", "ik", "qs", "ks", "kmean"), got, want):
        assert np.array_equal(np.asarray(g).view(np.uint8), np.asarray(w).view(np.uint8)), name
    out = run_attention(dq, H, D)                  # default threshold: Sage
    check_attention(qkv, out, H, D, sage=True, rows=sample_rows(S, H, 4096, seed=S))
    # size-independent property: every output row lies in the convex hull of v (softmax weights), so |o| <= max |v|
    v = dq.view(S, 3, H, D)[:, 2].float()
    assert out.float().abs().amax() <= v.abs().amax() * 1.001


def test_sdpa_c1_full(cuda):
    S, H, D = 2159, 32, 128
    qkv = make_qkv(S, H, D, seed=1)
    out = run_attention(qkv.to(cuda), H, D)        # below 8192: fp16 SDPA
    check_attention(qkv, out, H, D, sage=False, rows=sample_rows(S, H, 4096, seed=2))
