"""The Ulysses exchange entry points on one GPU, with one process playing every rank: h3s_ulysses_push_qkv,
h3s_ulysses_push_out and h3s_attention_ulysses take the rank, the rank count and the destination table as arguments,
so P ranks' calls can run in turn with every destination a local buffer. This checks the index maps of both push
kernels and the attention epilogue's choice of destination rank per output row (Sage and fp16 paths), bit for bit
against the token <-> head re-sharding they replace; the multi-process form over CUDA IPC is
tests/test_gpu_ulysses_peer.py."""
import pytest
import torch

from sycl_minimax_h3_b200 import native, ops, ulysses

pytestmark = pytest.mark.gpu

CODE = {torch.float16: native.F16, torch.bfloat16: native.BF16, torch.float32: native.F32}


def _bits(t: torch.Tensor) -> torch.Tensor:
    return t.view(torch.int32) if t.element_size() == 4 else t.view(torch.int16)


@pytest.mark.parametrize("P,S,H,D,dtype", [
    (2, 256, 8, 128, torch.float16),
    (4, 512, 8, 64, torch.bfloat16),
    (2, 96, 4, 12, torch.bfloat16),        # 24-byte heads: element copies
    (4, 128, 8, 32, torch.float32),
    (8, 1024, 16, 128, torch.float16),
])
def test_push_kernels_every_rank(P, S, H, D, dtype, cuda):
    ctx = ops.context(cuda)
    g = torch.Generator().manual_seed(P * 1000 + S + D)
    full = torch.randn(S, 3 * H * D, generator=g).to(dtype).to(cuda)
    s, h, es = S // P, H // P, full.element_size()
    heads = [torch.full((S, 3 * h * D), float("nan"), dtype=dtype, device=cuda) for _ in range(P)]
    for r in range(P):
        shard = full[r * s:(r + 1) * s].contiguous()
        ctx.ulysses_push_qkv(shard.data_ptr(), s, H, D, es, P, r, [t.data_ptr() for t in heads])
    ctx.wait()
    for p in range(P):
        assert torch.equal(_bits(heads[p]), _bits(ulysses.head_slice(full, p, P, H, D))), f"forward, rank {p}"
    # inverse: rank p's output = the v columns of its heads; every rank's token shard gets its rows of all heads
    outs = [torch.full((s, H * D), float("nan"), dtype=dtype, device=cuda) for _ in range(P)]
    for p in range(P):
        out_heads = heads[p][:, 2 * h * D:].contiguous()
        ctx.ulysses_push_out(out_heads.data_ptr(), s, H, D, es, P, p, [t.data_ptr() for t in outs])
    ctx.wait()
    for q in range(P):
        assert torch.equal(_bits(outs[q]), _bits(full[q * s:(q + 1) * s, 2 * H * D:].contiguous())), f"inverse, rank {q}"


@pytest.mark.parametrize("P,S,H,D,dtype", [
    (2, 8192, 4, 128, torch.float16),      # the Sage path (S >= 8192)
    (4, 16384, 8, 128, torch.float16),
    (2, 1280, 8, 64, torch.bfloat16),      # the fp16 path, bf16 rows converted first, 64-wide heads
    (4, 640, 8, 128, torch.float16),
])
def test_attention_with_the_exchange(P, S, H, D, dtype, cuda):
    ctx = ops.context(cuda)
    g = torch.Generator().manual_seed(S + P)
    full = torch.randn(S, 3 * H * D, generator=g).to(dtype).to(cuda)
    s, h = S // P, H // P
    outs = [torch.full((s, H * D), float("nan"), dtype=dtype, device=cuda) for _ in range(P)]
    want = [torch.empty_like(o) for o in outs]
    for p in range(P):
        hp = ulysses.head_slice(full, p, P, H, D).contiguous()          # rank p's heads, all tokens
        q, k, v = ops.Rows.qkv(hp, h, D)
        out_heads = torch.empty(S, h * D, dtype=dtype, device=cuda)
        ops.attention(q, k, v, out_heads)
        for r in range(P):                                              # where the push would put it
            want[r][:, p * h * D:(p + 1) * h * D] = out_heads[r * s:(r + 1) * s]
        ctx.attention_ulysses(q.ptr(), k.ptr(), v.ptr(), CODE[dtype], S, h, D, 3 * h * D,
                              [o.data_ptr() for o in outs], P, p, CODE[dtype])
    ctx.wait()
    for r in range(P):
        assert torch.equal(_bits(outs[r]), _bits(want[r])), f"rank {r}'s token shard"


def test_refusals(cuda):
    ctx = ops.context(cuda)
    x = torch.zeros(64, 3 * 8 * 16, dtype=torch.float16, device=cuda)
    d = [x.data_ptr()] * 2
    with pytest.raises(native.H3Error, match="ranks"):
        ctx.ulysses_push_qkv(x.data_ptr(), 32, 8, 16, 2, 9, 0, [x.data_ptr()] * 9)
    with pytest.raises(native.H3Error, match="multiple of the ranks"):
        ctx.ulysses_push_qkv(x.data_ptr(), 32, 7, 16, 2, 2, 0, d)
    with pytest.raises(native.H3Error, match="null"):
        ctx.ulysses_push_out(x.data_ptr(), 32, 8, 16, 2, 2, 1, [x.data_ptr(), 0])
    with pytest.raises(native.H3Error, match="dividing the sequence"):
        ctx.attention_ulysses(x.data_ptr(), x.data_ptr(), x.data_ptr(), native.F16, 63, 4, 16, 3 * 4 * 16, d, 2, 0,
                              native.F16)
