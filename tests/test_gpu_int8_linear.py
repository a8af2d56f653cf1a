"""h3s_int8_linear on the GPU through the C ABI against the oracle: the int8 ConvRot linear of every denoiser block
(kernels/h3sycl.h:74-85, kernels/h3sycl.cpp:404-652; engine/h3-core/src/ops.rs:25-80).

The rotation runs in the order of the reference's fused kernel, the quantisation and the rescale with every step
rounded, and the int8 products are exact, so the results must be bit-exact with the oracle: all input and output
types, every group size the reference accepts, rows that stay in shared memory and rows that do not, K that is not a
multiple of 16 or of the 128-byte K slice, tile edges in M and N, per-output scales and bias, more tiles than SMs, row
chunks, and the reference's refusals. Against the reference's own semantics (engine/h3-core/src/reference.rs): with
rotated weights the layer stays within quantisation of the plain float linear."""
import numpy as np
import pytest
import torch

import oracle
from sycl_minimax_h3_b200 import native, ops

pytestmark = pytest.mark.gpu

CODE = {torch.float16: native.F16, torch.bfloat16: native.BF16, torch.float32: native.F32}
TORCH = {v: k for k, v in CODE.items()}


def bits(t: torch.Tensor) -> np.ndarray:
    c = t.cpu().contiguous()
    return c.view(torch.int16).numpy().view(np.uint16) if c.element_size() == 2 else c.numpy()


def inputs(M, K, N, dtype, seed, per_n=False, bias=True):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(M, K, generator=g) * 2
    x[:, ::37] *= 8                                  # a few large features per row, as activations have
    x = x.to(dtype)
    w = torch.randint(-127, 128, (N, K), generator=g, dtype=torch.int8)
    ws = (torch.rand(N if per_n else 1, generator=g) * 0.02 + 0.001).float()
    b = torch.randn(N, generator=g).float() if bias else None
    return x, w, ws, b


def run(x, w, ws, b, out_dtype, group, cuda):
    M, K = x.shape
    N = w.shape[0]
    out = torch.full((M, N), float("nan"), dtype=out_dtype, device=cuda)
    xd, wd, wsd = x.to(cuda), w.to(cuda), ws.to(cuda)
    bd = b.to(cuda) if b is not None else None
    ctx = ops.context(cuda)
    ctx.int8_linear(xd.data_ptr(), CODE[x.dtype], M, K, wd.data_ptr(), N, wsd.data_ptr(), ws.numel(),
                    bd.data_ptr() if bd is not None else 0, out.data_ptr(), CODE[out_dtype], group)
    ctx.wait()
    return out


def expect(x, w, ws, b, out_dtype, group):
    M, K = x.shape
    return oracle.int8_linear(bits(x), CODE[x.dtype], M, K, w.numpy(), w.shape[0], ws.numpy(),
                              None if b is None else b.numpy(), CODE[out_dtype], group)


def check(M, K, N, dtype, out_dtype, group, cuda, seed=0, per_n=False, bias=True):
    x, w, ws, b = inputs(M, K, N, dtype, seed, per_n, bias)
    got = bits(run(x, w, ws, b, out_dtype, group, cuda))
    want = expect(x, w, ws, b, out_dtype, group)
    assert np.array_equal(got, want), f"{np.count_nonzero(got != want)} of {got.size} differ"


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float16, torch.float32])
@pytest.mark.parametrize("group", [0, 2, 4, 8, 16, 32, 64, 128, 256])
def test_bit_exact_every_group(dtype, group, cuda):
    check(300, 512, 600, dtype, torch.bfloat16, group, cuda, seed=group + 1)


@pytest.mark.parametrize("out_dtype", [torch.bfloat16, torch.float16, torch.float32])
@pytest.mark.parametrize("per_n,bias", [(False, False), (False, True), (True, False), (True, True)])
def test_output_types_scales_and_bias(out_dtype, per_n, bias, cuda):
    check(130, 768, 520, torch.bfloat16, out_dtype, 256, cuda, seed=7, per_n=per_n, bias=bias)


@pytest.mark.parametrize("K,group", [
    (4096, 256),       # one window of the rotation kernel
    (12288, 256),      # three windows, the row kept in shared memory
    (16384, 64),       # the longest row kept in shared memory
    (20480, 256),      # longer: rotated twice
    (100, 4),          # K % 16 != 0: the weight is copied with padded rows, the loads are scalar
    (24, 8),
    (40, 0),
    (136, 0),          # a partial 128-byte K slice
    (8, 2),
])
def test_row_lengths(K, group, cuda):
    check(70, K, 300, torch.bfloat16, torch.bfloat16, group, cuda, seed=K)


@pytest.mark.parametrize("M,N", [(1, 256), (129, 37), (2, 8), (257, 513), (128, 255)])
def test_tile_edges(M, N, cuda):
    check(M, 256, N, torch.float16, torch.float16, 256, cuda, seed=M * 1000 + N, per_n=True)


def test_more_tiles_than_sms(cuda):
    """2048 x 4096 outputs: 256 tiles of 128 x 256, so every CTA of the persistent kernel takes several and both
    accumulators cycle."""
    check(2048, 256, 4096, torch.bfloat16, torch.bfloat16, 256, cuda, seed=11, per_n=True)


def _sampled_rows(M, K, N, group, cuda, seed, rows=48):
    """A large layer on the GPU, checked row by row against the oracle on a sample of rows (rows are independent)."""
    gen = torch.Generator(device=cuda).manual_seed(seed)
    x = (torch.randn(M, K, generator=gen, device=cuda) * 2).to(torch.bfloat16)
    g = torch.Generator().manual_seed(seed)
    w = torch.randint(-127, 128, (N, K), generator=g, dtype=torch.int8)
    ws = (torch.rand(N, generator=g) * 0.02 + 0.001).float()
    b = torch.randn(N, generator=g).float()
    out = torch.empty(M, N, dtype=torch.bfloat16, device=cuda)
    ops.Int8Linear(w.to(cuda), ws.to(cuda), b.to(cuda), group).forward(x, out)
    ops.context(cuda).wait()
    pick = torch.cat([torch.tensor([0, M - 1]), torch.randperm(M, generator=g)[:rows - 2]]).sort().values
    xs = x[pick.to(cuda)].cpu()
    want = oracle.int8_linear(bits(xs), native.BF16, len(pick), K, w.numpy(), N, ws.numpy(), b.numpy(), native.BF16,
                              group)
    got = bits(out[pick.to(cuda)])
    assert np.array_equal(got, want), f"{np.count_nonzero(got != want)} of {got.size} differ"


def test_block_size_qkv(cuda):
    """The qkv projection of a 47k-token block (hidden 4096 -> 3 x 4096), bit-exact on sampled rows."""
    _sampled_rows(47232, 4096, 12288, 256, cuda, seed=3)


def test_row_chunks(cuda):
    """More than 1 GiB of int8 activations (70000 x 16384): the entry point runs two row chunks."""
    _sampled_rows(70000, 16384, 256, 256, cuda, seed=4, rows=24)


def test_rotated_weights_match_a_plain_linear(cuda):
    """reference.rs:115-127's check with the rotation on: weights stored rotated (W . H per group, quantised per output
    row), x rotated on the fly; the layer is within quantisation of the plain float linear x . W^T."""
    M, K, N, G = 64, 1024, 96, 256
    g = torch.Generator().manual_seed(5)
    x = torch.randn(M, K, generator=g)
    wf = torch.randn(N, K, generator=g) / 32
    # the normalised Hadamard matrix of G, h4 (x) h4 (x) h4 (x) h4 (kernels/h3sycl.cpp:185-200)
    h4 = torch.tensor([[1, 1, 1, -1], [1, 1, -1, 1], [1, -1, 1, 1], [-1, 1, 1, 1]], dtype=torch.float64)
    h = torch.ones(1, 1, dtype=torch.float64)
    for _ in range(4):
        h = torch.kron(h4, h)
    h = h / 16
    wr = (wf.double().reshape(N, K // G, G) @ h).reshape(N, K)
    sc = wr.abs().amax(1) / 127
    wq = torch.round(wr / sc[:, None]).clamp(-127, 127).to(torch.int8)
    out = torch.empty(M, N, dtype=torch.float32, device=cuda)
    ops.Int8Linear(wq.to(cuda), sc.float().to(cuda), None, G).forward(x.to(cuda), out)
    ops.context(cuda).wait()
    want = x.double() @ wf.double().T
    got = out.cpu().double()
    rel = ((got - want).norm() / want.norm()).item()
    cos = (torch.dot(got.flatten(), want.flatten()) / (got.norm() * want.norm())).item()
    assert rel < 0.02 and cos > 0.999, (rel, cos)


def test_quantiser_ties(cuda):
    """Quotients exactly on a half (round half to even: 0.5 -> 0, 1.5 -> 2, -2.5 -> -2) and one float step either side
    of it, read through an identity weight (out = the int8 codes times the row scale). Rows 0-1 have scales 1 and 2
    (max 127 and 254), so the quotients are exact; rows 2-3 sit one step off the halves; the rest are random."""
    K = 256
    x = np.random.default_rng(2).standard_normal((6, K)).astype(np.float32) * 3
    halves = np.arange(-127, 127, dtype=np.float32) + np.float32(0.5)      # -126.5 .. 126.5: columns 1-254
    x[:4, 255] = 0
    x[0, 0], x[0, 1:255] = 127, halves
    x[1, 0], x[1, 1:255] = 254, 2 * halves
    x[2, 0], x[2, 1:255] = 127, np.nextafter(halves, np.float32(np.inf))
    x[3, 0], x[3, 1:255] = 127, np.nextafter(halves, np.float32(-np.inf))
    xt = torch.from_numpy(x)
    w = torch.eye(K, dtype=torch.int8)
    ws = torch.ones(1)
    got = run(xt, w, ws, None, torch.float32, 0, cuda).cpu().numpy()
    want = expect(xt, w, ws, None, torch.float32, 0)
    assert np.array_equal(got, want)
    codes = np.rint(halves.astype(np.float64))
    assert np.array_equal(got[0, 1:255], codes) and np.array_equal(got[1, 1:255], 2 * codes)
    assert np.array_equal(got[2, 1:255], np.ceil(halves)) and np.array_equal(got[3, 1:255], np.floor(halves))


def test_refusals_and_degenerate_sizes(cuda):
    ctx = ops.context(cuda)
    x = torch.randn(4, 64, device=cuda).half()
    w = torch.ones(8, 64, dtype=torch.int8, device=cuda)
    ws = torch.ones(1, device=cuda)
    out = torch.zeros(4, 8, device=cuda).half()
    for group in (3, 6, 512, 128 * 3):
        with pytest.raises(native.H3Error, match="unsupported ConvRot group size"):
            ctx.int8_linear(x.data_ptr(), native.F16, 4, 64, w.data_ptr(), 8, ws.data_ptr(), 1, 0, out.data_ptr(),
                            native.F16, group)
    with pytest.raises(native.H3Error, match="unsupported ConvRot group size"):      # K % group != 0
        ctx.int8_linear(x.data_ptr(), native.F16, 4, 48, w.data_ptr(), 8, ws.data_ptr(), 1, 0, out.data_ptr(),
                        native.F16, 32)
    with pytest.raises(native.H3Error, match="n_wscale"):
        ctx.int8_linear(x.data_ptr(), native.F16, 4, 64, w.data_ptr(), 8, ws.data_ptr(), 2, 0, out.data_ptr(),
                        native.F16, 0)
    with pytest.raises(native.H3Error, match="element type"):
        ctx.int8_linear(x.data_ptr(), 9, 4, 64, w.data_ptr(), 8, ws.data_ptr(), 1, 0, out.data_ptr(), native.F16, 0)
    for M, K, N in ((0, 64, 8), (4, 0, 8), (4, 64, 0), (-1, 64, 8)):
        ctx.int8_linear(x.data_ptr(), native.F16, M, K, w.data_ptr(), N, ws.data_ptr(), 1, 0, out.data_ptr(),
                        native.F16, 3)
    ctx.wait()
    assert torch.count_nonzero(out).item() == 0
    # ops-level checks (ops.rs:47-58)
    lin = ops.Int8Linear(w, torch.ones(3, device=cuda), None, None)
    with pytest.raises(native.H3Error, match="3 weight scales for 8 outputs"):
        lin.forward(x, out)
    with pytest.raises(native.H3Error, match="do not fit"):
        ops.Int8Linear(w, ws).forward(x, torch.zeros(4, 9, device=cuda).half())
    with pytest.raises(native.H3Error, match="must be int8"):
        ops.Int8Linear(w.float(), ws).forward(x, out)


def test_one_sm_gemm_variant_bit_exact(tmp_path):
    """The one-SM GEMM (i8gemm, H3S_LIN_KERNEL=1: read once per process, so a child process) gives the same bits as
    the oracle, as the SM-pair kernel the product runs by default does."""
    import os
    import subprocess
    import sys

    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    code = f"""
import sys
sys.path[:0] = [{root!r}, {os.path.join(root, 'oracle')!r}, {os.path.join(root, 'tests')!r}]
import numpy as np, torch
import oracle
from test_gpu_int8_linear import inputs, run, bits, CODE
cuda = torch.device("cuda", 0)
for (M, K, N, dt, group) in ((300, 512, 700, torch.bfloat16, 256), (129, 1024, 260, torch.float16, 32), (70, 136, 300, torch.bfloat16, 0)):
    x, w, ws, b = inputs(M, K, N, dt, seed=M + K, per_n=True)
    got = run(x, w, ws, b, dt, group, cuda)
    want = oracle.int8_linear(bits(x), CODE[dt], M, K, w.numpy(), N, ws.numpy(), b.numpy(), CODE[dt], group)
    assert np.array_equal(bits(got), want), (M, K, N)
print("ok")
"""
    env = dict(os.environ, H3S_LIN_KERNEL="1")
    res = subprocess.run([sys.executable, "-c", code], env=env, capture_output=True, text=True, timeout=600)
    assert res.returncode == 0 and res.stdout.strip().endswith("ok"), res.stdout[-2000:] + res.stderr[-2000:]
