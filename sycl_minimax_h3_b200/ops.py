"""The reference engine's attention operators over torch tensors, on libh3cuda.so.

A Python restatement of ``engine/h3-core/src/ops.rs`` of maxfridbe/sycl_minimax_h3 for this path: ``Rows`` (ops.rs
:299-324) describes token rows of ``heads x dim`` features inside a wider row-major buffer - how q, k and v sit inside
the qkv linear's output (offset i*H*D, stride 3*H*D) - and ``attention`` / ``attention_batch`` (ops.rs:405-461) check
the layouts exactly as the reference does, then call ``h3s_attention`` / ``h3s_attention_batch``.
"""
from __future__ import annotations

from dataclasses import dataclass

import torch

from .native import Context, H3Error, dt_code

_ctx: dict[tuple[int, int], Context] = {}


def context(device=None) -> Context:
    """The h3s context of a device around PyTorch's current stream on it (made once per (device, stream))."""
    dev = torch.device("cuda", torch.cuda.current_device() if device is None else torch.device(device).index or 0)
    with torch.cuda.device(dev):
        s = torch.cuda.current_stream()
        key = (dev.index, int(s.cuda_stream))
        if key not in _ctx:
            _ctx[key] = Context(s)
        return _ctx[key]


@dataclass(frozen=True)
class Rows:
    """Token rows of ``heads`` x ``dim`` features inside a wider row-major buffer: row s starts at element
    ``offset + s * stride`` of ``t`` (ops.rs:299-308)."""

    t: torch.Tensor
    offset: int
    stride: int
    tokens: int
    heads: int
    dim: int

    def layout(self):
        return (self.tokens, self.heads, self.dim, self.stride)

    def ptr(self) -> int:
        """The device address of row 0, after the reference's bounds check (ops.rs:310-323)."""
        last = self.offset + (max(self.tokens, 1) - 1) * self.stride + self.heads * self.dim
        if self.stride < self.heads * self.dim or last > self.t.numel():
            raise H3Error(f"rows of {self.heads} x {self.dim} at offset {self.offset} with stride {self.stride} do not "
                          f"fit {list(self.t.shape)}")
        if not self.t.is_contiguous():
            raise H3Error("rows must live in a contiguous tensor")
        return self.t.data_ptr() + self.offset * self.t.element_size()

    @staticmethod
    def qkv(qkv: torch.Tensor, heads: int, dim: int):
        """q, k, v as the three strided parts of a qkv linear's output [tokens, 3 * heads * dim] (dit.rs:346-350)."""
        tokens = qkv.shape[0]
        w = heads * dim
        return tuple(Rows(qkv, i * w, 3 * w, tokens, heads, dim) for i in range(3))

    @staticmethod
    def packed(x: torch.Tensor, heads: int, dim: int) -> "Rows":
        """Rows of a packed [tokens, heads * dim] tensor."""
        return Rows(x, 0, heads * dim, x.shape[0], heads, dim)


def _floats(t: torch.Tensor, what: str, n: int) -> int:
    """A float32 device tensor of exactly n values (ops.rs `floats`)."""
    if t.dtype != torch.float32 or t.numel() != n or not t.is_contiguous():
        raise H3Error(f"{what}: {n} contiguous float32 values expected, got {list(t.shape)} {t.dtype}")
    return t.data_ptr()


def rms_rope(x: Rows, weight: torch.Tensor, eps: float, cs: torch.Tensor, rot_dim: int) -> None:
    """Per-head RMS norm (weight float32 [dim]) and the rotary rotation, in place; ``cs`` float32
    [tokens, rot_dim/2, 2] of (cos, sin) (ops.rs:326-345, kernels/h3sycl.h:165-174)."""
    ctx = context(x.t.device)
    ctx.rms_rope(x.ptr(), dt_code(x.t.dtype), x.tokens, x.heads, x.dim, x.stride,
                 _floats(weight, "the norm weight", x.dim), eps, _floats(cs, "the rotation table", x.tokens * rot_dim),
                 rot_dim)


@dataclass(frozen=True)
class Int8Linear:
    """A linear layer with int8 weights (one layer of an ``int8_convrot`` checkpoint), on the device (ops.rs:25-80):
    ``weight`` int8 [N, K], ``scale`` float32 with 1 or N values, ``bias`` float32 [N] or None, ``group`` the rotation
    group size when the weights were stored rotated."""

    weight: torch.Tensor
    scale: torch.Tensor
    bias: torch.Tensor | None = None
    group: int | None = None

    def inputs(self) -> int:
        return self.weight.shape[1]

    def outputs(self) -> int:
        return self.weight.shape[0]

    def forward(self, x: torch.Tensor, out: torch.Tensor) -> None:
        """``out = linear(x)``: x [M, K] in a float type, out [M, N] in out's type (ops.rs:45-79)."""
        n, k = self.outputs(), self.inputs()
        m = x.numel() // k
        if self.weight.dtype != torch.int8 or self.scale.dtype != torch.float32:
            raise H3Error("int8_linear: the weight must be int8 and its scale float32")
        if x.numel() != m * k or out.numel() != m * n:
            raise H3Error(f"int8_linear: x {list(x.shape)} and out {list(out.shape)} do not fit a [{n}, {k}] weight")
        ns = self.scale.numel()
        if ns != 1 and ns != n:
            raise H3Error(f"int8_linear: {ns} weight scales for {n} outputs")
        for t, what in ((x, "x"), (out, "out"), (self.weight, "the weight"), (self.scale, "the scale")):
            if not t.is_contiguous():
                raise H3Error(f"int8_linear: {what} must be contiguous")
        bias = _floats(self.bias, "the bias", n) if self.bias is not None else 0
        ctx = context(out.device)
        ctx.int8_linear(x.data_ptr(), dt_code(x.dtype), m, k, self.weight.data_ptr(), n, self.scale.data_ptr(), ns,
                        bias, out.data_ptr(), dt_code(out.dtype), self.group or 0)


def attention_causal(q: Rows, k: Rows, v: Rows, out: torch.Tensor) -> None:
    """Causal attention with grouped heads (the text encoder's call, te.rs:340-346): q has the query heads, k and v the
    key/value heads (a divisor of them), all with the same tokens and head size; out [tokens, q.heads * dim] in q's
    type (kernels/h3sycl.h:105-108)."""
    if k.layout()[1:3] != v.layout()[1:3] or k.stride != v.stride or q.tokens != k.tokens or k.tokens != v.tokens:
        raise H3Error("attention_causal: k and v must have the same layout, and q, k, v the same tokens")
    if q.dim != k.dim or k.heads == 0 or q.heads % k.heads != 0:
        raise H3Error(f"attention_causal: {q.heads} query heads over {k.heads} key/value heads of {k.dim}")
    if q.t.dtype != k.t.dtype or q.t.dtype != v.t.dtype or out.dtype != q.t.dtype:
        raise H3Error("attention_causal: q, k, v and out must have one element type")
    if out.numel() != q.tokens * q.heads * q.dim or not out.is_contiguous():
        raise H3Error(f"attention_causal: out {list(out.shape)} for {q.tokens} tokens of {q.heads} x {q.dim}")
    ctx = context(out.device)
    ctx.attention_causal(q.ptr(), k.ptr(), v.ptr(), dt_code(q.t.dtype), q.tokens, q.heads, k.heads, q.dim, q.stride,
                         k.stride, out.data_ptr())


def attention(q: Rows, k: Rows, v: Rows, out: torch.Tensor) -> None:
    """``out = softmax(q . k^T / sqrt(dim)) . v`` per head; out [tokens, heads * dim] (ops.rs:436-461)."""
    if q.layout() != k.layout() or q.layout() != v.layout():
        raise H3Error("attention: q, k and v must have the same layout")
    if out.numel() != q.tokens * q.heads * q.dim:
        raise H3Error(f"attention: out {list(out.shape)} for {q.tokens} tokens of {q.heads} x {q.dim}")
    if not out.is_contiguous():
        raise H3Error("attention: out must be contiguous")
    ctx = context(out.device)
    ctx.attention(q.ptr(), k.ptr(), v.ptr(), dt_code(q.t.dtype), q.tokens, q.heads, q.dim, q.stride, out.data_ptr(),
                  dt_code(out.dtype))


def attention_batch(q: Rows, k: Rows, v: Rows, seqs: int, out: torch.Tensor) -> None:
    """Attention over ``seqs`` independent sequences of ``q.tokens / seqs`` tokens each, in one call (ops.rs:405-434)."""
    if q.layout() != k.layout() or q.layout() != v.layout():
        raise H3Error("attention_batch: q, k and v must have the same layout")
    if seqs == 0 or q.tokens % seqs != 0:
        raise H3Error(f"attention_batch: {q.tokens} tokens are not {seqs} equal sequences")
    if out.numel() != q.tokens * q.heads * q.dim:
        raise H3Error(f"attention_batch: out {list(out.shape)} for {q.tokens} tokens of {q.heads} x {q.dim}")
    ctx = context(out.device)
    ctx.attention_batch(q.ptr(), k.ptr(), v.ptr(), dt_code(q.t.dtype), seqs, q.tokens // seqs, q.heads, q.dim, q.stride,
                        out.data_ptr(), dt_code(out.dtype))


def attention_rms_rope(q: Rows, k: Rows, v: Rows, out: torch.Tensor, q_norm: torch.Tensor, k_norm: torch.Tensor,
                       eps: float, cs: torch.Tensor, rot_dim: int) -> None:
    """A denoiser block's ``rms_rope(q)``, ``rms_rope(k)``, ``attention(q, k, v, out)`` in one call (dit.rs:347-350):
    q and k are left normalised and rotated in place, as the two ``rms_rope`` calls leave them."""
    if q.layout() != k.layout() or q.layout() != v.layout():
        raise H3Error("attention_rms_rope: q, k and v must have the same layout")
    if out.numel() != q.tokens * q.heads * q.dim or not out.is_contiguous():
        raise H3Error(f"attention_rms_rope: out {list(out.shape)} for {q.tokens} tokens of {q.heads} x {q.dim}")
    ctx = context(out.device)
    ctx.attention_rms_rope(q.ptr(), k.ptr(), v.ptr(), dt_code(q.t.dtype), q.tokens, q.heads, q.dim, q.stride,
                           out.data_ptr(), dt_code(out.dtype), _floats(q_norm, "the q norm weight", q.dim),
                           _floats(k_norm, "the k norm weight", q.dim), eps,
                           _floats(cs, "the rotation table", q.tokens * rot_dim), rot_dim)
