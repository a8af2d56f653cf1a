"""Synthetic inputs of the benchmark configurations (BASELINE.json ``configs``).

No public dataset is involved: the denoiser's q, k, v are stood in for by seeded normal values with the stated
distributions. Q, V ~ N(0, 1); K = N(0, 1) + c[h, d], with the per-channel offset c ~ N(0, 4) drawn once per (head,
channel), so the K channel-mean smoothing of SageAttention matters. Softmax scale 1/sqrt(128).
"""
from __future__ import annotations

from dataclasses import dataclass

import torch


@dataclass(frozen=True)
class Config:
    name: str
    S: int
    H: int
    D: int = 128
    path: str = "sage"


CONFIGS = {
    "c0": Config("c0: 8 heads x 2,048 tokens (parity case)", 2048, 8),
    "c1": Config("c1: 32 heads x 2,159 tokens, fp16 SDPA (1-step preview)", 2159, 32, path="sdpa"),
    "c2": Config("c2: 32 heads x 16,848 tokens, Sage (5-second clip)", 16848, 32),
    "c3": Config("c3: 32 heads x 47,232 tokens, Sage x 50 blocks (15-second clip)", 47232, 32),
}


def make_qkv(S: int, H: int, D: int = 128, seed: int = 0, device="cpu", dtype=torch.float16) -> torch.Tensor:
    """A qkv buffer [S, 3*H*D] as the qkv linear produces it: q, k, v side by side in every token row (stride 3*H*D)."""
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    qkv = torch.randn(S, 3 * H * D, generator=g, device=device, dtype=torch.float32)
    offset = torch.randn(H * D, generator=g, device=device, dtype=torch.float32) * 2.0
    qkv[:, H * D:2 * H * D] += offset
    return qkv.to(dtype)


def bits(t: torch.Tensor):
    """A CPU numpy view of a tensor for the oracle: uint16 bit patterns for half/bfloat16, float32 as is."""
    t = t.detach().contiguous().cpu()
    if t.dtype in (torch.float16, torch.bfloat16):
        return t.view(torch.int16).numpy().view("uint16")
    return t.numpy()
