"""Ulysses sequence parallelism for the denoiser's self-attention: head <-> sequence all-to-all over NCCL.

The reference runs one sequence on one GPU (its attention has no multi-GPU form). Here a sequence of S tokens starts
sharded by tokens over P ranks (S/P rows of all H heads each, row-major [S/P, 3*H*D] qkv). One all-to-all re-shards
q, k and v to "all S tokens x H/P heads" per rank; each rank then runs the whole attention path (K mean over all S
tokens, per-64-row quantisation, Sage or SDPA) on its heads - bit for bit what one GPU would compute for those heads,
because every head's statistics see the full sequence; and the inverse all-to-all of the output restores the token
shards. Head sharding needs no exchange at all when the activations are already head-sharded.

Layouts (P ranks, rank r, s = S/P, h = H/P, D features):
  qkv_shard [s, 3*H*D]       token rows r*s .. r*s+s-1, all heads (q | k | v)
  qkv_heads [S, 3*h*D]       all tokens, heads r*h .. r*h+h-1 (q | k | v), token order
  out_heads [S, h*D]         the attention output of this rank's heads
  out_shard [s, H*D]         token rows of this rank, all heads
"""
from __future__ import annotations

import torch
import torch.distributed as dist


def _split_heads(x: torch.Tensor, P: int, parts: int, H: int, D: int) -> torch.Tensor:
    """[s, parts*H*D] -> [P, s, parts*(H/P)*D]: for each destination rank, its heads of every part (q, k, v)."""
    s = x.shape[0]
    h = H // P
    return x.view(s, parts, P, h * D).permute(2, 0, 1, 3).reshape(P, s, parts * h * D)


def seq_to_heads(qkv_shard: torch.Tensor, H: int, D: int, group=None) -> torch.Tensor:
    """The forward all-to-all: token-sharded qkv [s, 3*H*D] -> head-sharded qkv [S, 3*(H/P)*D] (token order)."""
    P = dist.get_world_size(group)
    if H % P:
        raise ValueError(f"{H} heads do not split over {P} ranks")
    s = qkv_shard.shape[0]
    send = _split_heads(qkv_shard, P, 3, H, D).contiguous()          # [P, s, 3*h*D]
    recv = torch.empty_like(send)                                    # [P (source rank = token block), s, 3*h*D]
    dist.all_to_all_single(recv, send, group=group)
    return recv.view(P * s, send.shape[2])


def heads_to_seq(out_heads: torch.Tensor, H: int, D: int, group=None) -> torch.Tensor:
    """The inverse all-to-all: head-sharded output [S, (H/P)*D] -> token-sharded output [S/P, H*D]."""
    P = dist.get_world_size(group)
    S = out_heads.shape[0]
    s, h = S // P, H // P
    send = out_heads.contiguous().view(P, s, h * D)                  # token block p goes to rank p
    recv = torch.empty_like(send)                                    # [P (source rank = head block), s, h*D]
    dist.all_to_all_single(recv, send, group=group)
    return recv.permute(1, 0, 2).reshape(s, H * D)


def head_slice(qkv: torch.Tensor, rank: int, P: int, H: int, D: int) -> torch.Tensor:
    """Rank r's heads of a full qkv buffer [S, 3*H*D] -> [S, 3*(H/P)*D] (the layout seq_to_heads produces)."""
    S = qkv.shape[0]
    h = H // P
    return qkv.view(S, 3, H, D)[:, :, rank * h:(rank + 1) * h, :].reshape(S, 3 * h * D)
