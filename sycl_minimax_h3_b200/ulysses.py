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


class _DeviceBuffer:
    """A device allocation of the h3s context seen as a torch tensor (through __cuda_array_interface__; 2-byte types
    as int16, viewed as the element type afterwards)."""

    def __init__(self, ptr: int, shape: tuple[int, ...], es: int):
        self.__cuda_array_interface__ = {"shape": shape, "typestr": "<i2" if es == 2 else "<f4", "data": (ptr, False),
                                         "version": 3, "strides": None}


def _as_tensor(ptr: int, shape: tuple[int, ...], dtype: torch.dtype, dev: torch.device) -> torch.Tensor:
    es = torch.empty((), dtype=dtype).element_size()
    return torch.as_tensor(_DeviceBuffer(ptr, shape, es), device=dev).view(dtype)


class PeerExchange:
    """The Ulysses all-to-alls as stores into the other ranks' memory (h3s_ulysses_push_qkv / _out over CUDA IPC),
    for P ranks on one node (one process per GPU). The relayout and the transfer are one kernel per direction; the
    ranks meet through a one-element all-reduce on the current stream before a push (nobody still reads the buffer
    being overwritten) and after it (everything has arrived). Same layouts and results as seq_to_heads /
    heads_to_seq; the receive buffers belong to this object and are reused by every call."""

    def __init__(self, s: int, H: int, D: int, dtype: torch.dtype = torch.float16, group=None):
        from .ops import context   # loads libh3cuda.so: no exchange without it

        self.group = group
        self.P = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if H % self.P or self.P > 8:
            raise ValueError(f"{H} heads over {self.P} ranks: H must be a multiple of the ranks, at most 8 ranks")
        self.s, self.H, self.D, self.dtype = s, H, D, dtype
        self.h = H // self.P
        self.es = torch.empty((), dtype=dtype).element_size()
        self.ctx = context()
        dev = torch.device("cuda", torch.cuda.current_device())
        S = self.P * s
        self._own = [self.ctx.alloc(S * 3 * self.h * D * self.es), self.ctx.alloc(s * H * D * self.es)]
        self.heads = _as_tensor(self._own[0], (S, 3 * self.h * D), dtype, dev)
        self.out = _as_tensor(self._own[1], (s, H * D), dtype, dev)
        # every rank's two buffers: handles gathered over the group, opened where they are another rank's. A failure
        # on any rank is decided together (below), so that no rank is left waiting in a collective the others skip.
        why = ""
        try:
            mine = bytes(self.ctx.ipc_handle(self._own[0]) + self.ctx.ipc_handle(self._own[1]))
        except Exception as e:
            why, mine = str(e), bytes(128)
        mine_t = torch.frombuffer(bytearray(mine), dtype=torch.uint8).to(dev)
        every = [torch.empty_like(mine_t) for _ in range(self.P)]
        dist.all_gather(every, mine_t, group=group)
        self._opened = []
        self.dst_heads, self.dst_out = [], []
        try:
            if why:
                raise RuntimeError(why)
            for p, t in enumerate(every):
                if p == self.rank:
                    self.dst_heads.append(self._own[0])
                    self.dst_out.append(self._own[1])
                    continue
                raw = bytes(t.cpu().numpy().tobytes())
                self._opened.append(self.ctx.ipc_open(raw[:64]))
                self.dst_heads.append(self._opened[-1])
                self._opened.append(self.ctx.ipc_open(raw[64:]))
                self.dst_out.append(self._opened[-1])
        except Exception as e:  # decided together below, so that every rank takes the same path
            why = str(e)
        self._flag = torch.zeros(1, device=dev)
        ok = torch.tensor([0.0 if why else 1.0], device=dev)
        dist.all_reduce(ok, op=dist.ReduceOp.MIN, group=group)
        if ok.item() < 1.0:
            self.close()
            raise RuntimeError(f"PeerExchange: a rank could not open the other ranks' buffers ({why or 'elsewhere'})")
        self._meet()

    def _meet(self) -> None:
        dist.all_reduce(self._flag, group=self.group)

    def seq_to_heads(self, shard: torch.Tensor) -> torch.Tensor:
        """Token-sharded qkv [s, 3*H*D] -> this rank's head-sharded qkv [S, 3*(H/P)*D] (token order)."""
        if shard.shape != (self.s, 3 * self.H * self.D) or shard.dtype != self.dtype or not shard.is_contiguous():
            raise ValueError(f"shard {list(shard.shape)} {shard.dtype}: [{self.s}, {3 * self.H * self.D}] "
                             f"{self.dtype} contiguous expected")
        self._meet()
        self.ctx.ulysses_push_qkv(shard.data_ptr(), self.s, self.H, self.D, self.es, self.P, self.rank, self.dst_heads)
        self._meet()
        return self.heads

    def heads_to_seq(self, out_heads: torch.Tensor) -> torch.Tensor:
        """Head-sharded output [S, (H/P)*D] -> this rank's token-sharded output [S/P, H*D]."""
        if out_heads.shape != (self.P * self.s, self.h * self.D) or out_heads.dtype != self.dtype or \
                not out_heads.is_contiguous():
            raise ValueError(f"output {list(out_heads.shape)}: [{self.P * self.s}, {self.h * self.D}] expected")
        self._meet()
        self.ctx.ulysses_push_out(out_heads.data_ptr(), self.s, self.H, self.D, self.es, self.P, self.rank,
                                  self.dst_out)
        self._meet()
        return self.out

    def attention_to_seq(self, heads: torch.Tensor, dst: list[int] | None = None) -> torch.Tensor:
        """The attention of this rank's heads over all tokens (heads [S, 3*(H/P)*D], q | k | v, as seq_to_heads
        returns it), with the inverse exchange in the attention's epilogue (h3s_attention_ulysses): each output row
        is stored straight into its rank's token shard. Returns this rank's token-sharded output [S/P, H*D].

        The ranks meet before the attention (no rank still reads its shard from the previous call) and after it
        (every row has arrived). A wait that gives up inside the kernel is reported by check(), not here.
        dst replaces the destination table (P device pointers); a table of this rank's own buffer P times keeps
        every store local, which times the same kernel without the NVLink traffic."""
        from .native import dt_code

        S, h, D = self.P * self.s, self.h, self.D
        if heads.shape != (S, 3 * h * D) or heads.dtype != self.dtype or not heads.is_contiguous():
            raise ValueError(f"heads {list(heads.shape)}: [{S}, {3 * h * D}] {self.dtype} contiguous expected")
        base, es = heads.data_ptr(), self.es
        # every rank has finished reading its token shard (self.out) of the previous call before any epilogue
        # overwrites it
        self._meet()
        self.ctx.attention_ulysses(base, base + h * D * es, base + 2 * h * D * es, dt_code(self.dtype), S, h, D,
                                   3 * h * D, dst if dst is not None else self.dst_out, self.P, self.rank,
                                   dt_code(self.dtype))
        self._meet()
        return self.out

    def check(self) -> None:
        """Raises on every rank together when a kernel of any rank gave up on a wait since the last check.

        A rank whose attention gave up sets only its own context's error word and skips its stores into the other
        ranks' shards, which then hold stale rows with no error of their own. This waits for the rank's stream, reads
        and clears its error word (h3s_wait), and takes the maximum over the group, so that no rank goes on with
        rows another rank failed to write. Collective: every rank calls it at the same point."""
        why = ""
        try:
            self.ctx.wait()
        except Exception as e:  # decided together below
            why = str(e)
        bad = torch.tensor([1.0 if why else 0.0], device=self._flag.device)
        dist.all_reduce(bad, op=dist.ReduceOp.MAX, group=self.group)
        if bad.item() > 0:
            raise RuntimeError(f"PeerExchange: a kernel gave up on a wait ({why or 'on another rank'})")

    def close(self) -> None:
        """Unmaps the other ranks' buffers and frees this rank's (after every rank is done with them)."""
        torch.cuda.synchronize()
        self._meet()
        torch.cuda.synchronize()
        for p in self._opened:
            self.ctx.ipc_close(p)
        self._opened = []
        self._meet()
        torch.cuda.synchronize()
        for p in self._own:
            self.ctx.free(p)
        self._own = []
