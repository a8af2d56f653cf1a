"""The Ulysses re-sharding on CPU ranks (gloo, world size 2 and 4): token shards -> head shards -> token shards.

The attention between the two all-to-alls is stood in for by a per-head function of the whole sequence (the cumulative
sum over tokens of each channel), which is wrong unless every rank really holds all S tokens of exactly its heads."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from sycl_minimax_h3_b200 import ulysses


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, S, H, D, q):
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
        dist.init_process_group("gloo", rank=rank, world_size=world)
        g = torch.Generator().manual_seed(0)
        full = torch.randn(S, 3 * H * D, generator=g)            # every rank makes the same full input
        s = S // world
        shard = full[rank * s:(rank + 1) * s].contiguous()
        heads = ulysses.seq_to_heads(shard, H, D)
        assert torch.equal(heads, ulysses.head_slice(full, rank, world, H, D)), "forward all-to-all"
        h = H // world
        # a per-head "attention" over all tokens: cumulative sum of v over the sequence
        v = heads.view(S, 3, h * D)[:, 2]
        out_heads = torch.cumsum(v, dim=0)
        back = ulysses.heads_to_seq(out_heads, H, D)
        want = torch.cumsum(full.view(S, 3, H * D)[:, 2], dim=0)[rank * s:(rank + 1) * s]
        assert torch.allclose(back, want), "inverse all-to-all"
        dist.destroy_process_group()
        q.put((rank, "ok"))
    except Exception as e:  # reported to the parent
        q.put((rank, repr(e)))


@pytest.mark.parametrize("world", [2, 4])
def test_ulysses_round_trip_gloo(world):
    S, H, D = 24, 8, 4
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_worker, args=(r, world, port, S, H, D, q)) for r in range(world)]
    for p in ps:
        p.start()
    res = dict(q.get(timeout=120) for _ in ps)
    for p in ps:
        p.join(timeout=60)
    assert all(v == "ok" for v in res.values()), res


def test_heads_must_split():
    class G:  # a stand-in group of 3 ranks for the argument check
        pass

    import unittest.mock as um

    with um.patch.object(dist, "get_world_size", return_value=3):
        with pytest.raises(ValueError, match="do not split"):
            ulysses.seq_to_heads(torch.zeros(4, 3 * 8 * 2), 8, 2, group=G())
