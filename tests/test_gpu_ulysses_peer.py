"""The Ulysses exchange over peer memory (h3s_ulysses_push_qkv / _out through CUDA IPC) on 2, 4 and 8 GPUs of one node,
and the attention with the inverse exchange in its epilogue (h3s_attention_ulysses, both the Sage and the fp16 path):
the same bits as the token <-> head re-sharding it replaces (ulysses.head_slice, and the inverse), for half,
bfloat16 and float32 rows, with 16-byte vectors and with element copies (a head of 12 features is 24 bytes).
Skipped with fewer GPUs than ranks (the round-end single-GPU run)."""
import os
import queue
import socket
import time

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, report):
    try:
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
        torch.cuda.set_device(rank)
        import datetime

        dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", rank))
        from sycl_minimax_h3_b200 import ulysses

        for S, H, D, dtype in ((1024, 8, 128, torch.float16), (512, 8, 12, torch.bfloat16), (256, 4, 64, torch.float32),
                               (4096 * world, 32, 128, torch.float16), (8192 * world, 8, 128, torch.float16),
                               (640 * world, 8, 64, torch.bfloat16)):
            if H % world:
                continue                                                        # fewer heads than ranks
            g = torch.Generator(device="cuda")
            g.manual_seed(S + H + D)
            # every rank makes the same input (the same seeded generator on every GPU)
            full = torch.randn(S, 3 * H * D, generator=g, device="cuda").to(dtype)
            s = S // world
            ex = ulysses.PeerExchange(s, H, D, dtype)
            for step in range(2):                                               # the buffers are reused
                shard = (full[rank * s:(rank + 1) * s] + step).contiguous()
                heads = ex.seq_to_heads(shard)
                want = ulysses.head_slice(full + step, rank, world, H, D)
                assert torch.equal(heads.view(torch.int16 if dtype != torch.float32 else torch.int32),
                                   want.view(torch.int16 if dtype != torch.float32 else torch.int32)), "forward"
                h = H // world
                out_heads = heads[:, 2 * h * D:].contiguous()                   # v of this rank's heads, all tokens
                back = ex.heads_to_seq(out_heads)
                want_b = (full + step)[rank * s:(rank + 1) * s, 2 * H * D:]
                assert torch.equal(back.float(), want_b.float()), "inverse"
            if D in (64, 128) and dtype != torch.float32:
                # the attention with the exchange in its epilogue: the same bits as the attention on this rank's
                # heads followed by the inverse push
                from sycl_minimax_h3_b200 import ops

                heads = ex.seq_to_heads(full[rank * s:(rank + 1) * s].contiguous())
                h = H // world
                out_heads = torch.empty(S, h * D, dtype=dtype, device="cuda")
                q, k, v = ops.Rows.qkv(heads, h, D)
                ops.attention(q, k, v, out_heads)
                want = ex.heads_to_seq(out_heads).clone()
                # NaN in every rank's shard first: each row the comparison sees must have been stored over CUDA IPC by
                # the epilogue of the rank that owns its heads (attention_to_seq meets before any epilogue stores)
                ex.out.fill_(float("nan"))
                got = ex.attention_to_seq(heads)
                ex.check()
                assert torch.equal(got.view(torch.int16), want.view(torch.int16)), "attention with the exchange"
                # twice in a row: the second call's stores wait for every rank to have read the first call's rows
                first = got.clone()
                again = ex.attention_to_seq(heads)
                ex.check()
                assert torch.equal(again.view(torch.int16), first.view(torch.int16)), "second attention"
            ex.close()
        dist.destroy_process_group()
        report.put((rank, "ok"))
    except Exception as e:  # reported to the parent
        report.put((rank, repr(e)))


@pytest.mark.parametrize("world", [2, 4, 8])
def test_peer_exchange(world):
    if torch.cuda.device_count() < world:
        pytest.skip(f"needs {world} GPUs")
    ctx = mp.get_context("spawn")
    report = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_worker, args=(r, world, port, report)) for r in range(world)]
    for p in ps:
        p.start()
    res = {}
    deadline = time.monotonic() + 300
    while len(res) < world and time.monotonic() < deadline:
        try:
            r, v = report.get(timeout=5)
            res[r] = v
        except queue.Empty:
            # a worker that ended without reporting fails the test now, not at the deadline
            dead = [i for i, p in enumerate(ps) if p.exitcode is not None and i not in res]
            if dead:
                break
    for p in ps:
        p.join(timeout=60)
    assert len(res) == world and all(v == "ok" for v in res.values()), res
