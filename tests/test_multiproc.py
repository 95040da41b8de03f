"""Multi-process host logic on CPU (gloo, world size 2): row sharding, gathering the
shards, and detecting a lost rank between steps.  The per-shard compute here is the
oracle (CPU); on GPUs each rank calls the same library operator on its shard."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from icpp_tuning_b200.shard import PeerLost, StepGuard, gather_rows, row_shard, sharded_apply


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _init(rank, world, port):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=__import__("datetime").timedelta(seconds=30))


def _worker_gather(rank, world, port, M, q):
    try:
        _init(rank, world, port)
        from oracle import ref_ops as R
        g = torch.Generator().manual_seed(5)
        a = torch.randn(M, 64, generator=g).bfloat16()
        b = torch.randn(64, 96, generator=g).bfloat16()
        bias = torch.randn(96, generator=g).bfloat16()
        out, lo, hi = sharded_apply(lambda x: R.gemm_bias_act(x, b, bias, "gelu_tanh"), a, world, rank)
        full = gather_rows(out.contiguous(), M)
        into = gather_rows(out.contiguous(), M, out=torch.empty_like(full))  # caller-provided output
        ref = R.gemm_bias_act(a, b, bias, "gelu_tanh")
        q.put((rank, bool(torch.equal(full, ref) and torch.equal(into, ref)), lo, hi))
        dist.destroy_process_group()
    except Exception as e:  # pragma: no cover - reported through the queue
        q.put((rank, repr(e), -1, -1))


@pytest.mark.parametrize("M", [1000, 256, 100])
def test_sharded_gather_equals_full(M):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    ps = [ctx.Process(target=_worker_gather, args=(r, 2, port, M, q)) for r in range(2)]
    for p in ps:
        p.start()
    res = sorted(q.get(timeout=120) for _ in ps)
    for p in ps:
        p.join(60)
    assert [r[1] for r in res] == [True, True], res
    assert res[0][2] == 0 and res[0][3] == res[1][2] and res[1][3] == M


def test_row_shard_tiles():
    for M in (1, 127, 128, 129, 1000, 16384):
        for world in (1, 2, 3, 8):
            spans = [row_shard(M, world, r) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == M
            for (lo, hi), (lo2, _) in zip(spans, spans[1:]):
                assert hi == lo2 and (lo % 128 == 0 or lo == M)
    with pytest.raises(ValueError):
        row_shard(10, 2, 2)


def _worker_guard(rank, world, port, q):
    try:
        _init(rank, world, port)
        guard = StepGuard(dist.distributed_c10d._get_default_store(), world, rank, timeout_s=3.0)
        guard.check_in()  # step 0: everyone present
        if rank == 1:
            q.put((rank, "left"))
            q.close()
            q.join_thread()  # flush the message before leaving
            os._exit(0)  # leaves between steps, nothing in flight
        try:
            guard.check_in()
            q.put((rank, "no error"))
        except PeerLost as e:
            q.put((rank, "PeerLost" if "[1]" in str(e) else repr(e)))
    except Exception as e:  # pragma: no cover
        q.put((rank, repr(e)))


def test_lost_rank_detected_between_steps():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    ps = [ctx.Process(target=_worker_guard, args=(r, 2, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    res = dict(q.get(timeout=120) for _ in ps)
    for p in ps:
        p.join(30)
        if p.is_alive():
            p.kill()
    assert res == {0: "PeerLost", 1: "left"}
