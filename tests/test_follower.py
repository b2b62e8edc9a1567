"""Lockstep control messages of tensor / pipeline parallel serving (gloo, 2 CPU ranks)."""
import os
import socket

import torch.multiprocessing as mp


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _rank(rank, port, q):
    import torch.distributed as dist

    from vramancer_b200.parallel.follower import StepBroadcaster
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=2)
    bc = StepBroadcaster()
    sent = [None, [], [("add", ([1, 2, 3], {"max_tokens": 4}, "r1")), ("abort", "r0")], [], "stop"]
    got = [bc.exchange(m if rank == 0 else None) for m in sent]
    if rank == 1:
        q.put(got)
    dist.destroy_process_group()


def test_step_broadcaster_sends_events_only_when_there_are_some():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    ps = [ctx.Process(target=_rank, args=(r, port, q)) for r in range(2)]
    for p in ps:
        p.start()
    got = q.get(timeout=120)
    for p in ps:
        p.join(60)
        assert p.exitcode == 0
    assert got == [None, None, [("add", ([1, 2, 3], {"max_tokens": 4}, "r1")), ("abort", "r0")], None, "stop"]
