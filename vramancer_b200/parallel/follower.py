"""Non-zero ranks of a tensor-parallel server: run the engine in lockstep with rank 0.

Rank 0 owns the HTTP front end; at every scheduler step it broadcasts the new
requests and aborts (a CPU gloo group carries the small control messages) and all
ranks then call `engine.step()` with identical state, so their collectives line up.
"""
from __future__ import annotations

import pickle

import torch
import torch.distributed as dist


class StepBroadcaster:
    """Per-step control message from rank 0.  The common case (no new request, no
    abort) costs one 8-byte broadcast on the gloo group; events are pickled and sent as
    a byte tensor only in steps that have some."""

    STOP = -1

    def __init__(self):
        self.group = dist.new_group(backend="gloo") if dist.is_initialized() else None

    def exchange(self, msgs):
        if self.group is None:
            return msgs
        n = torch.zeros(1, dtype=torch.int64)
        payload = None
        if dist.get_rank() == 0:
            if msgs == "stop":
                n[0] = self.STOP
            elif msgs:
                payload = torch.frombuffer(bytearray(pickle.dumps(msgs)), dtype=torch.uint8)
                n[0] = payload.numel()
        dist.broadcast(n, src=0, group=self.group)
        size = int(n[0])
        if size == self.STOP:
            return "stop"
        if size == 0:
            return None
        if payload is None:
            payload = torch.empty(size, dtype=torch.uint8)
        dist.broadcast(payload, src=0, group=self.group)
        return pickle.loads(payload.numpy().tobytes())


def follow(pipe) -> int:
    """Follower loop: apply rank 0's request events, then step."""
    from ..engine.engine import SamplingParams
    bc = StepBroadcaster()
    pipe._stop.set()                      # followers do not run their own loop thread
    eng = pipe.engine
    while True:
        msgs = bc.exchange(None)
        if msgs == "stop":
            break
        for kind, payload in msgs or []:
            if kind == "add":
                ids, params, rid = payload
                eng.add_request(ids, SamplingParams(**params), request_id=rid)
            elif kind == "abort":
                eng.abort(payload)
        if eng.has_unfinished():
            eng.step()
    return 0
