"""Non-zero ranks of a tensor-parallel server: run the engine in lockstep with rank 0.

Rank 0 owns the HTTP front end; at every scheduler step it broadcasts the new
requests and aborts (a CPU gloo group carries the small control messages) and all
ranks then call `engine.step()` with identical state, so their collectives line up.
"""
from __future__ import annotations

import torch.distributed as dist


class StepBroadcaster:
    def __init__(self):
        self.group = dist.new_group(backend="gloo") if dist.is_initialized() else None

    def exchange(self, msgs):
        box = [msgs]
        if self.group is not None:
            dist.broadcast_object_list(box, src=0, group=self.group)
        return box[0]


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
