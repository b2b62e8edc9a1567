"""Data-parallel cluster router with CPU worker processes: requests spread over the
workers, every future resolves with the single-model text, and when a worker process
dies mid-request (killed on the host) it is restarted and its request is served again."""
import os
import signal
import time

from vramancer_b200.cluster.router import ClusterRouter, Gateway
from vramancer_b200.pipeline import InferencePipeline

KW = {"device": "cpu", "max_model_len": 128, "kv_pages": 32, "max_batch": 4}


def test_router_serves_and_survives_a_dead_worker():
    ref = InferencePipeline(enable_metrics=False).load("tiny-qwen2", **KW)
    prompts = [f"prompt number {i}" for i in range(6)]
    want = [ref.generate(p, max_new_tokens=8) for p in prompts]
    long_want = ref.generate("a long one", max_new_tokens=20)
    ref.shutdown()

    router = ClusterRouter("tiny-qwen2", [None, None], load_kw=KW, monitor_interval_s=0.2).start(timeout=300)
    try:
        futs = [router.submit(p, max_new_tokens=8) for p in prompts]
        assert [f.result(timeout=120) for f in futs] == want
        st = router.stats()
        assert st["alive"] == 2 and sum(st["served"].values()) == 6

        # a worker killed on the host is restarted and the router keeps serving
        os.kill(router.procs[0].pid, signal.SIGKILL)
        t0 = time.time()
        while router.stats()["restarts"] < 1 and time.time() - t0 < 60:
            time.sleep(0.05)
        assert router.submit("a long one", max_new_tokens=20).result(timeout=300) == long_want
    finally:
        router.stop()


class _Proc:
    def __init__(self, alive):
        self.alive = alive
        self.pid = 0

    def is_alive(self):
        return self.alive


class _Conn:
    def __init__(self):
        self.sent = []

    def send(self, m):
        self.sent.append(m)

    def close(self):
        pass


def test_dead_worker_requests_go_to_the_others_then_fail():
    """Resubmission logic on fake worker handles: the requests a dead worker held are
    sent to a live worker once; when that one dies too, their futures fail."""
    from concurrent.futures import Future
    router = ClusterRouter("tiny-qwen2", [None, None], max_retries=1)
    router._spawn = lambda slot: router.procs.__setitem__(slot, _Proc(False))   # stays down
    router.procs = {0: _Proc(False), 1: _Proc(True)}
    router.conns = {0: _Conn(), 1: _Conn()}
    router.ready_slots = {0, 1}
    fut = Future()
    router.pending["r1"] = fut
    router.requests["r1"] = ["hello", {"max_new_tokens": 4}, 0]
    router.assigned[0] = ["r1"]
    router._check_workers()
    assert router.resubmitted == 1 and not fut.done()
    assert router.conns[1].sent == [("r1", "hello", {"max_new_tokens": 4})] and router.assigned[1] == ["r1"]
    router.procs[1].alive = False
    router._check_workers()
    assert fut.done() and isinstance(fut.exception(), RuntimeError)
    assert "r1" not in router.pending and router.restarts == 3


def test_gateway_skips_unreachable_nodes():
    gw = Gateway(["http://127.0.0.1:9", "http://127.0.0.1:1"], timeout=1.0)
    health = gw.check()
    assert health == {"http://127.0.0.1:9": False, "http://127.0.0.1:1": False}
