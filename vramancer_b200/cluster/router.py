"""Data-parallel serving: one worker process per GPU behind one request queue, and a
gateway that spreads whole requests over several `vramancer serve` nodes.

`ClusterRouter` spawns workers (each pins one GPU through CUDA_VISIBLE_DEVICES and
loads its own InferencePipeline), sends each request to the live worker with the
fewest outstanding requests over that worker's pipe, demultiplexes results by request
id in a collector thread and restarts workers that die (the requests a dead worker
held go to the others again, once by default).  `Gateway` forwards to the
least-loaded healthy node of a node list (health loop on /health, load from
/api/queue/status).

Reference parity: core/cluster_router.py:42-309 (ClusterRouter, _worker_main,
monitor auto-restart, serve_cluster), core/cluster_gateway.py:21-171.
"""
from __future__ import annotations

import json
import multiprocessing as mp
import os
import queue
import threading
import time
import urllib.request
import uuid
from concurrent.futures import Future
from typing import Dict, List, Optional, Sequence


def _worker_main(slot: int, gpu: Optional[int], model: str, load_kw: Dict, conn) -> None:
    if gpu is not None:
        os.environ["CUDA_VISIBLE_DEVICES"] = str(gpu)
    from ..pipeline import InferencePipeline
    pipe = InferencePipeline(enable_metrics=False).load(model, **load_kw)
    conn.send(("ready", slot))
    while True:
        try:
            item = conn.recv()
        except (EOFError, OSError):
            break
        if item is None:
            break
        rid, prompt, kw = item
        try:
            text = pipe.generate(prompt, **kw)
            conn.send(("done", rid, True, text))
        except Exception as e:  # noqa: BLE001
            conn.send(("done", rid, False, repr(e)))
    pipe.shutdown()


class ClusterRouter:
    """Worker processes with one duplex pipe each.  A shared multiprocessing queue is
    not used on purpose: a worker killed while it blocks in get() keeps the queue's
    reader lock and every other worker stalls behind it; a pipe only affects its own
    worker (EOF).  Requests go to the live worker with the fewest assigned requests;
    the requests assigned to a worker that dies go to the others again (up to
    max_retries times each, then their futures fail)."""

    def __init__(self, model: str, gpus: Sequence[Optional[int]], load_kw: Optional[Dict] = None,
                 start_method: str = "spawn", monitor_interval_s: float = 2.0, max_retries: int = 1):
        self.model = model
        self.gpus = list(gpus)
        self.load_kw = load_kw or {}
        self.ctx = mp.get_context(start_method)
        self.procs: Dict[int, mp.Process] = {}
        self.conns: Dict[int, object] = {}
        self.ready_slots: set = set()
        self.pending: Dict[str, Future] = {}
        self.requests: Dict[str, list] = {}     # rid -> [prompt, kw, attempts]
        self.assigned: Dict[int, List[str]] = {i: [] for i in range(len(self.gpus))}
        self.backlog: List[str] = []            # requests waiting for a live worker
        self.served: Dict[int, int] = {i: 0 for i in range(len(self.gpus))}
        self.restarts = 0
        self.resubmitted = 0
        self.max_retries = max_retries
        self._stop = threading.Event()
        self._lock = threading.RLock()
        self.monitor_interval = monitor_interval_s

    # kept for code that looks at the request a worker is on
    @property
    def inflight(self) -> Dict[int, str]:
        with self._lock:
            return {s: rids[0] for s, rids in self.assigned.items() if rids}

    def _spawn(self, slot: int) -> None:
        parent, child = self.ctx.Pipe(duplex=True)
        p = self.ctx.Process(target=_worker_main, args=(slot, self.gpus[slot], self.model, self.load_kw, child),
                             daemon=True)
        p.start()
        child.close()
        with self._lock:
            self.procs[slot] = p
            self.conns[slot] = parent
            self.ready_slots.discard(slot)

    def start(self, wait_ready: bool = True, timeout: float = 600.0) -> "ClusterRouter":
        for i in range(len(self.gpus)):
            self._spawn(i)
        threading.Thread(target=self._collect, name="vrm-cluster-collect", daemon=True).start()
        threading.Thread(target=self._monitor, name="vrm-cluster-monitor", daemon=True).start()
        if wait_ready:
            t0 = time.time()
            while len(self.ready_slots) < len(self.gpus):
                if time.time() - t0 > timeout:
                    raise TimeoutError("cluster workers did not come up")
                time.sleep(0.05)
        return self

    def _dispatch(self, rid: str) -> None:
        """Sends a request to the live, ready worker with the fewest assigned requests
        (or parks it until one is ready).  Caller holds the lock."""
        live = [s for s in self.ready_slots if self.procs.get(s) is not None and self.procs[s].is_alive()]
        if not live:
            self.backlog.append(rid)
            return
        slot = min(live, key=lambda s: len(self.assigned[s]))
        prompt, kw, _ = self.requests[rid]
        try:
            self.conns[slot].send((rid, prompt, kw))
            self.assigned[slot].append(rid)
        except (OSError, EOFError, BrokenPipeError):
            self.backlog.append(rid)             # the monitor restarts that worker

    def _collect(self) -> None:
        from multiprocessing.connection import wait
        while not self._stop.is_set():
            with self._lock:
                conns = {c: s for s, c in self.conns.items()}
            if not conns:
                time.sleep(0.05)
                continue
            for c in wait(list(conns), timeout=0.2):
                slot = conns[c]
                try:
                    msg = c.recv()
                except (EOFError, OSError):
                    with self._lock:
                        if self.conns.get(slot) is c:
                            self.ready_slots.discard(slot)
                    continue
                if msg[0] == "ready":
                    with self._lock:
                        self.ready_slots.add(slot)
                        parked, self.backlog = self.backlog, []
                        for rid in parked:
                            self._dispatch(rid)
                    continue
                _, rid, ok, payload = msg
                with self._lock:
                    if rid in self.assigned[slot]:
                        self.assigned[slot].remove(rid)
                    fut = self.pending.pop(rid, None)
                    self.requests.pop(rid, None)
                    self.served[slot] = self.served.get(slot, 0) + 1
                if fut is not None:
                    fut.set_result(payload) if ok else fut.set_exception(RuntimeError(payload))

    def _monitor(self) -> None:
        while not self._stop.wait(self.monitor_interval):
            self._check_workers()

    def _check_workers(self) -> None:
        """Restarts dead workers and sends the requests they held elsewhere."""
        for slot, p in list(self.procs.items()):
            if p.is_alive():
                continue
            self.restarts += 1
            with self._lock:
                self.ready_slots.discard(slot)
                held, self.assigned[slot] = self.assigned[slot], []
                old = self.conns.pop(slot, None)
                for rid in held:
                    req = self.requests.get(rid)
                    if req is None:
                        continue
                    req[2] += 1
                    if req[2] > self.max_retries:
                        self.requests.pop(rid, None)
                        fut = self.pending.pop(rid, None)
                        if fut is not None:
                            fut.set_exception(RuntimeError(f"worker {slot} died while serving the request"))
                        continue
                    self.resubmitted += 1
                    self._dispatch(rid)
            if old is not None:
                try:
                    old.close()
                except OSError:
                    pass
            self._spawn(slot)

    def submit(self, prompt: str, **kw) -> Future:
        rid = uuid.uuid4().hex
        fut: Future = Future()
        with self._lock:
            self.pending[rid] = fut
            self.requests[rid] = [prompt, kw, 0]
            self._dispatch(rid)
        return fut

    def stats(self) -> Dict:
        return {"workers": len(self.procs), "alive": sum(p.is_alive() for p in self.procs.values()),
                "served": dict(self.served), "pending": len(self.pending), "restarts": self.restarts,
                "resubmitted": self.resubmitted}

    def stop(self) -> None:
        self._stop.set()
        with self._lock:
            for c in self.conns.values():
                try:
                    c.send(None)
                except (OSError, EOFError, BrokenPipeError):
                    pass
        for p in self.procs.values():
            p.join(timeout=10)
            if p.is_alive():
                p.terminate()


class Gateway:
    """Least-loaded routing of whole requests over HTTP nodes."""

    def __init__(self, nodes: Sequence[str], timeout: float = 600.0):
        self.nodes = list(nodes)
        self.timeout = timeout
        self.health: Dict[str, bool] = {n: True for n in self.nodes}
        self.load: Dict[str, int] = {n: 0 for n in self.nodes}

    def check(self) -> Dict[str, bool]:
        for n in self.nodes:
            try:
                with urllib.request.urlopen(n.rstrip("/") + "/health", timeout=2) as r:
                    self.health[n] = json.loads(r.read()).get("status") in ("ok", "degraded")
                with urllib.request.urlopen(n.rstrip("/") + "/api/queue/status", timeout=2) as r:
                    q = json.loads(r.read())
                    self.load[n] = int(q.get("in_flight", 0)) + int(q.get("waiting", 0))
            except Exception:
                self.health[n] = False
        return dict(self.health)

    def pick(self) -> str:
        live = [n for n in self.nodes if self.health.get(n)]
        if not live:
            raise RuntimeError("no healthy node")
        return min(live, key=lambda n: self.load.get(n, 0))

    def forward(self, path: str, body: Dict, headers: Optional[Dict] = None) -> Dict:
        node = self.pick()
        self.load[node] = self.load.get(node, 0) + 1
        try:
            req = urllib.request.Request(node.rstrip("/") + path, data=json.dumps(body).encode(),
                                         headers={"Content-Type": "application/json", **(headers or {})})
            with urllib.request.urlopen(req, timeout=self.timeout) as r:
                return json.loads(r.read())
        finally:
            self.load[node] = max(0, self.load[node] - 1)
