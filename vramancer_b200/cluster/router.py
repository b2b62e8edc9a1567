"""Data-parallel serving: one worker process per GPU behind one request queue, and a
gateway that spreads whole requests over several `vramancer serve` nodes.

`ClusterRouter` spawns workers (each pins one GPU through CUDA_VISIBLE_DEVICES and
loads its own InferencePipeline), feeds them from a shared queue (work stealing: an
idle worker takes the next request), demultiplexes results by request id in a
collector thread and restarts workers that die.  `Gateway` forwards to the
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


def _worker_main(gpu: Optional[int], model: str, load_kw: Dict, inq, outq, ready) -> None:
    if gpu is not None:
        os.environ["CUDA_VISIBLE_DEVICES"] = str(gpu)
    from ..pipeline import InferencePipeline
    pipe = InferencePipeline(enable_metrics=False).load(model, **load_kw)
    ready.put(gpu)
    while True:
        item = inq.get()
        if item is None:
            break
        rid, prompt, kw = item
        try:
            text = pipe.generate(prompt, **kw)
            outq.put((rid, True, text, gpu))
        except Exception as e:  # noqa: BLE001
            outq.put((rid, False, repr(e), gpu))
    pipe.shutdown()


class ClusterRouter:
    def __init__(self, model: str, gpus: Sequence[Optional[int]], load_kw: Optional[Dict] = None,
                 start_method: str = "spawn", monitor_interval_s: float = 2.0):
        self.model = model
        self.gpus = list(gpus)
        self.load_kw = load_kw or {}
        self.ctx = mp.get_context(start_method)
        self.inq = self.ctx.Queue()
        self.outq = self.ctx.Queue()
        self.ready = self.ctx.Queue()
        self.procs: Dict[int, mp.Process] = {}
        self.pending: Dict[str, Future] = {}
        self.served: Dict[Optional[int], int] = {g: 0 for g in self.gpus}
        self.restarts = 0
        self._stop = threading.Event()
        self._lock = threading.Lock()
        self.monitor_interval = monitor_interval_s

    def _spawn(self, slot: int) -> None:
        p = self.ctx.Process(target=_worker_main, args=(self.gpus[slot], self.model, self.load_kw, self.inq,
                                                        self.outq, self.ready), daemon=True)
        p.start()
        self.procs[slot] = p

    def start(self, wait_ready: bool = True, timeout: float = 600.0) -> "ClusterRouter":
        for i in range(len(self.gpus)):
            self._spawn(i)
        if wait_ready:
            for _ in self.gpus:
                self.ready.get(timeout=timeout)
        threading.Thread(target=self._collect, name="vrm-cluster-collect", daemon=True).start()
        threading.Thread(target=self._monitor, name="vrm-cluster-monitor", daemon=True).start()
        return self

    def _collect(self) -> None:
        while not self._stop.is_set():
            try:
                rid, ok, payload, gpu = self.outq.get(timeout=0.2)
            except queue.Empty:
                continue
            with self._lock:
                fut = self.pending.pop(rid, None)
                self.served[gpu] = self.served.get(gpu, 0) + 1
            if fut is not None:
                fut.set_result(payload) if ok else fut.set_exception(RuntimeError(payload))

    def _monitor(self) -> None:
        while not self._stop.wait(self.monitor_interval):
            for slot, p in list(self.procs.items()):
                if not p.is_alive():
                    self.restarts += 1
                    self._spawn(slot)

    def submit(self, prompt: str, **kw) -> Future:
        rid = uuid.uuid4().hex
        fut: Future = Future()
        with self._lock:
            self.pending[rid] = fut
        self.inq.put((rid, prompt, kw))
        return fut

    def stats(self) -> Dict:
        return {"workers": len(self.procs), "alive": sum(p.is_alive() for p in self.procs.values()),
                "served": dict(self.served), "pending": len(self.pending), "restarts": self.restarts}

    def stop(self) -> None:
        self._stop.set()
        for _ in self.procs:
            self.inq.put(None)
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
