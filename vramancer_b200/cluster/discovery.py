"""Node discovery: UDP broadcast announcements, a static node list, heartbeats.

Each `vramancer serve` node can `announce()` itself (JSON datagram with host, port,
model, GPU count) on the discovery port; `ClusterDiscovery` listens, keeps a table of
nodes with last-seen times and drops nodes whose heartbeat is older than `ttl_s`.
VRM_NODES (comma-separated URLs) adds static nodes, and cluster/mdns.py finds nodes
by mDNS / DNS-SD (service "_vramancer._tcp.local.") into the same table.

Reference parity: experimental/cluster_discovery.py:225-1016 (mDNS + UDP broadcast +
static list, heartbeat), core/cluster_gateway.py discovery hook.
"""
from __future__ import annotations

import json
import os
import socket
import threading
import time
from typing import Dict, List, Optional

_nodes: Dict[str, Dict] = {}
_lock = threading.Lock()


def register_node(url: str, info: Optional[Dict] = None) -> None:
    with _lock:
        d = _nodes.setdefault(url, {"url": url})
        d.update(info or {})
        d["last_seen"] = time.time()


def known_nodes(ttl_s: float = 30.0) -> List[Dict]:
    now = time.time()
    static = [u.strip() for u in os.environ.get("VRM_NODES", "").split(",") if u.strip()]
    with _lock:
        for u in static:
            _nodes.setdefault(u, {"url": u, "static": True, "last_seen": now})
        for u in [u for u, d in _nodes.items() if not d.get("static") and now - d["last_seen"] > ttl_s]:
            del _nodes[u]
        return [dict(d) for d in _nodes.values()]


def announce(host: str, port: int, info: Optional[Dict] = None, discovery_port: int = 5353,
             broadcast_addr: str = "255.255.255.255") -> bool:
    msg = json.dumps({"vramancer": 1, "url": f"http://{host}:{port}", **(info or {})}).encode()
    try:
        s = socket.socket(socket.AF_INET, socket.SOCK_DGRAM)
        s.setsockopt(socket.SOL_SOCKET, socket.SO_BROADCAST, 1)
        s.sendto(msg, (broadcast_addr, discovery_port))
        s.close()
        return True
    except OSError:
        return False


class ClusterDiscovery:
    def __init__(self, port: int = 5353, bind: str = "0.0.0.0"):
        self.port, self.bind = port, bind
        self._stop = threading.Event()
        self._thread: Optional[threading.Thread] = None
        self.sock: Optional[socket.socket] = None

    def start(self) -> bool:
        try:
            self.sock = socket.socket(socket.AF_INET, socket.SOCK_DGRAM)
            self.sock.setsockopt(socket.SOL_SOCKET, socket.SO_REUSEADDR, 1)
            self.sock.bind((self.bind, self.port))
            self.sock.settimeout(0.5)
        except OSError:
            return False
        self._thread = threading.Thread(target=self._loop, name="vrm-discovery", daemon=True)
        self._thread.start()
        return True

    def _loop(self):
        while not self._stop.is_set():
            try:
                data, _ = self.sock.recvfrom(65536)
                d = json.loads(data.decode())
                if d.get("vramancer") and d.get("url"):
                    register_node(d["url"], d)
            except socket.timeout:
                continue
            except Exception:
                continue

    def stop(self):
        self._stop.set()
        if self.sock:
            self.sock.close()
