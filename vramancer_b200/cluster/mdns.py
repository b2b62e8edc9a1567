"""mDNS / DNS-SD discovery of serving nodes (RFC 6762 / 6763), without extra packages.

A node runs an `MDNSResponder` for its service instance `<name>._vramancer._tcp.local.`:
it answers PTR queries for the service type with the instance's PTR, SRV (host,
port), TXT (model, GPUs, URL) and A records, and announces them unsolicited when it
starts.  An `MDNSBrowser` sends the PTR query and registers every answering node in
the discovery table (cluster/discovery.py `register_node`), next to the UDP-broadcast
and static-list sources.

Queries from a port other than 5353 ("legacy unicast", RFC 6762 section 6.7) and
queries with the unicast-response bit get their answer sent back to the sender; others
are answered on the multicast group 224.0.0.251:5353.  Group and port are parameters,
so tests run it on loopback.

Reference parity: experimental/cluster_discovery.py:225-560 (service type
"_vramancer._tcp.local.", zeroconf registration and browsing, mDNS first then UDP
broadcast, heartbeat table).  zeroconf is not installed here; the wire format is
written directly.
"""
from __future__ import annotations

import socket
import struct
import threading
import time
from typing import Dict, List, Optional, Tuple

from .discovery import register_node

SERVICE_TYPE = "_vramancer._tcp.local."
MDNS_GROUP, MDNS_PORT = "224.0.0.251", 5353
T_A, T_PTR, T_TXT, T_SRV = 1, 12, 16, 33
C_IN, C_FLUSH, C_QU = 1, 0x8000, 0x8000


# ---------------------------------------------------------------- wire format
def _name(n: str) -> bytes:
    out = b""
    for label in n.rstrip(".").split("."):
        b = label.encode()
        if not 0 < len(b) < 64:
            raise ValueError(f"bad DNS label in {n!r}")
        out += bytes([len(b)]) + b
    return out + b"\x00"


def _read_name(buf: bytes, off: int) -> Tuple[str, int]:
    labels, jumped, end, hops = [], False, off, 0
    while True:
        if off >= len(buf) or hops > 64:
            raise ValueError("truncated or looping DNS name")
        n = buf[off]
        if n & 0xC0 == 0xC0:                      # compression pointer
            ptr = ((n & 0x3F) << 8) | buf[off + 1]
            if not jumped:
                end = off + 2
            off, jumped, hops = ptr, True, hops + 1
            continue
        if n == 0:
            if not jumped:
                end = off + 1
            return ".".join(labels) + ".", end
        labels.append(buf[off + 1:off + 1 + n].decode(errors="replace"))
        off += 1 + n


def _rr(name: str, rtype: int, rdata: bytes, ttl: int = 120, flush: bool = False) -> bytes:
    cls = C_IN | (C_FLUSH if flush else 0)
    return _name(name) + struct.pack("!HHIH", rtype, cls, ttl, len(rdata)) + rdata


def _txt(d: Dict[str, str]) -> bytes:
    out = b""
    for k, v in d.items():
        e = f"{k}={v}".encode()[:255]
        out += bytes([len(e)]) + e
    return out or b"\x00"


def build_query(name: str = SERVICE_TYPE, qtype: int = T_PTR, unicast: bool = True, qid: int = 0) -> bytes:
    return struct.pack("!HHHHHH", qid, 0, 1, 0, 0, 0) + _name(name) + struct.pack(
        "!HH", qtype, C_IN | (C_QU if unicast else 0))


def parse_message(buf: bytes) -> Dict:
    """Questions and resource records of a DNS message (A, PTR, SRV, TXT decoded)."""
    qid, flags, qd, an, ns, ar = struct.unpack("!HHHHHH", buf[:12])
    off = 12
    qs = []
    for _ in range(qd):
        n, off = _read_name(buf, off)
        qt, qc = struct.unpack("!HH", buf[off:off + 4])
        off += 4
        qs.append((n, qt, qc))
    rrs = []
    for _ in range(an + ns + ar):
        n, off = _read_name(buf, off)
        rt, rc, ttl, rl = struct.unpack("!HHIH", buf[off:off + 10])
        off += 10
        rd = buf[off:off + rl]
        val = rd
        if rt == T_A and rl == 4:
            val = socket.inet_ntoa(rd)
        elif rt == T_PTR:
            val = _read_name(buf, off)[0]
        elif rt == T_SRV:
            pr, w, port = struct.unpack("!HHH", rd[:6])
            val = (pr, w, port, _read_name(buf, off + 6)[0])
        elif rt == T_TXT:
            items, i = {}, 0
            while i < len(rd):
                ln = rd[i]
                s = rd[i + 1:i + 1 + ln].decode(errors="replace")
                if "=" in s:
                    k, v = s.split("=", 1)
                    items[k] = v
                i += 1 + ln
            val = items
        rrs.append((n, rt, rc, ttl, val))
        off += rl
    return {"id": qid, "response": bool(flags & 0x8000), "questions": qs, "records": rrs}


# ---------------------------------------------------------------- responder
class MDNSResponder:
    """Answers DNS-SD queries for one serving node."""

    def __init__(self, instance: str, host_ip: str, port: int, txt: Optional[Dict[str, str]] = None,
                 group: str = MDNS_GROUP, mdns_port: int = MDNS_PORT, bind: str = "0.0.0.0"):
        self.instance = f"{instance}.{SERVICE_TYPE}"
        self.hostname = f"{instance}-host.local."
        self.host_ip, self.port = host_ip, port
        self.txt = {"url": f"http://{host_ip}:{port}", **{k: str(v) for k, v in (txt or {}).items()}}
        self.group, self.mdns_port, self.bind = group, mdns_port, bind
        self.sock: Optional[socket.socket] = None
        self._stop = threading.Event()
        self._thread: Optional[threading.Thread] = None
        self.answered = 0

    def records(self) -> bytes:
        srv = struct.pack("!HHH", 0, 0, self.port) + _name(self.hostname)
        ans = _rr(SERVICE_TYPE, T_PTR, _name(self.instance), ttl=4500)
        extra = (_rr(self.instance, T_SRV, srv, flush=True) + _rr(self.instance, T_TXT, _txt(self.txt), flush=True)
                 + _rr(self.hostname, T_A, socket.inet_aton(self.host_ip), flush=True))
        return struct.pack("!HHHHHH", 0, 0x8400, 0, 1, 0, 3) + ans + extra

    def start(self) -> bool:
        try:
            s = socket.socket(socket.AF_INET, socket.SOCK_DGRAM, socket.IPPROTO_UDP)
            s.setsockopt(socket.SOL_SOCKET, socket.SO_REUSEADDR, 1)
            if hasattr(socket, "SO_REUSEPORT"):
                s.setsockopt(socket.SOL_SOCKET, socket.SO_REUSEPORT, 1)
            s.bind((self.bind, self.mdns_port))
            if self.group.startswith("224."):
                mreq = socket.inet_aton(self.group) + socket.inet_aton("0.0.0.0")
                s.setsockopt(socket.IPPROTO_IP, socket.IP_ADD_MEMBERSHIP, mreq)
                s.setsockopt(socket.IPPROTO_IP, socket.IP_MULTICAST_TTL, 255)
            s.settimeout(0.3)
        except OSError:
            return False
        self.sock = s
        self._thread = threading.Thread(target=self._loop, name="vrm-mdns", daemon=True)
        self._thread.start()
        try:                                        # unsolicited announcement
            s.sendto(self.records(), (self.group, self.mdns_port))
        except OSError:
            pass
        return True

    def _loop(self) -> None:
        while not self._stop.is_set():
            try:
                data, src = self.sock.recvfrom(9000)
                msg = parse_message(data)
            except socket.timeout:
                continue
            except (OSError, ValueError, struct.error):
                continue
            if msg["response"]:
                continue
            for name, qt, qc in msg["questions"]:
                if name.lower() == SERVICE_TYPE.lower() and qt in (T_PTR, 255):
                    reply = bytearray(self.records())
                    reply[0:2] = struct.pack("!H", msg["id"])
                    dest = src if (qc & C_QU or src[1] != MDNS_PORT) else (self.group, self.mdns_port)
                    try:
                        self.sock.sendto(bytes(reply), dest)
                        self.answered += 1
                    except OSError:
                        pass

    def stop(self) -> None:
        self._stop.set()
        if self.sock:
            self.sock.close()


# ---------------------------------------------------------------- browser
def browse(timeout: float = 1.0, group: str = MDNS_GROUP, mdns_port: int = MDNS_PORT,
           register: bool = True) -> List[Dict]:
    """Sends one DNS-SD query for the service and collects the answers for `timeout`
    seconds; every node found goes into the discovery table (discovery="mdns")."""
    s = socket.socket(socket.AF_INET, socket.SOCK_DGRAM, socket.IPPROTO_UDP)
    s.bind(("0.0.0.0", 0))
    s.settimeout(0.1)
    found: Dict[str, Dict] = {}
    try:
        s.sendto(build_query(unicast=True, qid=0x5652), (group, mdns_port))
        t_end = time.time() + timeout
        while time.time() < t_end:
            try:
                data, src = s.recvfrom(9000)
                msg = parse_message(data)
            except socket.timeout:
                continue
            except (ValueError, struct.error):
                continue
            if not msg["response"]:
                continue
            srv, txt, addr = {}, {}, {}
            instances = []
            for name, rt, _, _, val in msg["records"]:
                if rt == T_PTR and name.lower() == SERVICE_TYPE.lower():
                    instances.append(val)
                elif rt == T_SRV:
                    srv[name] = val
                elif rt == T_TXT:
                    txt[name] = val
                elif rt == T_A:
                    addr[name] = val
            for inst in instances:
                info = dict(txt.get(inst, {}))
                if inst in srv:
                    _, _, port, target = srv[inst]
                    ip = addr.get(target, src[0])
                    info.setdefault("url", f"http://{ip}:{port}")
                info["instance"] = inst
                info["discovery"] = "mdns"
                if "url" in info:
                    found[info["url"]] = info
    finally:
        s.close()
    if register:
        for url, info in found.items():
            register_node(url, info)
    return list(found.values())
