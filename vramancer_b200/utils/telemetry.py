"""Compact binary node telemetry (24 bytes per sample) for cluster heartbeats.

Layout (little-endian): u16 node_id | u8 gpu_util (0-255 = 0-100%) | u8 temp_c |
f32 vram_used_gb | f32 vram_total_gb | f32 tok_s | u16 power_w | u16 flags | u32 ts_s.

Reference parity: core/telemetry.py (24-byte binary node telemetry).
"""
from __future__ import annotations

import socket
import struct
import time
from dataclasses import dataclass, field

_FMT = "<HBBfffHHI"
SIZE = struct.calcsize(_FMT)
assert SIZE == 24


@dataclass
class NodeTelemetry:
    node_id: int
    gpu_util: float = 0.0
    vram_used_gb: float = 0.0
    vram_total_gb: float = 0.0
    tok_s: float = 0.0
    temp_c: int = 0
    power_w: int = 0
    flags: int = 0
    ts: int = field(default_factory=lambda: int(time.time()))

    def pack(self) -> bytes:
        return struct.pack(_FMT, self.node_id & 0xFFFF, max(0, min(255, int(round(self.gpu_util * 255)))),
                           max(0, min(255, int(self.temp_c))), self.vram_used_gb, self.vram_total_gb, self.tok_s,
                           max(0, min(65535, int(self.power_w))), self.flags & 0xFFFF, self.ts & 0xFFFFFFFF)

    @classmethod
    def unpack(cls, raw: bytes) -> "NodeTelemetry":
        nid, util, temp, used, total, toks, pw, flags, ts = struct.unpack(_FMT, raw[:SIZE])
        return cls(nid, util / 255.0, used, total, toks, temp, pw, flags, ts)


def send(sample: NodeTelemetry, host: str = "127.0.0.1", port: int = 9109) -> None:
    with socket.socket(socket.AF_INET, socket.SOCK_DGRAM) as s:
        s.sendto(sample.pack(), (host, port))
