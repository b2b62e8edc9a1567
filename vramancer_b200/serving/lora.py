"""LoRA adapter hot-swap by weight merging.

An adapter is a dict of low-rank pairs (A [r, in], B [out, r], scale alpha / r) per
projection, read from a PEFT-style safetensors file (`...q_proj.lora_A.weight`).
`set_adapter(name)` merges W += scale * B @ A into the served weights (fused qkv and
interleaved gate/up rows included) and `disable()` subtracts it again, so switching
adapters costs one pass over the touched weights and decoding runs at base speed.

Reference parity: core/lora_manager.py:19-76 (PEFT load_adapter / set_adapter /
delete_adapter / disable), InferencePipeline.lora (core/inference_pipeline.py:1175).
"""
from __future__ import annotations

import json
import os
import threading
from typing import Dict, Optional, Tuple

import torch

_TARGETS = {"q_proj": ("qkv_w", "q"), "k_proj": ("qkv_w", "k"), "v_proj": ("qkv_w", "v"),
            "o_proj": ("o_w", None), "gate_proj": ("gate_up_w", "gate"), "up_proj": ("gate_up_w", "up"),
            "down_proj": ("down_w", None)}


class LoRAManager:
    def __init__(self, llm):
        self.llm = llm
        self.adapters: Dict[str, Dict[Tuple[int, str], Tuple[torch.Tensor, torch.Tensor, float]]] = {}
        self.active: Optional[str] = None
        self._lock = threading.Lock()

    @property
    def weights(self):
        return getattr(self.llm, "weights", None)

    def load_adapter(self, name: str, path_or_tensors, alpha: Optional[float] = None) -> int:
        """Registers an adapter from a directory/file (PEFT naming) or a ready dict
        {(layer, proj): (A, B)}; returns the number of projections it touches."""
        pairs: Dict[Tuple[int, str], Tuple[torch.Tensor, torch.Tensor, float]] = {}
        if isinstance(path_or_tensors, dict):
            for (layer, proj), (A, B) in path_or_tensors.items():
                r = A.shape[0]
                pairs[(layer, proj)] = (A, B, (alpha or r) / r)
        else:
            from safetensors.torch import load_file
            path = path_or_tensors
            f = os.path.join(path, "adapter_model.safetensors") if os.path.isdir(path) else path
            cfgp = os.path.join(os.path.dirname(f), "adapter_config.json")
            r_cfg, a_cfg = None, alpha
            if os.path.exists(cfgp):
                c = json.load(open(cfgp))
                r_cfg, a_cfg = c.get("r"), a_cfg or c.get("lora_alpha")
            t = load_file(f)
            tmp: Dict[Tuple[int, str], Dict[str, torch.Tensor]] = {}
            for k, v in t.items():
                parts = k.split(".")
                if "layers" not in parts:
                    continue
                layer = int(parts[parts.index("layers") + 1])
                proj = next((p for p in parts if p in _TARGETS), None)
                if proj is None:
                    continue
                which = "A" if "lora_A" in k else "B" if "lora_B" in k else None
                if which:
                    tmp.setdefault((layer, proj), {})[which] = v
            for key, d in tmp.items():
                if "A" in d and "B" in d:
                    r = r_cfg or d["A"].shape[0]
                    pairs[key] = (d["A"], d["B"], (a_cfg or r) / r)
        with self._lock:
            self.adapters[name] = pairs
        return len(pairs)

    def _apply(self, name: str, sign: float) -> None:
        w = self.weights
        if w is None:
            raise RuntimeError("LoRA merging needs a single-device model with resident weights")
        cfg = self.llm.cfg
        for (layer, proj), (A, B, scale) in self.adapters[name].items():
            key, part = _TARGETS[proj]
            W = w.get(f"layers.{layer}.{key}")
            if W is None:
                continue
            delta = (B.float() @ A.float()) * (scale * sign)
            delta = delta.to(W.device)
            nw = getattr(W, "_vrm_norm_w", None)
            if nw is not None:
                # W carries its input RMSNorm weight in its columns (folded norms)
                delta = delta * nw.float().view(1, -1)
            if key == "qkv_w":
                off = {"q": 0, "k": cfg.q_size, "v": cfg.q_size + cfg.kv_size}[part]
                rows = W[off:off + delta.shape[0]]
            elif key == "gate_up_w":
                rows = W[0::2] if part == "gate" else W[1::2]
                new = (rows.float() + delta).to(W.dtype)
                if part == "gate":
                    W[0::2] = new
                else:
                    W[1::2] = new
                continue
            else:
                rows = W
            rows.copy_((rows.float() + delta).to(W.dtype))

    def set_adapter(self, name: str) -> None:
        with self._lock:
            if name not in self.adapters:
                raise KeyError(name)
            if self.active == name:
                return
            if self.active is not None:
                self._apply(self.active, -1.0)
            self._apply(name, 1.0)
            self.active = name

    def disable(self) -> None:
        with self._lock:
            if self.active is not None:
                self._apply(self.active, -1.0)
                self.active = None

    def delete_adapter(self, name: str) -> None:
        if self.active == name:
            self.disable()
        with self._lock:
            self.adapters.pop(name, None)

    def list_adapters(self):
        return {"adapters": sorted(self.adapters), "active": self.active}
