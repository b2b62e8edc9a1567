"""Drop-in acceleration for HuggingFace code: `vramancer_b200.patch()`.

After `patch()`, `AutoModelForCausalLM.from_pretrained(path_or_name)` returns a
`VRAMancerCausalLM` for architectures this framework implements (Qwen2, Llama,
Mistral, GPT-2, Qwen2-MoE) when the weights are available locally (a directory of
safetensors) or the name is a known preset (random-init benchmark weights); its
`.generate(input_ids, max_new_tokens=...)` runs on the paged-KV engine with
prompt-lookup speculation on by default (`prompt_lookup_num_tokens=10` as in the
reference).  Anything else falls through to the original from_pretrained.
`compute_max_memory()` returns the per-GPU budget map HF loaders accept.

Reference parity: vramancer/dropin.py (compute_max_memory 38-61, prompt-lookup wrap
75-96, light/heavy wrappers 99-168, patch/unpatch/is_patched 174-200).
"""
from __future__ import annotations

import os
from typing import Any, Optional

import torch

from .parallel.placement import compute_max_memory  # noqa: F401  (public re-export)

_orig = None


class VRAMancerCausalLM:
    def __init__(self, name_or_path: str, **kw):
        from .pipeline import InferencePipeline
        self.name = name_or_path
        self.pipeline = InferencePipeline(enable_metrics=False).load(name_or_path, **kw)
        self.config = self.pipeline.llm.cfg

    @torch.no_grad()
    def generate(self, input_ids=None, max_new_tokens: int = 32, do_sample: bool = False, temperature: float = 1.0,
                 top_k: int = 0, top_p: float = 1.0, prompt_lookup_num_tokens: Optional[int] = 10, **kw):
        ids = input_ids if input_ids is not None else kw.get("inputs")
        rows = ids.tolist() if isinstance(ids, torch.Tensor) else ids
        if rows and isinstance(rows[0], int):
            rows = [rows]
        outs = []
        for r in rows:
            if not do_sample and prompt_lookup_num_tokens:
                from .engine.speculative import PromptLookupDecoder
                new = PromptLookupDecoder(self.pipeline.llm, num_draft=prompt_lookup_num_tokens).generate(
                    r, max_new_tokens)
            else:
                new = self.pipeline.generate(r, max_new_tokens=max_new_tokens,
                                             temperature=temperature if do_sample else 0.0, top_k=top_k,
                                             top_p=top_p, return_ids=True)
            outs.append(list(r) + list(new))
        width = max(len(o) for o in outs)
        pad = 0
        t = torch.full((len(outs), width), pad, dtype=torch.long)
        for i, o in enumerate(outs):
            t[i, :len(o)] = torch.tensor(o)
        return t

    def __call__(self, input_ids, **kw):
        logits = torch.stack([self.pipeline.infer(r) for r in input_ids.tolist()])
        return type("Out", (), {"logits": logits.unsqueeze(1)})()


def _supported(name: str) -> bool:
    from .models.config import ALIASES, PRESETS
    if os.path.isdir(name) and os.path.exists(os.path.join(name, "config.json")):
        import json
        mt = json.load(open(os.path.join(name, "config.json"))).get("model_type", "")
        return mt in ("qwen2", "llama", "mistral", "gpt2", "qwen2_moe")
    return name in PRESETS or name in ALIASES


def patch(mode: str = "light") -> None:
    global _orig
    from transformers import AutoModelForCausalLM
    if _orig is not None:
        return
    _orig = AutoModelForCausalLM.from_pretrained.__func__ if hasattr(
        AutoModelForCausalLM.from_pretrained, "__func__") else AutoModelForCausalLM.from_pretrained

    def from_pretrained(cls, name, *args, **kwargs):
        if isinstance(name, str) and _supported(name):
            kw = {k: kwargs[k] for k in ("num_gpus", "max_batch", "max_model_len") if k in kwargs}
            return VRAMancerCausalLM(name, **kw)
        return _orig(cls, name, *args, **kwargs)

    AutoModelForCausalLM.from_pretrained = classmethod(from_pretrained)


def unpatch() -> None:
    global _orig
    from transformers import AutoModelForCausalLM
    if _orig is None:
        return
    AutoModelForCausalLM.from_pretrained = classmethod(_orig)
    _orig = None


def is_patched() -> bool:
    return _orig is not None
