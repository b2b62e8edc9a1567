"""`TurboEngine`: the reference's single-model engine object, over this framework's engine.

    eng = TurboEngine(hf_model, tokenizer, device="cuda:0", max_seq_len=4096)
    eng.warmup()
    text = eng.generate("Hello", max_new_tokens=64)
    for piece in eng.generate_stream("Hello"): ...
    ids = eng.generate_ids(input_ids, max_new_tokens=64)       # [1, prompt + new]

`model` may be a loaded Hugging Face causal LM (its config and state dict are converted
into this framework's fused layout: q|k|v and gate|up fused, experts stacked), a preset
name or checkpoint directory, a `ModelConfig`, or an existing `LLM`.  The engine then
holds its own weights (bf16 on a GPU, fp32 on the host), a paged KV pool sized for
`max_seq_len` and decode steps replayed from CUDA graphs -- the reference's
`torch.compile` and `cuda_graph` options both name that fast path, which is on
unless both are False.  Sampling follows the reference's rule: `do_sample=False` is
greedy whatever the temperature; with `do_sample=True` temperature, top-k and top-p
apply.

`MultiGPUTurboEngine` runs a model whose layers are spread over devices
(`layer_devices` {layer: device}) as an in-process pipeline; `SpeculativeTurboEngine`
pairs a target with a small draft model (gamma-adaptive, rejection sampling when
sampling); `create_turbo_engine` picks between the first two from the model's
`hf_device_map`.

Reference parity: core/turbo_engine.py:257-803 (TurboEngine: constructor arguments,
warmup, generate, generate_stream, generate_ids), :806-997 (MultiGPUTurboEngine),
:1000-1377 (SpeculativeTurboEngine, stats keys), :1380-1440 (create_turbo_engine).
"""
from __future__ import annotations

from typing import Dict, Iterator, List, Optional, Sequence, Union

import torch

from ..llm import LLM
from ..models.config import ModelConfig
from ..models.weights import weights_from_state_dict
from .engine import SamplingParams


def _is_hf_model(model) -> bool:
    return hasattr(model, "config") and hasattr(model, "state_dict") and hasattr(model.config, "to_dict")


def _hf_config(model) -> ModelConfig:
    d = model.config.to_dict()
    return ModelConfig.from_hf_config(d, name=str(d.get("_name_or_path", "")))


def _dtype_for(device: torch.device) -> torch.dtype:
    return torch.bfloat16 if device.type == "cuda" else torch.float32


def _kv_for(device: torch.device) -> str:
    return "bf16" if device.type == "cuda" else "fp32"


def _pages(max_seq_len: int, max_batch: int) -> int:
    return max_batch * ((max_seq_len + 15) // 16) + 16


def build_llm(model, device: Union[str, torch.device] = "cuda:0", *, max_seq_len: int = 2048, max_batch: int = 8,
              use_cuda_graph: bool = True, eos_token_id: Optional[int] = None) -> LLM:
    """An `LLM` on `device` for any of the model forms `TurboEngine` accepts."""
    if isinstance(model, LLM):
        return model
    dev = torch.device(device)
    if dev.type == "cuda" and not torch.cuda.is_available():
        raise RuntimeError(f"device {dev} requested but CUDA is not available")
    kw = dict(device=str(dev), dtype=_dtype_for(dev), kv_cache_dtype=_kv_for(dev), max_batch=max_batch,
              max_model_len=max_seq_len, kv_pages=_pages(max_seq_len, max_batch),
              use_cuda_graph=use_cuda_graph and dev.type == "cuda", eos_token_id=eos_token_id)
    if _is_hf_model(model):
        cfg = _hf_config(model)
        w = weights_from_state_dict(cfg, model.state_dict(), device=dev, dtype=_dtype_for(dev))
        return LLM(cfg, weights=w, **kw)
    return LLM(model, **kw)


class _TextIO:
    """Prompt text <-> token ids through an HF-style tokenizer (`__call__` with
    return_tensors, or `encode`) or ids given directly."""

    def __init__(self, tokenizer):
        self.tokenizer = tokenizer
        self.eos_token_id = getattr(tokenizer, "eos_token_id", None)

    def encode(self, prompt) -> List[int]:
        if isinstance(prompt, torch.Tensor):
            return [int(t) for t in prompt.flatten().tolist()]
        if not isinstance(prompt, str):
            return [int(t) for t in prompt]
        tok = self.tokenizer
        if tok is None:
            raise ValueError("a text prompt needs a tokenizer")
        if callable(tok):
            try:
                enc = tok(prompt, return_tensors="pt")
                ids = enc["input_ids"] if isinstance(enc, dict) or hasattr(enc, "keys") else enc
                if isinstance(ids, torch.Tensor):
                    return [int(t) for t in ids.flatten().tolist()]
            except TypeError:
                pass
        return [int(t) for t in tok.encode(prompt)]

    def decode(self, ids: Sequence[int]) -> str:
        try:
            return self.tokenizer.decode(list(ids), skip_special_tokens=True)
        except TypeError:
            return self.tokenizer.decode(list(ids))


def _params(max_new_tokens, temperature, top_k, top_p, do_sample) -> SamplingParams:
    if not do_sample:
        return SamplingParams(max_tokens=max_new_tokens)
    return SamplingParams(max_tokens=max_new_tokens, temperature=max(float(temperature), 1e-5), top_k=int(top_k),
                          top_p=float(top_p))


class TurboEngine:
    def __init__(self, model, tokenizer=None, device: str = "cuda:0", max_seq_len: int = 2048, compile: bool = True,
                 cuda_graph: bool = False, max_batch: int = 8):
        self.io = _TextIO(tokenizer)
        self.tokenizer = tokenizer
        self.max_seq_len = max_seq_len
        self.llm = build_llm(model, device, max_seq_len=max_seq_len, max_batch=max_batch,
                             use_cuda_graph=bool(compile or cuda_graph), eos_token_id=self.io.eos_token_id)
        self._init_common()

    def _init_common(self):
        cfg = self.llm.cfg
        self.device = self.llm.device
        self.n_layers, self.n_kv_heads, self.head_dim = cfg.num_layers, cfg.num_kv_heads, cfg.head_dim
        self.vocab_size = cfg.vocab_size
        self.eos_token_id = self.io.eos_token_id
        self.dtype = next(iter(self.llm.weights.values())).dtype if self.llm.weights else _dtype_for(self.device)

    # ------------------------------------------------------------------ helpers
    def _check_len(self, ids: List[int]) -> None:
        if len(ids) >= self.max_seq_len:
            raise ValueError(f"Prompt length {len(ids)} exceeds max_seq_len {self.max_seq_len}")

    def _budget(self, ids: List[int], max_new_tokens: int) -> int:
        return max(1, min(max_new_tokens, self.max_seq_len - len(ids)))

    def _run(self, ids: List[int], params: SamplingParams) -> List[int]:
        return list(self.llm.engine.generate([ids], params)[0].output_ids)

    # ------------------------------------------------------------------ API
    def warmup(self, prompt: str = "Hello", n_tokens: int = 10, rounds: int = 3) -> None:
        """Captures the batch-1 decode graph and runs `rounds` short generations."""
        if self.llm.runner.use_graph:
            self.llm.warmup([1])
        ids = self.io.encode(prompt) if (self.tokenizer is not None or not isinstance(prompt, str)) else [0]
        for _ in range(max(1, rounds)):
            self._run(ids or [0], SamplingParams(max_tokens=n_tokens, ignore_eos=True))

    def generate(self, prompt, max_new_tokens: int = 128, temperature: float = 1.0, top_k: int = 0,
                 top_p: float = 1.0, do_sample: bool = False, **kwargs) -> str:
        ids = self.io.encode(prompt)
        self._check_len(ids)
        out = self._run(ids, _params(self._budget(ids, max_new_tokens), temperature, top_k, top_p, do_sample))
        return self.io.decode(out)

    def generate_stream(self, prompt, max_new_tokens: int = 128, temperature: float = 1.0, top_k: int = 0,
                        top_p: float = 1.0, do_sample: bool = False, **kwargs) -> Iterator[str]:
        """Text pieces as tokens are produced (an end-of-sequence token ends the stream
        and is not shown); a piece is the text the new tokens add to the decoded output.
        Text ending in an incomplete UTF-8 sequence (U+FFFD) is held back until a later
        token completes it or the stream ends, so multi-token characters come out whole."""
        ids = self.io.encode(prompt)
        self._check_len(ids)
        eng = self.llm.engine
        got: List[int] = []
        req = eng.add_request(ids, _params(self._budget(ids, max_new_tokens), temperature, top_k, top_p, do_sample),
                              on_token=lambda r, t: got.append(t))
        shown, prev = 0, ""
        try:
            while True:
                finished = req.finished
                if not finished:
                    eng.step()
                if len(got) > shown or finished:
                    keep = [t for t in got if t != self.eos_token_id] if self.eos_token_id is not None else got
                    text = self.io.decode(keep)
                    shown = len(got)
                    if not finished:
                        text = text.rstrip("\ufffd")
                    if len(text) > len(prev) and text.startswith(prev):
                        yield text[len(prev):]
                        prev = text
                if finished:
                    break
        finally:
            if not req.finished:
                eng.abort(req.request_id)
                while eng.has_unfinished():
                    eng.step()

    def generate_ids(self, input_ids, max_new_tokens: int = 128, temperature: float = 1.0, top_k: int = 0,
                     top_p: float = 1.0, do_sample: bool = False) -> torch.Tensor:
        """Prompt ids [1, P] (or a flat sequence) -> [1, P + new] on the prompt's device."""
        ids = self.io.encode(input_ids)
        self._check_len(ids)
        out = self._run(ids, _params(self._budget(ids, max_new_tokens), temperature, top_k, top_p, do_sample))
        dev = input_ids.device if isinstance(input_ids, torch.Tensor) else self.device
        return torch.tensor([ids + out], dtype=torch.long, device=dev)


def _blocks_from_layer_devices(layer_devices: Dict[int, object], num_layers: int):
    """Contiguous runs of layers on one device -> placement Blocks (every layer must be
    named; a device may appear in several runs)."""
    from ..parallel.placement import Block
    missing = [i for i in range(num_layers) if i not in layer_devices]
    if missing:
        raise ValueError(f"layer_devices names no device for layers {missing[:8]}")
    blocks = []
    start = 0
    for i in range(1, num_layers + 1):
        if i == num_layers or str(layer_devices[i]) != str(layer_devices[start]):
            blocks.append(Block(len(blocks), start, i, str(torch.device(layer_devices[start]))))
            start = i
    return blocks


class MultiGPUTurboEngine(TurboEngine):
    """Layers on several devices as one in-process pipeline: each run of consecutive
    layers on one device is a stage with its own KV pool; hidden states cross between
    stages through `transfer_manager.send_tensor` when given, else a peer copy."""

    def __init__(self, model, tokenizer=None, layer_devices: Optional[Dict[int, object]] = None,
                 transfer_manager=None, max_seq_len: int = 2048, max_batch: int = 8):
        self.io = _TextIO(tokenizer)
        self.tokenizer = tokenizer
        self.max_seq_len = max_seq_len
        self.transfer_manager = transfer_manager
        if _is_hf_model(model):
            cfg = _hf_config(model)
            sd = model.state_dict()
        elif isinstance(model, ModelConfig):
            cfg, sd = model, None
        else:
            from ..models.config import get_config
            cfg, sd = get_config(model), None
        if layer_devices is None:
            n = max(1, torch.cuda.device_count())
            per = (cfg.num_layers + n - 1) // n
            layer_devices = {i: f"cuda:{i // per}" for i in range(cfg.num_layers)}
        blocks = _blocks_from_layer_devices(layer_devices, cfg.num_layers)
        dev0 = torch.device(blocks[0].device)
        dtype = _dtype_for(dev0)
        weights = weights_from_state_dict(cfg, sd, dtype=dtype) if sd is not None else None
        transfer = None
        if transfer_manager is not None:
            def transfer(t, device, _tm=transfer_manager):
                d = torch.device(device)
                return _tm.send_tensor(t, d.index if d.type == "cuda" else -1)
        self.layer_devices = dict(layer_devices)
        self.primary_device = dev0
        from ..kv.pool import kv_dtype_from_str
        self.llm = LLM.from_local_pipeline(cfg, blocks, num_pages=_pages(max_seq_len, max_batch), max_batch=max_batch,
                                           max_model_len=max_seq_len, dtype=dtype,
                                           kv_dtype=kv_dtype_from_str(_kv_for(dev0)), weights=weights,
                                           transfer=transfer, eos_token_id=self.io.eos_token_id)
        self._init_common()

    def warmup(self, prompt: str = "Hello", n_tokens: int = 10, rounds: int = 1) -> None:
        super().warmup(prompt, n_tokens, rounds)


class SpeculativeTurboEngine:
    """A target model verifying a draft model's proposals, gamma tokens per round
    (adaptive in [2, 12] from the recent acceptance).  Greedy requests accept the
    longest matching prefix plus the target's token; sampled requests accept by
    rejection sampling, so outputs follow the target's distribution."""

    def __init__(self, main_model, draft_model, tokenizer=None, device: str = "cuda:0", gamma: int = 5,
                 max_seq_len: int = 2048, compile_main: bool = True, compile_draft: bool = True):
        from .speculative import DraftModelDecoder
        self.io = _TextIO(tokenizer)
        self.tokenizer = tokenizer
        self.device = torch.device(device)
        self.max_seq_len = max_seq_len
        self.eos_token_id = self.io.eos_token_id
        self.main = build_llm(main_model, device, max_seq_len=max_seq_len, max_batch=2,
                              use_cuda_graph=compile_main, eos_token_id=self.eos_token_id)
        self.draft = build_llm(draft_model, device, max_seq_len=max_seq_len, max_batch=2,
                               use_cuda_graph=compile_draft, eos_token_id=self.eos_token_id)
        self.decoder = DraftModelDecoder(self.main, self.draft, gamma=gamma)
        self._seed = 0

    @property
    def gamma(self) -> int:
        return self.decoder.gamma

    def warmup(self, prompt: str = "Hello", n_tokens: int = 10, rounds: int = 3) -> None:
        for llm in (self.main, self.draft):
            if llm.runner.use_graph:
                llm.warmup([1])
        ids = self.io.encode(prompt) if self.tokenizer is not None else [0]
        for _ in range(max(1, rounds)):
            self.decoder.generate(ids or [0], n_tokens)

    def generate(self, prompt, max_new_tokens: int = 128, temperature: float = 1.0, top_k: int = 0,
                 top_p: float = 1.0, do_sample: bool = False, **kwargs) -> str:
        ids = self.io.encode(prompt)
        if len(ids) >= self.max_seq_len:
            raise ValueError(f"Prompt {len(ids)} exceeds max_seq_len {self.max_seq_len}")
        n = max(1, min(max_new_tokens, self.max_seq_len - len(ids)))
        params = _params(n, temperature, top_k, top_p, do_sample)
        self._seed += 1
        out = self.decoder.generate(ids, n, params=params, seed=self._seed)
        return self.io.decode(out)

    def stats(self) -> dict:
        s = self.decoder.stats
        rate = s.accepted / max(1, s.proposed)
        return {"drafted": s.proposed, "accepted": s.accepted, "rounds": s.steps, "acceptance_rate": rate,
                "effective_tokens_per_round": (s.accepted + s.steps) / max(1, s.steps)}


def create_turbo_engine(model, tokenizer=None, transfer_manager=None, max_seq_len: int = 2048, compile: bool = True,
                        cuda_graph: bool = False):
    """`MultiGPUTurboEngine` when the HF model's `hf_device_map` spans several devices
    (each decoder layer's device read from its parameters), else a `TurboEngine` on
    the device of the model's parameters."""
    device_map = getattr(model, "hf_device_map", None)
    if device_map and len({str(v) for v in device_map.values()}) > 1:
        inner = getattr(model, "model", model)
        layer_devices = {}
        for i, layer in enumerate(getattr(inner, "layers", [])):
            p = next(layer.parameters(), None)
            layer_devices[i] = p.device if p is not None else torch.device("cuda:0")
        return MultiGPUTurboEngine(model, tokenizer, layer_devices=layer_devices, transfer_manager=transfer_manager,
                                   max_seq_len=max_seq_len)
    device = "cuda:0"
    if hasattr(model, "parameters"):
        p = next(model.parameters(), None)
        if p is not None:
            device = str(p.device)
    return TurboEngine(model, tokenizer, device=device, max_seq_len=max_seq_len, compile=compile,
                       cuda_graph=cuda_graph)
