"""Inference backends behind one interface, and the factory that picks one.

  native       this package's engine (tcgen05 kernels, paged KV, CUDA graphs): every
               architecture of models/config.py (Qwen2 / Llama / Mistral / GPT-2 /
               Qwen2-MoE); the default
  huggingface  transformers AutoModelForCausalLM + generate(), for architectures the
               native engine does not implement
  vllm         vllm.LLM, when the package is installed
  llamacpp     llama-cpp-python over a GGUF file, when installed
  ollama       an Ollama server over HTTP (OLLAMA_HOST, default 127.0.0.1:11434)

`select_backend(model, backend="auto")`: GGUF files go to llama.cpp, known
architectures to the native engine, anything else to transformers.

Reference parity: core/backends.py select_backend / HuggingFaceBackend
(load_model, generate, infer), core/backends_vllm.py, core/backends_llamacpp.py,
core/backends_ollama.py.  The reference's auto order prefers vLLM over its HF path; here
the native engine comes first because it is this package's fast path.
"""
from __future__ import annotations

import json
import os
from typing import Any, List, Optional, Sequence, Union

import torch

Prompt = Union[str, Sequence[int]]


class Backend:
    backend_type = "base"

    def load_model(self, model_name: str, **kw) -> "Backend":
        raise NotImplementedError

    def generate(self, prompt: Prompt, max_new_tokens: int = 128, **sampling) -> str:
        raise NotImplementedError

    def generate_ids(self, ids: Sequence[int], max_new_tokens: int = 128, **sampling) -> List[int]:
        raise NotImplementedError

    def infer(self, input_ids: torch.Tensor) -> torch.Tensor:
        """Logits [B, T, V] of one forward (no sampling)."""
        raise NotImplementedError

    def unload(self) -> None:
        pass


class NativeBackend(Backend):
    backend_type = "native"

    def __init__(self, **pipeline_kw):
        from .pipeline import InferencePipeline
        self.pipe = InferencePipeline(**{k: v for k, v in pipeline_kw.items() if k in ("enable_metrics",)})
        self.load_kw = {k: v for k, v in pipeline_kw.items() if k != "enable_metrics"}

    def load_model(self, model_name: str, **kw) -> "NativeBackend":
        self.pipe.load(model_name, **{**self.load_kw, **kw})
        self.tokenizer = self.pipe.tokenizer
        return self

    def generate(self, prompt: Prompt, max_new_tokens: int = 128, **sampling) -> str:
        return self.pipe.generate(prompt, max_new_tokens=max_new_tokens, **sampling)

    def generate_ids(self, ids: Sequence[int], max_new_tokens: int = 128, **sampling) -> List[int]:
        return self.pipe.generate(list(ids), max_new_tokens=max_new_tokens, return_ids=True, **sampling)

    def infer(self, input_ids: torch.Tensor) -> torch.Tensor:
        return self.pipe.infer(input_ids)

    def unload(self) -> None:
        self.pipe.shutdown()


class HuggingFaceBackend(Backend):
    backend_type = "huggingface"

    def __init__(self, device: Optional[str] = None, dtype: torch.dtype = torch.bfloat16):
        self.device = device or ("cuda:0" if torch.cuda.is_available() else "cpu")
        self.dtype = dtype if self.device != "cpu" else torch.float32
        self.model = None
        self.tokenizer = None

    def load_model(self, model_name: str, config=None, **kw) -> "HuggingFaceBackend":
        """A local checkpoint directory, or `config` (a transformers PretrainedConfig)
        for a random-initialised model of that architecture."""
        from transformers import AutoModelForCausalLM
        if config is not None:
            with torch.device(self.device):
                self.model = AutoModelForCausalLM.from_config(config, torch_dtype=self.dtype)
        else:
            self.model = AutoModelForCausalLM.from_pretrained(model_name, torch_dtype=self.dtype, **kw).to(self.device)
        self.model.eval()
        from .serving.tokenizer import load_tokenizer
        vocab = self.model.config.vocab_size
        self.tokenizer = load_tokenizer(model_name if model_name and os.path.isdir(model_name) else None, vocab)
        return self

    @torch.no_grad()
    def generate_ids(self, ids: Sequence[int], max_new_tokens: int = 128, temperature: float = 0.0,
                     **sampling) -> List[int]:
        x = torch.tensor([list(ids)], device=self.device)
        kw = dict(max_new_tokens=max_new_tokens, min_new_tokens=sampling.pop("min_new_tokens", 0),
                  do_sample=temperature > 0, pad_token_id=0)
        if temperature > 0:
            kw.update(temperature=temperature, top_k=sampling.get("top_k", 0) or None,
                      top_p=sampling.get("top_p", 1.0))
        out = self.model.generate(x, **kw)
        return out[0, x.shape[1]:].tolist()

    def generate(self, prompt: Prompt, max_new_tokens: int = 128, **sampling) -> str:
        ids = self.tokenizer.encode(prompt) if isinstance(prompt, str) else list(prompt)
        return self.tokenizer.decode(self.generate_ids(ids, max_new_tokens, **sampling))

    @torch.no_grad()
    def infer(self, input_ids: torch.Tensor) -> torch.Tensor:
        return self.model(input_ids.to(self.device)).logits

    def unload(self) -> None:
        self.model = None
        if torch.cuda.is_available():
            torch.cuda.empty_cache()


class VLLMBackend(Backend):
    backend_type = "vllm"

    def __init__(self, tensor_parallel_size: int = 1, gpu_memory_utilization: float = 0.9):
        self.tp, self.util = tensor_parallel_size, gpu_memory_utilization
        self.llm = None

    def load_model(self, model_name: str, **kw) -> "VLLMBackend":
        try:
            from vllm import LLM as _VLLM
        except ImportError as e:
            raise ImportError("backend 'vllm' needs the vllm package") from e
        self.llm = _VLLM(model=model_name, tensor_parallel_size=self.tp, gpu_memory_utilization=self.util, **kw)
        return self

    def _params(self, max_new_tokens, temperature=0.0, top_p=1.0, top_k=0, **_):
        from vllm import SamplingParams
        return SamplingParams(max_tokens=max_new_tokens, temperature=temperature, top_p=top_p,
                              top_k=top_k if top_k > 0 else -1)

    def generate(self, prompt: Prompt, max_new_tokens: int = 128, **sampling) -> str:
        out = self.llm.generate([prompt] if isinstance(prompt, str) else [{"prompt_token_ids": list(prompt)}],
                                self._params(max_new_tokens, **sampling))
        return out[0].outputs[0].text

    def generate_ids(self, ids: Sequence[int], max_new_tokens: int = 128, **sampling) -> List[int]:
        out = self.llm.generate([{"prompt_token_ids": list(ids)}], self._params(max_new_tokens, **sampling))
        return list(out[0].outputs[0].token_ids)


class LlamaCppBackend(Backend):
    backend_type = "llamacpp"

    def __init__(self, n_ctx: int = int(os.environ.get("VRM_N_CTX", "4096")), n_gpu_layers: int = -1):
        self.n_ctx, self.n_gpu_layers = n_ctx, n_gpu_layers
        self.llm = None

    def load_model(self, model_name: str, **kw) -> "LlamaCppBackend":
        try:
            from llama_cpp import Llama
        except ImportError as e:
            raise ImportError("backend 'llamacpp' needs llama-cpp-python") from e
        self.llm = Llama(model_path=model_name, n_ctx=self.n_ctx, n_gpu_layers=self.n_gpu_layers, verbose=False, **kw)
        return self

    def generate(self, prompt: Prompt, max_new_tokens: int = 128, temperature: float = 0.0, **sampling) -> str:
        text = prompt if isinstance(prompt, str) else self.llm.detokenize(list(prompt)).decode("utf-8", "ignore")
        out = self.llm(text, max_tokens=max_new_tokens, temperature=temperature)
        return out["choices"][0]["text"]

    def generate_ids(self, ids: Sequence[int], max_new_tokens: int = 128, temperature: float = 0.0,
                     **sampling) -> List[int]:
        out = []
        for tok in self.llm.generate(list(ids), temp=temperature):
            out.append(int(tok))
            if len(out) >= max_new_tokens:
                break
        return out


class OllamaBackend(Backend):
    backend_type = "ollama"

    def __init__(self, host: Optional[str] = None, timeout: float = 600.0):
        self.host = (host or os.environ.get("OLLAMA_HOST", "127.0.0.1:11434")).rstrip("/")
        if not self.host.startswith("http"):
            self.host = "http://" + self.host
        self.timeout = timeout
        self.model = None

    def load_model(self, model_name: str, **kw) -> "OllamaBackend":
        self.model = model_name
        return self

    def generate(self, prompt: Prompt, max_new_tokens: int = 128, temperature: float = 0.0, **sampling) -> str:
        import requests
        if not isinstance(prompt, str):
            raise TypeError("the ollama backend takes text prompts")
        r = requests.post(f"{self.host}/api/generate", timeout=self.timeout,
                          data=json.dumps({"model": self.model, "prompt": prompt, "stream": False,
                                           "options": {"num_predict": max_new_tokens, "temperature": temperature}}))
        r.raise_for_status()
        return r.json().get("response", "")


def _is_gguf(name: str) -> bool:
    return str(name).lower().endswith(".gguf")


def native_supports(model_name: str) -> bool:
    """True when the native engine implements the model's architecture."""
    from .models.config import PRESETS, get_config
    if model_name in PRESETS:
        return True
    try:
        get_config(model_name)
        return True
    except Exception:  # noqa: BLE001 - unknown architecture / not a checkpoint
        return False


def select_backend(model_name: str, backend: str = "auto", num_gpus: int = 1, **kw) -> Backend:
    backend = (backend or "auto").lower()
    if backend == "native":
        return NativeBackend(num_gpus=num_gpus, **kw)
    if backend in ("huggingface", "hf"):
        return HuggingFaceBackend(**kw)
    if backend == "vllm":
        return VLLMBackend(tensor_parallel_size=max(1, num_gpus))
    if backend == "llamacpp":
        return LlamaCppBackend()
    if backend == "ollama":
        return OllamaBackend()
    if backend != "auto":
        raise ValueError(f"unknown backend {backend!r} (auto, native, huggingface, vllm, llamacpp, ollama)")
    if _is_gguf(model_name):
        return LlamaCppBackend()
    if native_supports(model_name):
        return NativeBackend(num_gpus=num_gpus, **kw)
    return HuggingFaceBackend(**kw)
