"""Model architecture descriptions and the named presets used by the benchmarks.

One `ModelConfig` covers the decoder-only families the reference serves through HF
(core/backends.py:1185-1412): Llama / Qwen2 / Mistral (RMSNorm, RoPE, GQA, SwiGLU),
Qwen3 (the same plus a per-head RMSNorm of q and k), GPT-2 (LayerNorm, learned
positions, GELU, fused c_attn) and mixture-of-experts decoders (top-k softmax router
over SwiGLU experts: Qwen2-MoE with a gated shared expert, Qwen3-MoE, Mixtral).  RoPE
scaling (linear, Llama 3, YaRN) is part of the config.  `from_hf_config` reads an HF
`config.json` so checkpoints load without transformers, and raises
`UnsupportedArchitecture` for anything else (the backend factory then picks another
backend rather than run a different model).
"""
from __future__ import annotations

import json
import os
from dataclasses import asdict, dataclass, field, replace
from typing import Any, Dict, Optional, Tuple


class UnsupportedArchitecture(ValueError):
    """An HF config the native engine does not implement (the backend factory then
    serves the model through another backend)."""


@dataclass(frozen=True)
class ModelConfig:
    arch: str = "qwen2"              # qwen2 | qwen3 | llama | mistral | gpt2 | qwen2_moe
    vocab_size: int = 152064
    hidden_size: int = 5120
    num_layers: int = 48
    num_heads: int = 40
    num_kv_heads: int = 8
    head_dim: int = 128
    intermediate_size: int = 13824
    max_position: int = 32768
    norm_eps: float = 1e-6
    rope_theta: float = 1_000_000.0
    rotary_dim: Optional[int] = None     # None -> head_dim (no RoPE for gpt2)
    # RoPE frequency scaling as sorted (key, value) pairs of the HF rope parameters
    # ("rope_type" linear | llama3 | yarn | dynamic, "factor", ...); None = plain RoPE
    rope_scaling: Optional[Tuple[Tuple[str, Any], ...]] = None
    qkv_bias: bool = True
    qk_norm: bool = False                # per-head RMSNorm of q and k before RoPE (Qwen3)
    tie_embeddings: bool = False
    # MoE
    num_experts: int = 0
    experts_per_token: int = 0
    expert_intermediate_size: int = 0
    shared_expert_intermediate_size: int = 0
    norm_topk_prob: bool = True
    name: str = ""

    # ------------------------------------------------------------------ derived
    @property
    def is_gpt2(self) -> bool:
        return self.arch == "gpt2"

    @property
    def is_moe(self) -> bool:
        return self.num_experts > 0

    @property
    def q_size(self) -> int:
        return self.num_heads * self.head_dim

    @property
    def kv_size(self) -> int:
        return self.num_kv_heads * self.head_dim

    @property
    def rot_dim(self) -> int:
        if self.is_gpt2:
            return 0
        return self.rotary_dim if self.rotary_dim is not None else self.head_dim

    def num_params(self) -> int:
        H, L, V = self.hidden_size, self.num_layers, self.vocab_size
        attn = H * (self.q_size + 2 * self.kv_size) + self.q_size * H
        if self.is_moe:
            mlp = self.num_experts * 3 * H * self.expert_intermediate_size + H * self.num_experts
            if self.shared_expert_intermediate_size:
                mlp += 3 * H * self.shared_expert_intermediate_size + H
        else:
            mlp = (2 if self.is_gpt2 else 3) * H * self.intermediate_size
        emb = V * H * (1 if self.tie_embeddings else 2)
        if self.is_gpt2:
            emb += self.max_position * H
        return L * (attn + mlp + 2 * H) + emb + H

    def kv_bytes_per_token(self, dtype_bytes: int = 2) -> int:
        return 2 * self.num_layers * self.kv_size * dtype_bytes

    def with_(self, **kw) -> "ModelConfig":
        return replace(self, **kw)

    def to_dict(self) -> Dict[str, Any]:
        return asdict(self)

    # ------------------------------------------------------------------ HF config
    @staticmethod
    def from_hf_config(cfg: Dict[str, Any], name: str = "") -> "ModelConfig":
        mt = cfg.get("model_type", "llama")
        if mt == "gpt2":
            H = cfg.get("n_embd", 768)
            nh = cfg.get("n_head", 12)
            return ModelConfig(arch="gpt2", vocab_size=cfg.get("vocab_size", 50257), hidden_size=H,
                               num_layers=cfg.get("n_layer", 12), num_heads=nh, num_kv_heads=nh,
                               head_dim=H // nh, intermediate_size=cfg.get("n_inner") or 4 * H,
                               max_position=cfg.get("n_positions", 1024),
                               norm_eps=cfg.get("layer_norm_epsilon", 1e-5), rope_theta=0.0, qkv_bias=True,
                               tie_embeddings=True, name=name)
        H = cfg["hidden_size"]
        nh = cfg["num_attention_heads"]
        kvh = cfg.get("num_key_value_heads", nh)
        hd = cfg.get("head_dim") or H // nh
        # RoPE: transformers 5 writes `rope_parameters` ({"rope_theta", "rope_type", ...});
        # older configs a top-level `rope_theta` and an optional `rope_scaling`
        rp = dict(cfg.get("rope_parameters") or {})
        theta = rp.pop("rope_theta", None) or cfg.get("rope_theta", 10000.0)
        if cfg.get("rope_scaling"):
            rp.update(cfg["rope_scaling"])
        if "type" in rp and "rope_type" not in rp:
            rp["rope_type"] = rp.pop("type")
        rp.pop("partial_rotary_factor", None)
        scaling = None
        if rp.get("rope_type", "default") != "default":
            if "original_max_position_embeddings" not in rp and cfg.get("original_max_position_embeddings"):
                rp["original_max_position_embeddings"] = cfg["original_max_position_embeddings"]
            scaling = tuple(sorted((k, v) for k, v in rp.items() if not isinstance(v, (list, dict))))
        prf = cfg.get("partial_rotary_factor") or (cfg.get("rope_parameters") or {}).get("partial_rotary_factor")
        rot = int(hd * prf) if prf else None
        arch = {"qwen2": "qwen2", "llama": "llama", "mistral": "mistral", "qwen2_moe": "qwen2_moe",
                "qwen3": "qwen3", "qwen3_moe": "qwen2_moe", "mixtral": "qwen2_moe"}.get(mt)
        if arch is None:
            raise UnsupportedArchitecture(f"model_type {mt!r} is not implemented by the native engine")
        act = cfg.get("hidden_act", "silu")
        if act not in ("silu", "swish"):
            raise UnsupportedArchitecture(f"hidden_act {act!r} (the native SwiGLU MLP needs silu)")
        if cfg.get("mlp_bias"):
            raise UnsupportedArchitecture("MLP biases are not implemented by the native engine")
        if mt in ("qwen2_moe", "qwen3_moe") and (cfg.get("mlp_only_layers") or cfg.get("decoder_sparse_step", 1) != 1):
            raise UnsupportedArchitecture("MoE models with dense layers between sparse ones are not implemented")
        moe = {}
        if arch == "qwen2_moe":
            # transformers 5 writes num_local_experts for Qwen3-MoE (Mixtral always did);
            # Mixtral's experts are intermediate_size wide and its top-k weights renormalised
            moe = dict(num_experts=cfg.get("num_experts") or cfg.get("num_local_experts") or 0,
                       experts_per_token=cfg.get("num_experts_per_tok", 0),
                       expert_intermediate_size=cfg.get("moe_intermediate_size") or cfg.get("intermediate_size", 0),
                       shared_expert_intermediate_size=cfg.get("shared_expert_intermediate_size", 0),
                       norm_topk_prob=True if mt == "mixtral" else cfg.get("norm_topk_prob", True))
        max_pos = cfg.get("max_position_embeddings", 32768)
        sw = cfg.get("sliding_window")
        if sw and cfg.get("use_sliding_window", True) and sw < max_pos:
            # sliding-window attention equals full attention while a sequence fits in
            # the window: the context is capped there instead of running SWA
            max_pos = int(sw)
        return ModelConfig(arch=arch, vocab_size=cfg["vocab_size"], hidden_size=H,
                           num_layers=cfg["num_hidden_layers"], num_heads=nh, num_kv_heads=kvh, head_dim=hd,
                           intermediate_size=cfg.get("intermediate_size", 4 * H),
                           max_position=max_pos,
                           norm_eps=cfg.get("rms_norm_eps", 1e-6), rope_theta=float(theta), rotary_dim=rot,
                           rope_scaling=scaling,
                           qkv_bias=bool(cfg.get("attention_bias", mt in ("qwen2", "qwen2_moe"))),
                           qk_norm=mt in ("qwen3", "qwen3_moe"),
                           tie_embeddings=bool(cfg.get("tie_word_embeddings", False)), name=name, **moe)

    @staticmethod
    def from_pretrained_dir(path: str) -> "ModelConfig":
        with open(os.path.join(path, "config.json")) as f:
            return ModelConfig.from_hf_config(json.load(f), name=os.path.basename(path.rstrip("/")))

    def to_hf_config(self) -> Dict[str, Any]:
        if self.is_gpt2:
            return {"model_type": "gpt2", "vocab_size": self.vocab_size, "n_embd": self.hidden_size,
                    "n_layer": self.num_layers, "n_head": self.num_heads, "n_positions": self.max_position,
                    "n_inner": self.intermediate_size, "layer_norm_epsilon": self.norm_eps,
                    "architectures": ["GPT2LMHeadModel"]}
        d = {"model_type": {"qwen2_moe": "qwen2_moe"}.get(self.arch, self.arch), "vocab_size": self.vocab_size,
             "hidden_size": self.hidden_size, "num_hidden_layers": self.num_layers,
             "num_attention_heads": self.num_heads, "num_key_value_heads": self.num_kv_heads,
             "head_dim": self.head_dim, "intermediate_size": self.intermediate_size,
             "max_position_embeddings": self.max_position, "rms_norm_eps": self.norm_eps,
             "rope_theta": self.rope_theta, "tie_word_embeddings": self.tie_embeddings,
             "hidden_act": "silu", "torch_dtype": "bfloat16"}
        if self.rope_scaling:
            d["rope_scaling"] = dict(self.rope_scaling)
        if self.rotary_dim is not None and self.rotary_dim != self.head_dim:
            d["partial_rotary_factor"] = self.rotary_dim / self.head_dim
        if self.qk_norm:
            d["model_type"] = "qwen3_moe" if self.is_moe else "qwen3"
            d["attention_bias"] = self.qkv_bias
        if self.arch == "qwen2":
            d["architectures"] = ["Qwen2ForCausalLM"]
        elif self.arch == "qwen3":
            d["architectures"] = ["Qwen3ForCausalLM"]
        elif self.arch in ("llama", "mistral"):
            d["architectures"] = ["LlamaForCausalLM"] if self.arch == "llama" else ["MistralForCausalLM"]
            d["attention_bias"] = self.qkv_bias
        if self.is_moe:
            d.update(num_experts=self.num_experts, num_experts_per_tok=self.experts_per_token,
                     moe_intermediate_size=self.expert_intermediate_size,
                     shared_expert_intermediate_size=self.shared_expert_intermediate_size,
                     norm_topk_prob=self.norm_topk_prob,
                     architectures=["Qwen3MoeForCausalLM" if self.qk_norm else "Qwen2MoeForCausalLM"])
        return d


# ---------------------------------------------------------------------------- presets
PRESETS: Dict[str, ModelConfig] = {
    # BASELINE config 1
    "gpt2": ModelConfig(arch="gpt2", vocab_size=50257, hidden_size=768, num_layers=12, num_heads=12,
                        num_kv_heads=12, head_dim=64, intermediate_size=3072, max_position=1024, norm_eps=1e-5,
                        rope_theta=0.0, qkv_bias=True, tie_embeddings=True, name="gpt2"),
    # BASELINE config 2
    "qwen2.5-7b": ModelConfig(arch="qwen2", vocab_size=152064, hidden_size=3584, num_layers=28, num_heads=28,
                              num_kv_heads=4, head_dim=128, intermediate_size=18944, max_position=32768,
                              norm_eps=1e-6, rope_theta=1_000_000.0, qkv_bias=True, name="qwen2.5-7b"),
    # BASELINE configs 3/4 (headline benchmark model)
    "qwen2.5-14b": ModelConfig(arch="qwen2", vocab_size=152064, hidden_size=5120, num_layers=48, num_heads=40,
                               num_kv_heads=8, head_dim=128, intermediate_size=13824, max_position=32768,
                               norm_eps=1e-6, rope_theta=1_000_000.0, qkv_bias=True, name="qwen2.5-14b"),
    # BASELINE config 5
    "moe-48l-128e": ModelConfig(arch="qwen2_moe", vocab_size=151936, hidden_size=2048, num_layers=48,
                                num_heads=32, num_kv_heads=4, head_dim=128, intermediate_size=768,
                                max_position=32768, norm_eps=1e-6, rope_theta=1_000_000.0, qkv_bias=False,
                                num_experts=128, experts_per_token=8, expert_intermediate_size=768,
                                norm_topk_prob=True, name="moe-48l-128e"),
    # further families served natively (random-init presets for the workloads)
    "qwen3-8b": ModelConfig(arch="qwen3", vocab_size=151936, hidden_size=4096, num_layers=36, num_heads=32,
                            num_kv_heads=8, head_dim=128, intermediate_size=12288, max_position=40960,
                            norm_eps=1e-6, rope_theta=1_000_000.0, qkv_bias=False, qk_norm=True, name="qwen3-8b"),
    "qwen3-30b-a3b": ModelConfig(arch="qwen2_moe", vocab_size=151936, hidden_size=2048, num_layers=48,
                                 num_heads=32, num_kv_heads=4, head_dim=128, intermediate_size=6144,
                                 max_position=40960, norm_eps=1e-6, rope_theta=1_000_000.0, qkv_bias=False,
                                 qk_norm=True, num_experts=128, experts_per_token=8, expert_intermediate_size=768,
                                 norm_topk_prob=True, name="qwen3-30b-a3b"),
    "llama-3.1-8b": ModelConfig(arch="llama", vocab_size=128256, hidden_size=4096, num_layers=32, num_heads=32,
                                num_kv_heads=8, head_dim=128, intermediate_size=14336, max_position=131072,
                                norm_eps=1e-5, rope_theta=500_000.0, qkv_bias=False,
                                rope_scaling=(("factor", 8.0), ("high_freq_factor", 4.0), ("low_freq_factor", 1.0),
                                              ("original_max_position_embeddings", 8192), ("rope_type", "llama3")),
                                name="llama-3.1-8b"),
    "mixtral-8x7b": ModelConfig(arch="qwen2_moe", vocab_size=32000, hidden_size=4096, num_layers=32, num_heads=32,
                                num_kv_heads=8, head_dim=128, intermediate_size=14336, max_position=32768,
                                norm_eps=1e-5, rope_theta=1_000_000.0, qkv_bias=False, num_experts=8,
                                experts_per_token=2, expert_intermediate_size=14336, norm_topk_prob=True,
                                name="mixtral-8x7b"),
    # default draft models for speculative decoding
    "qwen2.5-0.5b": ModelConfig(arch="qwen2", vocab_size=151936, hidden_size=896, num_layers=24, num_heads=14,
                                num_kv_heads=2, head_dim=64, intermediate_size=4864, max_position=32768,
                                norm_eps=1e-6, rope_theta=1_000_000.0, qkv_bias=True, tie_embeddings=True,
                                name="qwen2.5-0.5b"),
    "llama-3.2-1b": ModelConfig(arch="llama", vocab_size=128256, hidden_size=2048, num_layers=16, num_heads=32,
                                num_kv_heads=8, head_dim=64, intermediate_size=8192, max_position=131072,
                                norm_eps=1e-5, rope_theta=500_000.0, qkv_bias=False, tie_embeddings=True,
                                rope_scaling=(("factor", 32.0), ("high_freq_factor", 4.0), ("low_freq_factor", 1.0),
                                              ("original_max_position_embeddings", 8192), ("rope_type", "llama3")),
                                name="llama-3.2-1b"),
    "distilgpt2": ModelConfig(arch="gpt2", vocab_size=50257, hidden_size=768, num_layers=6, num_heads=12,
                              num_kv_heads=12, head_dim=64, intermediate_size=3072, max_position=1024, norm_eps=1e-5,
                              rope_theta=0.0, qkv_bias=True, tie_embeddings=True, name="distilgpt2"),
    # small shapes for tests
    "tiny-qwen3": ModelConfig(arch="qwen3", vocab_size=512, hidden_size=256, num_layers=2, num_heads=4,
                              num_kv_heads=2, head_dim=64, intermediate_size=512, max_position=2048,
                              norm_eps=1e-6, rope_theta=10000.0, qkv_bias=False, qk_norm=True, name="tiny-qwen3"),
    "tiny-qwen2": ModelConfig(arch="qwen2", vocab_size=512, hidden_size=256, num_layers=2, num_heads=4,
                              num_kv_heads=2, head_dim=64, intermediate_size=512, max_position=2048,
                              norm_eps=1e-6, rope_theta=10000.0, qkv_bias=True, name="tiny-qwen2"),
    "tiny-qwen2-d128": ModelConfig(arch="qwen2", vocab_size=1024, hidden_size=512, num_layers=2, num_heads=8,
                                   num_kv_heads=2, head_dim=128, intermediate_size=1024, max_position=4096,
                                   norm_eps=1e-6, rope_theta=1_000_000.0, qkv_bias=True, name="tiny-qwen2-d128"),
    # every head count, the FFN and the vocabulary divide over 8 tensor-parallel ranks
    "tiny-qwen2-tp8": ModelConfig(arch="qwen2", vocab_size=4096, hidden_size=1024, num_layers=2, num_heads=8,
                                  num_kv_heads=8, head_dim=128, intermediate_size=2048, max_position=4096,
                                  norm_eps=1e-6, rope_theta=1_000_000.0, qkv_bias=True, name="tiny-qwen2-tp8"),
    "tiny-gpt2": ModelConfig(arch="gpt2", vocab_size=500, hidden_size=128, num_layers=4, num_heads=2,
                             num_kv_heads=2, head_dim=64, intermediate_size=512, max_position=512, norm_eps=1e-5,
                             rope_theta=0.0, qkv_bias=True, tie_embeddings=True, name="tiny-gpt2"),
    "tiny-moe-wide": ModelConfig(arch="qwen2_moe", vocab_size=512, hidden_size=1024, num_layers=2, num_heads=8,
                                 num_kv_heads=2, head_dim=128, intermediate_size=256, max_position=2048,
                                 norm_eps=1e-6, rope_theta=10000.0, qkv_bias=False, num_experts=16,
                                 experts_per_token=4, expert_intermediate_size=256, norm_topk_prob=True,
                                 name="tiny-moe-wide"),
    "tiny-moe": ModelConfig(arch="qwen2_moe", vocab_size=512, hidden_size=256, num_layers=2, num_heads=4,
                            num_kv_heads=2, head_dim=64, intermediate_size=128, max_position=2048, norm_eps=1e-6,
                            rope_theta=10000.0, qkv_bias=False, num_experts=8, experts_per_token=2,
                            expert_intermediate_size=128, norm_topk_prob=True, name="tiny-moe"),
}

ALIASES = {
    "Qwen/Qwen2.5-14B": "qwen2.5-14b", "Qwen/Qwen2.5-14B-Instruct": "qwen2.5-14b",
    "Qwen/Qwen2.5-7B": "qwen2.5-7b", "Qwen/Qwen2.5-7B-Instruct": "qwen2.5-7b",
    "Qwen/Qwen3-8B": "qwen3-8b", "Qwen/Qwen3-30B-A3B": "qwen3-30b-a3b",
    "Qwen/Qwen2.5-0.5B": "qwen2.5-0.5b", "Qwen/Qwen2.5-0.5B-Instruct": "qwen2.5-0.5b",
    "meta-llama/Llama-3.2-1B": "llama-3.2-1b", "distilbert/distilgpt2": "distilgpt2",
    "meta-llama/Llama-3.1-8B": "llama-3.1-8b", "meta-llama/Llama-3.1-8B-Instruct": "llama-3.1-8b",
    "mistralai/Mixtral-8x7B-v0.1": "mixtral-8x7b", "mistralai/Mixtral-8x7B-Instruct-v0.1": "mixtral-8x7b",
    "openai-community/gpt2": "gpt2", "qwen2.5-14b-arch": "qwen2.5-14b", "qwen2.5-7b-arch": "qwen2.5-7b",
}


def get_config(name_or_path: str) -> ModelConfig:
    """Preset name, HF repo alias of a preset, or a local directory with config.json."""
    if os.path.isdir(name_or_path) and os.path.exists(os.path.join(name_or_path, "config.json")):
        return ModelConfig.from_pretrained_dir(name_or_path)
    key = ALIASES.get(name_or_path, name_or_path).lower()
    if key in PRESETS:
        return PRESETS[key]
    raise KeyError(f"unknown model '{name_or_path}' (presets: {sorted(PRESETS)})")
