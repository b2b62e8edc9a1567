"""Weight containers: random initialisation, HF safetensors loading, sharding.

Internal layout (per layer ``layers.{i}.``):
  in_norm_w [H] (+ in_norm_b for gpt2), qkv_w [(Hq+2KH)*D, H], qkv_b, o_w [H, Hq*D] (+ o_b),
  post_norm_w [H] (+ post_norm_b),
  dense SwiGLU: gate_up_w [2I, H] with rows interleaved (gate_j, up_j) so the GEMM
                epilogue can apply silu(gate)*up in registers, down_w [H, I]
  gpt2 MLP:     fc_w [I, H], fc_b, proj_w [H, I], proj_b
  MoE:          router_w [E, H], experts_gate_up_w [E, 2I, H] (interleaved), experts_down_w [E, H, I]
                (+ shared_gate_up_w, shared_down_w, shared_gate_w [1, H])
Globals: embed [V, H], pos_embed [P, H] (gpt2), final_norm_w (+ final_norm_b), lm_head [V, H].

Reference parity: the reference never owns weights (HF `from_pretrained` +
accelerate placement, core/backends.py:1185-1412); the loaders here read the same
HF safetensors names directly, shard-aware, without transformers.
"""
from __future__ import annotations

import json
import os
from typing import Dict, Iterable, Optional, Tuple

import torch

from .config import ModelConfig

Weights = Dict[str, torch.Tensor]


def interleave_gate_up(gate: torch.Tensor, up: torch.Tensor) -> torch.Tensor:
    """[I, H] x 2 -> [2I, H] with rows (gate_0, up_0, gate_1, up_1, ...)."""
    I = gate.shape[0]
    return torch.stack([gate, up], dim=1).reshape(2 * I, *gate.shape[1:])


def deinterleave_gate_up(gu: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor]:
    return gu[0::2], gu[1::2]


def layer_shapes(cfg: ModelConfig, tp_rank: int = 0, tp_size: int = 1) -> Dict[str, Tuple[int, ...]]:
    """Shapes of one layer's tensors for this tensor-parallel rank."""
    H, D = cfg.hidden_size, cfg.head_dim
    assert cfg.num_heads % tp_size == 0, "num_heads must divide by tp_size"
    hq = cfg.num_heads // tp_size
    kvh = max(1, cfg.num_kv_heads // tp_size)
    s: Dict[str, Tuple[int, ...]] = {
        "in_norm_w": (H,), "post_norm_w": (H,),
        "qkv_w": ((hq + 2 * kvh) * D, H), "o_w": (H, hq * D),
    }
    if cfg.qkv_bias:
        s["qkv_b"] = ((hq + 2 * kvh) * D,)
    if cfg.qk_norm:
        s["q_norm_w"] = (D,)
        s["k_norm_w"] = (D,)
    if cfg.is_gpt2:
        I = cfg.intermediate_size // tp_size
        s.update({"in_norm_b": (H,), "post_norm_b": (H,), "o_b": (H,), "fc_w": (I, H), "fc_b": (I,),
                  "proj_w": (H, I), "proj_b": (H,)})
    elif cfg.is_moe:
        E, I = cfg.num_experts, cfg.expert_intermediate_size
        s.update({"router_w": (E, H), "experts_gate_up_w": (E, 2 * I, H), "experts_down_w": (E, H, I)})
        if cfg.shared_expert_intermediate_size:
            Is = cfg.shared_expert_intermediate_size // tp_size
            s.update({"shared_gate_up_w": (2 * Is, H), "shared_down_w": (H, Is), "shared_gate_w": (1, H)})
    else:
        I = cfg.intermediate_size // tp_size
        s.update({"gate_up_w": (2 * I, H), "down_w": (H, I)})
    return s


def random_weights(cfg: ModelConfig, *, device="cpu", dtype=torch.bfloat16, seed: int = 0,
                   layers: Optional[Iterable[int]] = None, embed: bool = True, head: bool = True,
                   tp_rank: int = 0, tp_size: int = 1, std: float = 0.02, ep_rank: int = 0,
                   ep_size: int = 1) -> Weights:
    """N(0, std) matrices, unit norm weights, zero norm biases; deterministic in `seed`.

    Each tensor gets its own generator seeded from (seed, name), so a layer's values do
    not depend on which other layers this process builds (pipeline stages of a split
    model hold exactly the tensors of the single-device model).  With tp_size > 1 the
    full tensor is generated and this rank's shard is kept, so TP ranks hold slices of
    the TP=1 model.  With ep_size > 1 only this expert-parallel rank's experts are kept
    (generated in full and sliced, so EP ranks hold slices of the single-GPU model).
    """
    layers = range(cfg.num_layers) if layers is None else layers
    dev = torch.device(device)
    out: Weights = {}

    def gen(name: str, shape, kind: str = "mat") -> torch.Tensor:
        if kind == "ones":
            return torch.ones(shape, dtype=dtype, device=dev)
        if kind == "zeros":
            return torch.zeros(shape, dtype=dtype, device=dev)
        h = abs(hash_name(name)) % (2 ** 31)
        g = torch.Generator(device=dev).manual_seed(seed * 1_000_003 + h)
        t = torch.empty(shape, dtype=torch.float32 if dev.type == "cpu" else dtype, device=dev)
        t.normal_(0.0, std, generator=g)
        return t.to(dtype)

    full = layer_shapes(cfg, 0, 1)
    for i in layers:
        for n, shp in full.items():
            kind = "ones" if n.endswith("norm_w") else ("zeros" if n.endswith("norm_b") else "mat")
            t = gen(f"layers.{i}.{n}", shp, kind)
            if tp_size > 1:
                t = shard_tensor(cfg, n, t, tp_rank, tp_size)
            if ep_size > 1 and n.startswith("experts_"):
                t = _ep_slice(t, ep_rank, ep_size)
            out[f"layers.{i}.{n}"] = t
    H = cfg.hidden_size
    if embed:
        out["embed"] = gen("embed", (cfg.vocab_size, H))
        if cfg.is_gpt2:
            out["pos_embed"] = gen("pos_embed", (cfg.max_position, H))
    if head:
        out["final_norm_w"] = gen("final_norm_w", (H,), "ones")
        if cfg.is_gpt2:
            out["final_norm_b"] = gen("final_norm_b", (H,), "zeros")
        if cfg.tie_embeddings:
            out["lm_head"] = out["embed"] if "embed" in out else gen("embed", (cfg.vocab_size, H))
        else:
            out["lm_head"] = gen("lm_head", (cfg.vocab_size, H))
        if tp_size > 1:
            out["lm_head"] = shard_tensor(cfg, "lm_head", out["lm_head"], tp_rank, tp_size)
    return out


def _ep_slice(t: torch.Tensor, rank: int, size: int) -> torch.Tensor:
    n = t.shape[0] // size
    if n * size != t.shape[0]:
        raise ValueError(f"{t.shape[0]} experts do not divide over {size} expert-parallel ranks")
    return t[rank * n:(rank + 1) * n].clone()


def hash_name(name: str) -> int:
    """Stable (process-independent) 63-bit hash of a tensor name (FNV-1a)."""
    h = 0xCBF29CE484222325
    for ch in name.encode():
        h ^= ch
        h = (h * 0x100000001B3) & 0xFFFFFFFFFFFFFFFF
    return h >> 1


# ---------------------------------------------------------------------------- sharding
def _qkv_split(cfg: ModelConfig, t: torch.Tensor, rank: int, size: int) -> torch.Tensor:
    D = cfg.head_dim
    q, k, v = torch.split(t, [cfg.q_size, cfg.kv_size, cfg.kv_size], dim=0)
    hq = cfg.num_heads // size
    kvh = cfg.num_kv_heads // size if cfg.num_kv_heads >= size else 1
    if cfg.num_kv_heads >= size:
        ks = k[rank * kvh * D:(rank + 1) * kvh * D]
        vs = v[rank * kvh * D:(rank + 1) * kvh * D]
    else:  # replicate the kv head that this rank's q heads use
        grp = (rank * cfg.num_kv_heads) // size
        ks = k[grp * D:(grp + 1) * D]
        vs = v[grp * D:(grp + 1) * D]
    return torch.cat([q[rank * hq * D:(rank + 1) * hq * D], ks, vs], dim=0).contiguous()


def shard_tensor(cfg: ModelConfig, name: str, t: torch.Tensor, rank: int, size: int) -> torch.Tensor:
    """Column-parallel: qkv, gate_up, fc (rows); row-parallel: o, down, proj (cols);
    vocab-parallel lm_head (rows).  Norms, router, biases of row-parallel layers and
    embeddings are replicated (row-parallel biases are added once, after the reduce)."""
    if size == 1:
        return t
    base = name.split(".")[-1]
    if base in ("qkv_w", "qkv_b"):
        return _qkv_split(cfg, t, rank, size)
    if base in ("gate_up_w", "shared_gate_up_w"):
        n = t.shape[0] // size
        return t[rank * n:(rank + 1) * n].contiguous()      # pairs stay together (n even)
    if base in ("fc_w", "fc_b"):
        n = t.shape[0] // size
        return t[rank * n:(rank + 1) * n].contiguous()
    if base in ("o_w", "down_w", "proj_w", "shared_down_w"):
        n = t.shape[1] // size
        return t[:, rank * n:(rank + 1) * n].contiguous()
    if base == "lm_head":
        n = (t.shape[0] + size - 1) // size
        s = t[rank * n:(rank + 1) * n]
        if s.shape[0] < n:
            s = torch.cat([s, torch.zeros(n - s.shape[0], t.shape[1], dtype=t.dtype, device=t.device)], 0)
        return s.contiguous()
    return t


# ---------------------------------------------------------------------------- HF checkpoints
def _hf_map(cfg: ModelConfig, name: str) -> Optional[Tuple[str, str]]:
    """HF tensor name -> (internal name, role); role tells how to assemble fused tensors."""
    if cfg.is_gpt2:
        n = name[len("transformer."):] if name.startswith("transformer.") else name
        if n == "wte.weight":
            return "embed", "copy"
        if n == "wpe.weight":
            return "pos_embed", "copy"
        if n == "ln_f.weight":
            return "final_norm_w", "copy"
        if n == "ln_f.bias":
            return "final_norm_b", "copy"
        if n.startswith("h."):
            parts = n.split(".")
            i = parts[1]
            rest = ".".join(parts[2:])
            m = {"ln_1.weight": "in_norm_w", "ln_1.bias": "in_norm_b", "ln_2.weight": "post_norm_w",
                 "ln_2.bias": "post_norm_b", "attn.c_attn.weight": "qkv_w", "attn.c_attn.bias": "qkv_b",
                 "attn.c_proj.weight": "o_w", "attn.c_proj.bias": "o_b", "mlp.c_fc.weight": "fc_w",
                 "mlp.c_fc.bias": "fc_b", "mlp.c_proj.weight": "proj_w", "mlp.c_proj.bias": "proj_b"}.get(rest)
            if m is None:
                return None
            role = "conv1d" if rest.endswith("weight") and not rest.startswith("ln") else "copy"
            return f"layers.{i}.{m}", role
        return None
    if name == "model.embed_tokens.weight":
        return "embed", "copy"
    if name == "model.norm.weight":
        return "final_norm_w", "copy"
    if name == "lm_head.weight":
        return "lm_head", "copy"
    if not name.startswith("model.layers."):
        return None
    parts = name.split(".")
    i = parts[2]
    rest = ".".join(parts[3:])
    pre = f"layers.{i}."
    simple = {"input_layernorm.weight": ("in_norm_w", "copy"),
              "self_attn.q_norm.weight": ("q_norm_w", "copy"), "self_attn.k_norm.weight": ("k_norm_w", "copy"),
              "post_attention_layernorm.weight": ("post_norm_w", "copy"),
              "self_attn.o_proj.weight": ("o_w", "copy"),
              "self_attn.q_proj.weight": ("qkv_w", "q"), "self_attn.k_proj.weight": ("qkv_w", "k"),
              "self_attn.v_proj.weight": ("qkv_w", "v"), "self_attn.q_proj.bias": ("qkv_b", "q"),
              "self_attn.k_proj.bias": ("qkv_b", "k"), "self_attn.v_proj.bias": ("qkv_b", "v"),
              "mlp.gate_proj.weight": ("gate_up_w", "gate"), "mlp.up_proj.weight": ("gate_up_w", "up"),
              "mlp.down_proj.weight": ("down_w", "copy"), "mlp.gate.weight": ("router_w", "copy"),
              "mlp.shared_expert.gate_proj.weight": ("shared_gate_up_w", "gate"),
              "mlp.shared_expert.up_proj.weight": ("shared_gate_up_w", "up"),
              "mlp.shared_expert.down_proj.weight": ("shared_down_w", "copy"),
              "mlp.shared_expert_gate.weight": ("shared_gate_w", "copy")}
    if rest in simple:
        n, role = simple[rest]
        return pre + n, role
    if rest == "block_sparse_moe.gate.weight":                 # Mixtral router
        return pre + "router_w", "copy"
    if rest.startswith("mlp.experts.") or rest.startswith("block_sparse_moe.experts."):
        e = rest.split(".")[2]
        tail = ".".join(rest.split(".")[3:])
        # Qwen-MoE names, and Mixtral's w1 (gate) / w3 (up) / w2 (down)
        m = {"gate_proj.weight": ("experts_gate_up_w", f"egate:{e}"), "w1.weight": ("experts_gate_up_w", f"egate:{e}"),
             "up_proj.weight": ("experts_gate_up_w", f"eup:{e}"), "w3.weight": ("experts_gate_up_w", f"eup:{e}"),
             "down_proj.weight": ("experts_down_w", f"edown:{e}"),
             "w2.weight": ("experts_down_w", f"edown:{e}")}.get(tail)
        if m:
            return pre + m[0], m[1]
    return None


# quantised-tensor suffixes of one HF linear module: the reference's DirectFP4Linear
# buffers and ModelOpt-style NVFP4 tensors (quant/nvfp4_io.py)
_NVFP4_SUFFIX = {"w_qdata": "codes", "w_scale": "atoms", "w_per_tensor_scale": "gs", "w_scale_row": "scale_row",
                 "weight_scale": "scale_rm", "weight_scale_2": "gs", "input_scale": None}


def _tp_slice(cfg: ModelConfig, iname: str, role: str, shape, rank: int, size: int):
    """(rows, cols) slices of an HF tensor that this tensor-parallel rank keeps, or None
    (read whole).  Fused q/k/v and gate/up are sliced per part, so assembling the
    parts gives shard_tensor's result of the fused tensor."""
    if size == 1 or cfg.is_gpt2:
        return None
    base = iname.split(".")[-1]
    D = cfg.head_dim
    if base in ("qkv_w", "qkv_b"):
        if role == "q":
            hq = cfg.num_heads // size
            return slice(rank * hq * D, (rank + 1) * hq * D), None
        if cfg.num_kv_heads >= size:
            kvh = cfg.num_kv_heads // size
            return slice(rank * kvh * D, (rank + 1) * kvh * D), None
        grp = (rank * cfg.num_kv_heads) // size
        return slice(grp * D, (grp + 1) * D), None
    if base in ("gate_up_w", "shared_gate_up_w") and role in ("gate", "up"):
        n = shape[0] // size
        return slice(rank * n, (rank + 1) * n), None
    if base in ("o_w", "down_w", "shared_down_w") and len(shape) == 2:
        n = shape[1] // size
        return None, slice(rank * n, (rank + 1) * n)
    if base == "lm_head":
        n = (shape[0] + size - 1) // size
        return slice(rank * n, min(shape[0], (rank + 1) * n)), None
    return None


def _place(out: Weights, parts: Dict[str, Dict[str, torch.Tensor]], iname: str, role: str,
           t: torch.Tensor) -> None:
    """One mapped HF tensor: whole tensors (GPT-2 Conv1D weights transposed to [out, in])
    go to `out`, pieces of fused tensors (q / k / v, gate / up, one expert) to `parts`."""
    if role == "conv1d":
        out[iname] = t.t().contiguous()
    elif role == "copy":
        out[iname] = t
    else:
        parts.setdefault(iname, {})[role] = t


def _fuse_parts(out: Weights, parts: Dict[str, Dict[str, torch.Tensor]], experts) -> None:
    """q|k|v rows concatenated, gate / up interleaved, experts stacked (in id order)."""
    for iname, p in parts.items():
        base = iname.split(".")[-1]
        if base in ("qkv_w", "qkv_b"):
            out[iname] = torch.cat([p["q"], p["k"], p["v"]], 0)
        elif base in ("gate_up_w", "shared_gate_up_w"):
            out[iname] = interleave_gate_up(p["gate"], p["up"])
        elif base == "experts_gate_up_w":
            out[iname] = torch.stack([interleave_gate_up(p[f"egate:{e}"], p[f"eup:{e}"]) for e in sorted(experts)])
        elif base == "experts_down_w":
            out[iname] = torch.stack([p[f"edown:{e}"] for e in sorted(experts)])


def weights_from_state_dict(cfg: ModelConfig, state_dict, *, device="cpu", dtype=torch.bfloat16) -> Weights:
    """Internal weights from an in-memory HF state dict (a loaded `PreTrainedModel`'s
    `state_dict()`): the name mapping and fusing of `load_safetensors`, one device, no
    sharding.  Transformers 5 stores MoE experts fused ([E, 2I, H] gate_up_proj,
    [E, H, I] down_proj); those are split back into per-expert pieces here."""
    out: Weights = {}
    parts: Dict[str, Dict[str, torch.Tensor]] = {}
    experts = range(cfg.num_experts) if cfg.is_moe else range(0)
    for name, t in state_dict.items():
        t = t.detach()
        if name.endswith("mlp.experts.gate_up_proj") or name.endswith("mlp.experts.down_proj"):
            pre = name.rsplit(".", 1)[0]
            for e in experts:
                if name.endswith("gate_up_proj"):
                    g, u = t[e].chunk(2, 0) if t.shape[1] == 2 * cfg.expert_intermediate_size else t[e].t().chunk(2, 0)
                    for part, v in (("gate_proj", g), ("up_proj", u)):
                        m = _hf_map(cfg, f"{pre}.{e}.{part}.weight")
                        _place(out, parts, m[0], m[1], v)
                else:
                    v = t[e] if t.shape[1] == cfg.hidden_size else t[e].t()
                    m = _hf_map(cfg, f"{pre}.{e}.down_proj.weight")
                    _place(out, parts, m[0], m[1], v)
            continue
        m = _hf_map(cfg, name)
        if m is None:
            continue
        _place(out, parts, m[0], m[1], t)
    _fuse_parts(out, parts, experts)
    if "lm_head" not in out and "embed" in out:
        out["lm_head"] = out["embed"]
    res = {k: v.to(device=device, dtype=dtype).contiguous() for k, v in out.items()}
    if out.get("lm_head") is out.get("embed"):
        res["lm_head"] = res["embed"]
    return res


def _quantization_config(path: str) -> Optional[dict]:
    """The checkpoint's GPTQ / AWQ quantization_config (None for dense checkpoints and
    for the NVFP4 layouts, which are read tensor by tensor)."""
    fn = os.path.join(path, "config.json")
    if not os.path.exists(fn):
        return None
    with open(fn) as f:
        qc = json.load(f).get("quantization_config")
    if not qc or str(qc.get("quant_method", "")).lower() not in ("gptq", "awq"):
        return None
    from ..quant import int4_ckpt
    int4_ckpt.check_config(qc)
    return qc


def _wanted(cfg: ModelConfig, m: Tuple[str, str], want_layers, embed: bool, head: bool, own_experts) -> bool:
    iname, role = m
    if iname.startswith("layers."):
        if int(iname.split(".")[1]) not in want_layers:
            return False
    elif iname in ("embed", "pos_embed") and not embed and not (head and cfg.tie_embeddings):
        return False
    elif iname in ("final_norm_w", "final_norm_b", "lm_head") and not head:
        return False
    return not (":" in role and int(role.split(":")[1]) not in own_experts)


def load_safetensors(path: str, cfg: ModelConfig, *, device="cpu", dtype=torch.bfloat16,
                     layers: Optional[Iterable[int]] = None, embed: bool = True, head: bool = True,
                     tp_rank: int = 0, tp_size: int = 1, ep_rank: int = 0, ep_size: int = 1) -> Weights:
    """Reads an HF checkpoint directory (*.safetensors), keeping only the tensors this
    stage / rank needs, fusing q/k/v and gate/up into the internal layout.

    Tensor-parallel ranks read only their slices (safetensors get_slice), and
    expert-parallel ranks only their experts, so no rank reads the whole checkpoint.
    Projections stored NVFP4-quantised (the reference's DirectFP4Linear buffers
    w_qdata / w_scale / w_per_tensor_scale, or ModelOpt weight / weight_scale /
    weight_scale_2) load as NVFP4Weight without re-quantisation.  GPTQ / AWQ checkpoints
    (quantization_config in config.json) are dequantised per linear layer
    (quant/int4_ckpt.py) into the dense layout."""
    from safetensors import safe_open

    want_layers = set(range(cfg.num_layers) if layers is None else layers)
    files = sorted(f for f in os.listdir(path) if f.endswith(".safetensors"))
    if not files:
        raise FileNotFoundError(f"no .safetensors files in {path}")
    qc = _quantization_config(path)
    n_exp = cfg.num_experts // ep_size if cfg.is_moe else 0
    own_experts = set(range(ep_rank * n_exp, (ep_rank + 1) * n_exp))
    parts: Dict[str, Dict[str, torch.Tensor]] = {}
    nv_parts: Dict[str, Dict[str, Dict[str, torch.Tensor]]] = {}
    int_parts: Dict[Tuple[str, str], Dict[str, torch.Tensor]] = {}
    out: Weights = {}
    sharded = set()
    for fn in files:
        with safe_open(os.path.join(path, fn), framework="pt", device="cpu") as f:
            for name in f.keys():
                mod, _, leaf = name.rpartition(".")
                if qc is not None and leaf in ("qweight", "qzeros", "scales", "g_idx"):
                    m = _hf_map(cfg, mod + ".weight")
                    if m is not None and _wanted(cfg, m, want_layers, embed, head, own_experts):
                        int_parts.setdefault(m, {})[leaf] = f.get_tensor(name)
                    continue
                nv_part = _NVFP4_SUFFIX.get(leaf, "") if leaf in _NVFP4_SUFFIX else ""
                if nv_part is None:
                    continue                     # activation scale: not used
                m = _hf_map(cfg, mod + ".weight" if nv_part else name)
                if m is None:
                    continue
                iname, role = m
                if iname.startswith("layers."):
                    if int(iname.split(".")[1]) not in want_layers:
                        continue
                elif iname in ("embed", "pos_embed") and not embed and not (head and cfg.tie_embeddings):
                    continue
                elif iname in ("final_norm_w", "final_norm_b", "lm_head") and not head:
                    continue
                if ":" in role and int(role.split(":")[1]) not in own_experts:
                    continue                     # another expert-parallel rank's expert
                sl = f.get_slice(name)
                if not nv_part and sl.get_dtype() in ("U8", "I8") and leaf == "weight":
                    nv_part = "codes_mo"         # ModelOpt packed e2m1 codes
                if nv_part:
                    nv_parts.setdefault(iname, {}).setdefault(role, {})[nv_part] = f.get_tensor(name)
                    continue
                cut = _tp_slice(cfg, iname, role, sl.get_shape(), tp_rank, tp_size)
                if cut is None:
                    t = f.get_tensor(name)
                else:
                    rows, cols = cut
                    t = sl[rows] if cols is None else sl[:, cols]
                    t = t.contiguous()
                    sharded.add(iname)
                _place(out, parts, iname, role, t)
    if int_parts:
        from ..quant import int4_ckpt
        for (iname, role), pp in int_parts.items():
            w = int4_ckpt.dequantize_module(qc, pp)
            _place(out, parts, iname, role, w.t() if role == "conv1d" else w)
    _fuse_parts(out, parts, own_experts)
    if head and "lm_head" not in out and "embed" in out:
        out["lm_head"] = out["embed"]
    if not embed:
        out.pop("embed", None)
        out.pop("pos_embed", None)
    res: Weights = {}
    for k, t in out.items():
        if k == "lm_head" and k in sharded:
            n = (cfg.vocab_size + tp_size - 1) // tp_size
            if t.shape[0] < n:       # the last rank's slice is padded to the others' size
                t = torch.cat([t, torch.zeros(n - t.shape[0], t.shape[1], dtype=t.dtype)], 0)
        elif tp_size > 1 and k not in sharded:
            t = shard_tensor(cfg, k, t, tp_rank, tp_size)
        res[k] = t.to(device=device, dtype=dtype).contiguous()
    if "lm_head" in out and "embed" in out and out["lm_head"] is out["embed"] and tp_size == 1:
        res["lm_head"] = res["embed"]
    if nv_parts:
        from ..quant import nvfp4_io
        for iname, per_role in nv_parts.items():
            base = iname.split(".")[-1]
            mods = {role: nvfp4_io.assemble(pp, f"{iname}:{role}") for role, pp in per_role.items()}
            w = nvfp4_io.fuse_module_weights(base, mods)
            w = nvfp4_io.shard_nvfp4(cfg, iname, w, tp_rank, tp_size)
            res[iname] = nvfp4_io.from_rows(*nvfp4_io.rows_order(w), w.gs, device=device)
    return res


def save_safetensors(weights: Weights, cfg: ModelConfig, path: str) -> None:
    """Writes internal weights as an HF-named checkpoint (+ config.json)."""
    from safetensors.torch import save_file

    os.makedirs(path, exist_ok=True)
    hf: Dict[str, torch.Tensor] = {}
    if cfg.is_gpt2:
        inv = {"in_norm_w": "ln_1.weight", "in_norm_b": "ln_1.bias", "post_norm_w": "ln_2.weight",
               "post_norm_b": "ln_2.bias", "qkv_w": "attn.c_attn.weight", "qkv_b": "attn.c_attn.bias",
               "o_w": "attn.c_proj.weight", "o_b": "attn.c_proj.bias", "fc_w": "mlp.c_fc.weight",
               "fc_b": "mlp.c_fc.bias", "proj_w": "mlp.c_proj.weight", "proj_b": "mlp.c_proj.bias"}
        for k, t in weights.items():
            if k.startswith("layers."):
                _, i, n = k.split(".", 2)
                t2 = t.t().contiguous() if n.endswith("_w") and not n.endswith("norm_w") else t
                hf[f"transformer.h.{i}.{inv[n]}"] = t2.contiguous()
        hf["transformer.wte.weight"] = weights["embed"].contiguous()
        hf["transformer.wpe.weight"] = weights["pos_embed"].contiguous()
        hf["transformer.ln_f.weight"] = weights["final_norm_w"].contiguous()
        hf["transformer.ln_f.bias"] = weights["final_norm_b"].contiguous()
    else:
        for k, t in weights.items():
            if not k.startswith("layers."):
                continue
            _, i, n = k.split(".", 2)
            pre = f"model.layers.{i}."
            nw = getattr(t, "_vrm_norm_w", None)
            if nw is not None:
                # folded RMSNorm weight (LLM(fold_norms=True)): write the checkpoint's matrix
                # back.  The bf16 multiply-then-divide is not bit-exact (a last-bit
                # difference per element is possible); a column whose norm weight is 0 was
                # zeroed by the fold and is written as 0, which gives the same model
                # output since that column is multiplied by the 0 norm weight anyway.
                d = nw.float().view(1, -1)
                tf = t.float()
                t = torch.where(d == 0, torch.zeros_like(tf), tf / torch.where(d == 0, torch.ones_like(d), d)).to(t.dtype)
            if n in ("qkv_w", "qkv_b"):
                q, kk, v = torch.split(t, [cfg.q_size, cfg.kv_size, cfg.kv_size], 0)
                suf = "weight" if n == "qkv_w" else "bias"
                hf[pre + f"self_attn.q_proj.{suf}"] = q.contiguous()
                hf[pre + f"self_attn.k_proj.{suf}"] = kk.contiguous()
                hf[pre + f"self_attn.v_proj.{suf}"] = v.contiguous()
            elif n == "gate_up_w":
                g, u = deinterleave_gate_up(t)
                hf[pre + "mlp.gate_proj.weight"] = g.contiguous()
                hf[pre + "mlp.up_proj.weight"] = u.contiguous()
            elif n == "experts_gate_up_w":
                for e in range(t.shape[0]):
                    g, u = deinterleave_gate_up(t[e])
                    hf[pre + f"mlp.experts.{e}.gate_proj.weight"] = g.contiguous()
                    hf[pre + f"mlp.experts.{e}.up_proj.weight"] = u.contiguous()
            elif n == "experts_down_w":
                for e in range(t.shape[0]):
                    hf[pre + f"mlp.experts.{e}.down_proj.weight"] = t[e].contiguous()
            else:
                name = {"in_norm_w": "input_layernorm.weight", "post_norm_w": "post_attention_layernorm.weight",
                        "o_w": "self_attn.o_proj.weight", "down_w": "mlp.down_proj.weight",
                        "router_w": "mlp.gate.weight"}[n]
                hf[pre + name] = t.contiguous()
        hf["model.embed_tokens.weight"] = weights["embed"].contiguous()
        hf["model.norm.weight"] = weights["final_norm_w"].contiguous()
        if not cfg.tie_embeddings:
            hf["lm_head.weight"] = weights["lm_head"].contiguous()
    save_file({k: v.cpu() for k, v in hf.items()}, os.path.join(path, "model.safetensors"))
    with open(os.path.join(path, "config.json"), "w") as f:
        json.dump(cfg.to_hf_config(), f, indent=1)
