"""NVFP4 checkpoints: the reference's quantized layout, ModelOpt-style tensors, and the
conversions to this package's NVFP4Weight.

Layouts on disk (per quantised linear layer `<module>`):
  reference   <module>.w_qdata            uint8 [N, K/2]   e2m1 codes, element 2i in
                                                           the low nibble of byte i
              <module>.w_scale            uint8 [N*K/16]   e4m3 block scales (16 K
                                                           elements) in 512-byte atoms of
                                                           128 rows x 4 blocks
              <module>.w_per_tensor_scale fp32  []         per-tensor scale
              <module>.w_scale_row        bf16  [N, K/16]  block scale x per-tensor
                                                           scale (GEMV helper; only read
                                                           when w_scale is absent)
  ModelOpt    <module>.weight             uint8 [N, K/2]   codes as above
              <module>.weight_scale       e4m3  [N, K/16]  row-major block scales
              <module>.weight_scale_2     fp32  []         per-tensor scale
              (<module>.input_scale is ignored: activations stay 16-bit at decode and
              are quantised per token at prefill)
In both, w[n, k] = e2m1(code) * e4m3(scale[n, k // 16]) * per_tensor_scale, the NVFP4
convention this package quantises to.  The block-scale atoms are byte-for-byte the
layout csrc/nvfp4_bs.cu reads (NVFP4Weight.s_atoms), and the row-major codes are its
q_rows, so a reference checkpoint is used without re-quantisation; only the decode
kernel's fragment order (NVFP4Weight.q / .s) is rebuilt, by a fixed permutation.

Reference parity: core/nvfp4_direct.py:67-81 (_from_blocked: the atom layout),
core/nvfp4_direct.py:95-219 (DirectFP4Linear buffers w_qdata / w_scale /
w_per_tensor_scale / w_scale_row), core/backends.py:1051-1118 (quantise, then swap in
DirectFP4Linear).  The buffer names are kept so checkpoints move between the two.
"""
from __future__ import annotations

from typing import Dict, List, Optional, Sequence

import torch

from .nvfp4 import NVFP4Weight, atoms_to_sf, sf_to_atoms

REF_PARTS = {"w_qdata": "codes", "w_scale": "atoms", "w_per_tensor_scale": "gs", "w_scale_row": "scale_row"}
MODELOPT_PARTS = {"weight_scale": "scale_rm", "weight_scale_2": "gs", "input_scale": "ignore"}


# ---------------------------------------------------------------- permutations
def _unpack(codes: torch.Tensor) -> torch.Tensor:
    """uint8 [N, K/2] -> nibbles uint8 [N, K] (element 2i = low nibble of byte i)."""
    return torch.stack([codes & 15, codes >> 4], dim=-1).reshape(codes.shape[0], -1)


def _pack(nib: torch.Tensor) -> torch.Tensor:
    """nibbles [..., 2n] -> bytes [..., n], element 2i in the low nibble."""
    return (nib[..., 0::2] | (nib[..., 1::2] << 4)).to(torch.uint8)


def fragment_order(codes: torch.Tensor, s8: torch.Tensor):
    """Row-major codes [N, K/2] and row-major e4m3 scale bytes [N, K/16] -> the decode
    kernel's fragment-order bytes (q [N*K/2], s [N*K/16]); any device.

    Fragment order (csrc/nvfp4.cu): for each 16-row strip and 64-column tile, lane l of
    a warp holds, for k16 step j and register i, the two codes at row
    16 strip + l/4 + 8 (i & 1), columns 64 tile + 16 j + 2 (l % 4) + 8 (i >> 1) + {0, 1};
    its scale bytes are rows 16 strip + r + 8 h, block 4 tile + j."""
    N, K = codes.shape[0], codes.shape[1] * 2
    if N % 16 or K % 64:
        raise ValueError(f"nvfp4: N must be a multiple of 16 and K of 64, got {N}x{K}")
    nib = _unpack(codes)
    # row = 16 st + 8 rh + rl; col = 64 tl + 16 j + 8 ch + 2 cl + e
    v = nib.view(N // 16, 2, 8, K // 64, 4, 2, 4, 2)            # st rh rl tl j ch cl e
    f = v.permute(0, 3, 2, 6, 4, 5, 1, 7)                       # st tl rl cl j ch rh e
    q = _pack(f.reshape(-1))
    sv = s8.reshape(N, K // 16).view(N // 16, 2, 8, K // 64, 4)   # st h r tl j
    s = sv.permute(0, 3, 2, 4, 1).reshape(-1).contiguous()      # st tl r j h
    return q.contiguous(), s


def rows_order(w: NVFP4Weight):
    """Inverse of fragment_order: (codes [N, K/2], s8 [N, K/16]) row-major."""
    N, K = w.N, w.K
    q = w.q.reshape(-1)
    nib = torch.stack([q & 15, q >> 4], dim=-1).view(N // 16, K // 64, 8, 4, 4, 2, 2, 2)   # st tl rl cl j ch rh e
    v = nib.permute(0, 6, 2, 1, 4, 5, 3, 7).reshape(N, K)                                    # st rh rl tl j ch cl e
    s = w.s.view(N // 16, K // 64, 8, 4, 2).permute(0, 4, 2, 1, 3).reshape(N, K // 16)
    return _pack(v), s.contiguous()


# ---------------------------------------------------------------- construction
def from_rows(codes: torch.Tensor, s8: torch.Tensor, gs, device=None) -> NVFP4Weight:
    """NVFP4Weight from row-major codes [N, K/2], row-major e4m3 scale bytes [N, K/16]
    and the per-tensor scale (both layouts of the weight are built: fragment order for
    decode, rows + scale atoms for the block-scaled prefill GEMM when N % 128 == 0 and
    K % 256 == 0)."""
    dev = torch.device(device) if device is not None else codes.device
    codes = codes.to(dev).view(torch.uint8).contiguous()
    s8 = s8.to(dev).view(torch.uint8).reshape(codes.shape[0], -1).contiguous()
    N, K = codes.shape[0], codes.shape[1] * 2
    g = torch.as_tensor(gs, dtype=torch.float32).reshape(1).to(dev)
    q, s = fragment_order(codes, s8)
    qr = sa = None
    if N % 128 == 0 and K % 256 == 0:
        qr, sa = codes, sf_to_atoms(s8)
    return NVFP4Weight(q, s, g, N, K, qr, sa)


def from_reference(w_qdata: torch.Tensor, w_scale: Optional[torch.Tensor], w_per_tensor_scale,
                   w_scale_row: Optional[torch.Tensor] = None, device=None) -> NVFP4Weight:
    """The reference's DirectFP4Linear buffers -> NVFP4Weight."""
    N, K = w_qdata.shape[0], w_qdata.shape[1] * 2
    gs = torch.as_tensor(w_per_tensor_scale, dtype=torch.float32).reshape(1)
    if w_scale is not None:
        a = w_scale.reshape(-1).view(torch.uint8)
        rows = (N + 127) // 128 * 128
        nb = (K // 16 + 3) // 4 * 4
        s8 = atoms_to_sf(a, rows, nb * 16)[:N, :K // 16]
    elif w_scale_row is not None:
        # block scale x per-tensor scale in bf16: e4m3 values are exact in bf16, so
        # dividing out the per-tensor scale and rounding to e4m3 recovers the bytes
        s8 = (w_scale_row.float() / gs.to(w_scale_row.device)).to(torch.float8_e4m3fn).view(torch.uint8)
    else:
        raise ValueError("reference NVFP4 layer without w_scale or w_scale_row")
    return from_rows(w_qdata, s8, gs, device)


def from_modelopt(weight: torch.Tensor, weight_scale: torch.Tensor, weight_scale_2, device=None) -> NVFP4Weight:
    """ModelOpt-style NVFP4 tensors -> NVFP4Weight."""
    return from_rows(weight, weight_scale.view(torch.uint8), weight_scale_2, device)


def to_reference(w: NVFP4Weight) -> Dict[str, torch.Tensor]:
    """NVFP4Weight -> the reference's DirectFP4Linear buffers (host tensors)."""
    codes, s8 = rows_order(w)
    rows = (w.N + 127) // 128 * 128
    nb = (w.K // 16 + 3) // 4 * 4
    sp = torch.zeros(rows, nb, dtype=torch.uint8, device=s8.device)
    sp[:w.N, :w.K // 16] = s8
    gs = w.gs.float().reshape(())
    srow = (s8.view(torch.float8_e4m3fn).float() * gs).to(torch.bfloat16)
    return {"w_qdata": codes.cpu(), "w_scale": sf_to_atoms(sp).cpu(), "w_per_tensor_scale": gs.cpu().clone(),
            "w_scale_row": srow.cpu()}


def to_modelopt(w: NVFP4Weight) -> Dict[str, torch.Tensor]:
    codes, s8 = rows_order(w)
    return {"weight": codes.cpu(), "weight_scale": s8.view(torch.float8_e4m3fn).cpu(),
            "weight_scale_2": w.gs.float().reshape(()).cpu().clone()}


# ---------------------------------------------------------------- fusing and sharding
def _rescaled_rows(w: NVFP4Weight, gs_common: torch.Tensor):
    """Row-major (codes, e4m3 bytes) of w expressed against a larger per-tensor scale:
    block scales s * gs / gs_common, rounded to e4m3 (exact when the scales agree)."""
    codes, s8 = rows_order(w)
    g, gc = w.gs.float().reshape(()).to(s8.device), gs_common.float().reshape(()).to(s8.device)
    if torch.equal(g, gc):
        return codes, s8
    sf = s8.view(torch.float8_e4m3fn).float() * (g / gc)
    return codes, sf.to(torch.float8_e4m3fn).view(torch.uint8)


def concat_rows(parts: Sequence[NVFP4Weight], interleave_pairs: bool = False) -> NVFP4Weight:
    """Stacks weights along N (q / k / v -> qkv) or, with interleave_pairs, interleaves
    the rows of two weights (gate_0, up_0, gate_1, ...).  Different per-tensor scales
    are brought to their maximum by rescaling the block scales."""
    gs = torch.stack([p.gs.float().reshape(()) for p in parts]).amax()
    rows = [_rescaled_rows(p, gs) for p in parts]
    if interleave_pairs:
        (cg, sg), (cu, su) = rows
        codes = torch.stack([cg, cu], 1).reshape(-1, cg.shape[1])
        s8 = torch.stack([sg, su], 1).reshape(-1, sg.shape[1])
    else:
        codes = torch.cat([c for c, _ in rows], 0)
        s8 = torch.cat([s for _, s in rows], 0)
    return from_rows(codes, s8, gs, parts[0].q.device)


def slice_rows(w: NVFP4Weight, start: int, end: int) -> NVFP4Weight:
    codes, s8 = rows_order(w)
    return from_rows(codes[start:end], s8[start:end], w.gs, w.q.device)


def slice_cols(w: NVFP4Weight, start: int, end: int) -> NVFP4Weight:
    """Columns [start, end) of K (multiples of 64)."""
    if start % 64 or end % 64:
        raise ValueError("nvfp4: column slices must be multiples of 64")
    codes, s8 = rows_order(w)
    return from_rows(codes[:, start // 2:end // 2], s8[:, start // 16:end // 16], w.gs, w.q.device)


def shard_nvfp4(cfg, name: str, w: NVFP4Weight, rank: int, size: int) -> NVFP4Weight:
    """Tensor-parallel shard of a quantised projection, as models.weights.shard_tensor
    does for bf16 (column-parallel rows, row-parallel columns)."""
    if size == 1:
        return w
    base = name.split(".")[-1]
    if base == "qkv_w":
        D = cfg.head_dim
        hq = cfg.num_heads // size
        q = slice_rows(w, rank * hq * D, (rank + 1) * hq * D)
        if cfg.num_kv_heads >= size:
            kvh = cfg.num_kv_heads // size
            k0 = rank * kvh * D
        else:
            kvh = 1
            k0 = ((rank * cfg.num_kv_heads) // size) * D
        k = slice_rows(w, cfg.q_size + k0, cfg.q_size + k0 + kvh * D)
        v = slice_rows(w, cfg.q_size + cfg.kv_size + k0, cfg.q_size + cfg.kv_size + k0 + kvh * D)
        return concat_rows([q, k, v])
    if base in ("gate_up_w", "fc_w"):
        n = w.N // size
        return slice_rows(w, rank * n, (rank + 1) * n)
    if base in ("o_w", "down_w", "proj_w"):
        n = w.K // size
        return slice_cols(w, rank * n, (rank + 1) * n)
    return w


def assemble(parts: Dict[str, Dict[str, torch.Tensor]], role: str) -> NVFP4Weight:
    """One HF module's quantised tensors (reference or ModelOpt names) -> NVFP4Weight."""
    if "codes" in parts:
        return from_reference(parts["codes"], parts.get("atoms"), parts["gs"], parts.get("scale_row"))
    if "codes_mo" in parts:
        return from_modelopt(parts["codes_mo"], parts["scale_rm"], parts["gs"])
    raise ValueError(f"incomplete NVFP4 tensors for {role}: {sorted(parts)}")


def fuse_module_weights(base: str, per_role: Dict[str, NVFP4Weight]) -> NVFP4Weight:
    """q / k / v or gate / up module weights -> the internal fused tensor."""
    if base == "qkv_w":
        return concat_rows([per_role["q"], per_role["k"], per_role["v"]])
    if base in ("gate_up_w", "shared_gate_up_w"):
        return concat_rows([per_role["gate"], per_role["up"]], interleave_pairs=True)
    return per_role["copy"]


def save_nvfp4_checkpoint(weights: Dict[str, object], cfg, path: str, layout: str = "reference") -> None:
    """Writes a model whose projections are NVFP4Weights as an HF-named safetensors
    checkpoint in the reference's layout (or "modelopt"), unfused per HF module, with
    the unquantised tensors (embeddings, norms, biases, lm_head) in bf16."""
    import json
    import os

    from safetensors.torch import save_file

    from ..models.weights import deinterleave_gate_up
    os.makedirs(path, exist_ok=True)
    conv = to_reference if layout == "reference" else to_modelopt
    out: Dict[str, torch.Tensor] = {}
    plain: Dict[str, torch.Tensor] = {}
    for k, t in weights.items():
        if isinstance(t, NVFP4Weight):
            _, i, n = k.split(".", 2)
            pre = f"model.layers.{i}."
            if n == "qkv_w":
                mods = {"self_attn.q_proj": slice_rows(t, 0, cfg.q_size),
                        "self_attn.k_proj": slice_rows(t, cfg.q_size, cfg.q_size + cfg.kv_size),
                        "self_attn.v_proj": slice_rows(t, cfg.q_size + cfg.kv_size, cfg.q_size + 2 * cfg.kv_size)}
            elif n == "gate_up_w":
                codes, s8 = rows_order(t)
                mods = {"mlp.gate_proj": from_rows(codes[0::2], s8[0::2], t.gs),
                        "mlp.up_proj": from_rows(codes[1::2], s8[1::2], t.gs)}
            elif n == "o_w":
                mods = {"self_attn.o_proj": t}
            elif n == "down_w":
                mods = {"mlp.down_proj": t}
            else:
                raise ValueError(f"no HF name for quantised {k}")
            for m, w in mods.items():
                for part, v in conv(w).items():
                    out[f"{pre}{m}.{part}"] = v.contiguous()
        else:
            plain[k] = t
    if plain:
        from ..models.weights import save_safetensors
        tmp = os.path.join(path, "_plain")
        save_safetensors(plain, cfg, tmp)
        from safetensors import safe_open
        with safe_open(os.path.join(tmp, "model.safetensors"), framework="pt") as f:
            for name in f.keys():
                out[name] = f.get_tensor(name)
        for fn in os.listdir(tmp):
            os.unlink(os.path.join(tmp, fn))
        os.rmdir(tmp)
    save_file(out, os.path.join(path, "model.safetensors"))
    with open(os.path.join(path, "config.json"), "w") as f:
        json.dump({**cfg.to_hf_config(), "quantization_config": {"quant_method": "nvfp4", "layout": layout}}, f)
