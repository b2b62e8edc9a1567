"""Checkpoint loading: per-rank slices (get_slice) equal sharding the full tensors, and
NVFP4 checkpoints in the reference's DirectFP4Linear layout and in the ModelOpt layout
load without re-quantisation (CPU)."""
import math

import pytest
import torch

from vramancer_b200.engine.engine import SamplingParams
from vramancer_b200.llm import LLM
from vramancer_b200.models.config import PRESETS
from vramancer_b200.models.weights import load_safetensors, random_weights, save_safetensors, shard_tensor
from vramancer_b200.quant import nvfp4 as nv
from vramancer_b200.quant import nvfp4_io as io


def _from_blocked(blocked_flat, rows, cols):
    """The reference's inverse of the blocked scale swizzle, restated (the atom layout)."""
    data = blocked_flat.float().flatten()
    R, C = math.ceil(rows / 128), math.ceil(cols / 4)
    data = data.view(R * C, 32, 4, 4).transpose(1, 2).reshape(R, C, 128, 4).permute(0, 2, 1, 3)
    return data.reshape(R * 128, C * 4)[:rows, :cols]


def test_nvfp4_layout_conversions_are_exact():
    torch.manual_seed(0)
    w = torch.randn(256, 512) * 0.05
    ref = nv.quantize_ref(w)
    codes, s8 = io.rows_order(ref)
    assert torch.equal(s8, nv.block_scales_ref(w, nv.global_scale(w)))
    d = io.to_reference(ref)
    assert torch.equal(_from_blocked(d["w_scale"], 256, 32), s8.float())
    for got in (io.from_reference(d["w_qdata"], d["w_scale"], d["w_per_tensor_scale"]),
                io.from_reference(d["w_qdata"], None, d["w_per_tensor_scale"], d["w_scale_row"]),
                io.from_modelopt(**io.to_modelopt(ref))):
        assert torch.equal(got.q, ref.q) and torch.equal(got.s, ref.s) and torch.equal(got.gs, ref.gs)
    vals = nv.e2m1_values(io._unpack(codes)) * s8.view(torch.float8_e4m3fn).float().repeat_interleave(16, 1)
    assert torch.equal(vals * ref.gs, nv.dequantize_ref(ref))


def test_tp_slices_equal_sharded_full_tensors(tmp_path):
    cfg = PRESETS["tiny-qwen2-d128"]
    w = random_weights(cfg, device="cpu", dtype=torch.float32, seed=3)
    save_safetensors(w, cfg, str(tmp_path))
    full = load_safetensors(str(tmp_path), cfg, dtype=torch.float32)
    for size in (2, 4):
        for rank in range(size):
            part = load_safetensors(str(tmp_path), cfg, dtype=torch.float32, tp_rank=rank, tp_size=size)
            for k, t in full.items():
                want = shard_tensor(cfg, k, t, rank, size)
                assert torch.equal(part[k], want), (k, rank, size)


@pytest.mark.parametrize("layout", ["reference", "modelopt"])
def test_nvfp4_checkpoint_roundtrip_generates_identically(tmp_path, layout):
    cfg = PRESETS["tiny-qwen2-d128"]
    w = random_weights(cfg, device="cpu", dtype=torch.float32, seed=4, std=0.05)
    q = nv.quantize_model_weights(w, cfg)
    io.save_nvfp4_checkpoint(q, cfg, str(tmp_path), layout=layout)
    loaded = load_safetensors(str(tmp_path), cfg, dtype=torch.float32)
    for k, t in q.items():
        if isinstance(t, nv.NVFP4Weight):
            g = loaded[k]
            assert isinstance(g, nv.NVFP4Weight), k
            assert torch.equal(g.q, t.q) and torch.equal(g.s, t.s) and torch.equal(g.gs, t.gs), k
    kw = dict(device="cpu", dtype=torch.float32, kv_cache_dtype="fp32", max_batch=2, max_model_len=128,
              kv_pages=32)
    prompts = [[1, 2, 3, 4, 5, 6], [9, 8, 7]]
    a = [r.output_ids for r in LLM(cfg, weights=q, **kw).generate(prompts, SamplingParams(max_tokens=6))]
    b = [r.output_ids for r in LLM(str(tmp_path), **kw).generate(prompts, SamplingParams(max_tokens=6))]
    assert a == b
    # a tensor-parallel rank's load is the shard of the full quantised model
    part = load_safetensors(str(tmp_path), cfg, dtype=torch.float32, tp_rank=1, tp_size=2)
    for k, t in q.items():
        if isinstance(t, nv.NVFP4Weight):
            s = io.shard_nvfp4(cfg, k, t, 1, 2)
            assert torch.equal(part[k].q, s.q) and torch.equal(part[k].s, s.s), k
