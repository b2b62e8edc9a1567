"""HF safetensors round trip of the internal weight layout (fused qkv, interleaved
gate/up), including weights whose RMSNorm weight was folded into their columns."""
import torch

from vramancer_b200.models.config import PRESETS
from vramancer_b200.models.weights import load_safetensors, random_weights, save_safetensors


def test_round_trip_and_folded_weights(tmp_path):
    cfg = PRESETS["tiny-qwen2"]
    w = random_weights(cfg, device="cpu", dtype=torch.float32, seed=2)
    for i in range(cfg.num_layers):
        w[f"layers.{i}.in_norm_w"] = torch.rand(cfg.hidden_size) + 0.5
        w[f"layers.{i}.post_norm_w"] = torch.rand(cfg.hidden_size) + 0.5
    orig = {k: v.clone() for k, v in w.items()}
    save_safetensors(w, cfg, str(tmp_path / "a"))
    back = load_safetensors(str(tmp_path / "a"), cfg, device="cpu", dtype=torch.float32)
    for k, v in orig.items():
        assert torch.equal(back[k], v), k
    # fold as LLM(fold_norms=True) does (W' = W diag(norm_w), marked), then save
    for i in range(cfg.num_layers):
        for wk, nk in (("qkv_w", "in_norm_w"), ("gate_up_w", "post_norm_w")):
            W, nw = w[f"layers.{i}.{wk}"], w[f"layers.{i}.{nk}"]
            W.mul_(nw.view(1, -1))
            W._vrm_norm_w = nw.clone()
    save_safetensors(w, cfg, str(tmp_path / "b"))
    back = load_safetensors(str(tmp_path / "b"), cfg, device="cpu", dtype=torch.float32)
    for k, v in orig.items():
        assert torch.allclose(back[k], v, rtol=1e-6, atol=1e-7), k
