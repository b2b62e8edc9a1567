"""quickstart recommendations, the transformers drop-in patch, and LoRA hot-swap
(merge, switch, disable restores the base weights) on CPU."""
import torch

from vramancer_b200 import dropin, quickstart
from vramancer_b200.engine.engine import SamplingParams
from vramancer_b200.llm import LLM
from vramancer_b200.models.config import PRESETS
from vramancer_b200.models.weights import random_weights
from vramancer_b200.serving.lora import LoRAManager


def test_quickstart_recommend():
    assert quickstart.estimate_gb(14.8, "bf16") == 14.8 * 2.0 * 1.2 + 1.5
    r = quickstart.recommend("chat", 180.0)           # one B200
    assert r["model"] == "Qwen/Qwen2.5-72B-Instruct" and r["quantization"] == "bf16"   # 176 GB
    r = quickstart.recommend("chat", 100.0)
    assert r["model"] == "Qwen/Qwen2.5-72B-Instruct" and r["quantization"] == "fp8"    # 88.7 GB
    r = quickstart.recommend("code-assistant", 24.0)
    assert r["model"].endswith("Coder-14B-Instruct") and r["quantization"] == "fp8"
    r = quickstart.recommend("code-assistant", 24.0, blackwell=False)
    assert r["quantization"] in ("bf16", "fp8")
    assert quickstart.recommend("chat", 1.0) is None
    assert quickstart.recommend("unknown-use", 180.0)["use_case"] == "unknown-use"


def test_dropin_patch_serves_known_models():
    from transformers import AutoModelForCausalLM
    orig = AutoModelForCausalLM.from_pretrained
    dropin.patch()
    try:
        assert dropin.is_patched()
        m = AutoModelForCausalLM.from_pretrained("tiny-qwen2", max_model_len=64)
        assert isinstance(m, dropin.VRAMancerCausalLM)
        out = m.generate(torch.tensor([[3, 4, 5, 6]]), max_new_tokens=5, prompt_lookup_num_tokens=None)
        assert out.shape == (1, 9) and out[0, :4].tolist() == [3, 4, 5, 6]
        logits = m(torch.tensor([[3, 4, 5]])).logits
        assert logits.shape[-1] == PRESETS["tiny-qwen2"].vocab_size
        m.pipeline.shutdown()
    finally:
        dropin.unpatch()
    assert not dropin.is_patched()
    assert AutoModelForCausalLM.from_pretrained.__func__ is getattr(orig, "__func__", orig)


def test_lora_merge_switch_disable():
    cfg = PRESETS["tiny-qwen2"]
    w = random_weights(cfg, device="cpu", dtype=torch.float32, seed=1, std=0.2)
    llm = LLM(cfg, device="cpu", dtype=torch.float32, kv_cache_dtype="fp32", weights=w, max_batch=2,
              max_model_len=64, kv_pages=16)
    base_qkv = w["layers.0.qkv_w"].clone()
    base_gu = w["layers.1.gate_up_w"].clone()
    prompt = [[7, 8, 9, 10, 11]]
    base_out = llm.generate(prompt, SamplingParams(max_tokens=6))[0].output_ids
    H, r = cfg.hidden_size, 4
    g = torch.Generator().manual_seed(0)
    A = torch.randn(r, H, generator=g)
    Bq = torch.randn(cfg.head_dim * cfg.num_heads, r, generator=g)
    Bg = torch.randn(cfg.intermediate_size, r, generator=g)
    lora = LoRAManager(llm)
    assert lora.load_adapter("a", {(0, "q_proj"): (A, Bq), (1, "gate_proj"): (A, Bg)}, alpha=8.0) == 2
    assert lora.load_adapter("b", {(0, "q_proj"): (A, -Bq)}, alpha=8.0) == 1
    lora.set_adapter("a")
    q_rows = cfg.head_dim * cfg.num_heads
    want_q = base_qkv[:q_rows] + (Bq @ A) * (8.0 / r)
    assert torch.allclose(w["layers.0.qkv_w"][:q_rows], want_q, atol=1e-4)
    assert torch.allclose(w["layers.1.gate_up_w"][0::2], base_gu[0::2] + (Bg @ A) * 2.0, atol=1e-4)
    assert torch.equal(w["layers.1.gate_up_w"][1::2], base_gu[1::2])      # up rows untouched
    lora.set_adapter("b")                                                  # switch: a out, b in
    assert torch.allclose(w["layers.0.qkv_w"][:q_rows], base_qkv[:q_rows] - (Bq @ A) * 2.0, atol=1e-4)
    lora.disable()
    assert torch.allclose(w["layers.0.qkv_w"], base_qkv, atol=1e-4)
    assert torch.allclose(w["layers.1.gate_up_w"], base_gu, atol=1e-4)
    assert llm.generate(prompt, SamplingParams(max_tokens=6))[0].output_ids == base_out
    lora.delete_adapter("a")
    assert lora.list_adapters() == {"adapters": ["b"], "active": None}


def test_quickstart_launches_run_and_serve():
    from types import SimpleNamespace
    gpus = [SimpleNamespace(free_gb=178.0, capability=(10, 0))]
    calls = []

    def launcher(kind, ns):
        calls.append((kind, ns))
        return 0
    rec = quickstart.run_quickstart("chat", gpus=gpus, launcher=launcher)
    assert calls == [] and rec["command"].startswith("vramancer run ")
    rec = quickstart.run_quickstart("chat", run=True, prompt="hello", gpus=gpus, launcher=launcher)
    kind, ns = calls[-1]
    assert kind == "run" and rec["launched"] == "run" and ns.model == rec["model"] and ns.prompt == "hello"
    assert (ns.quantization or "bf16") == rec["quantization"]
    rec = quickstart.run_quickstart("code-assistant", serve=True, port=6001, gpus=gpus, launcher=launcher)
    kind, ns = calls[-1]
    assert kind == "serve" and ns.port == 6001 and rec["command"].startswith("vramancer serve ")


def test_quickstart_run_goes_through_the_run_command(monkeypatch):
    """Without a launcher the recommendation runs through cli._cmd_run (as `vramancer run`)."""
    from types import SimpleNamespace

    from vramancer_b200 import cli
    seen = {}
    monkeypatch.setattr(cli, "_cmd_run", lambda a: seen.setdefault("run", a.model) and 0)
    gpus = [SimpleNamespace(free_gb=30.0, capability=(10, 0))]
    rec = quickstart.run_quickstart("chat", run=True, gpus=gpus)
    assert seen["run"] == rec["model"] and rec["exit_code"] == 0
