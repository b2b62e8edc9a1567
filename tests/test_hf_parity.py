"""Model families against Hugging Face transformers (the implementation the reference
serves through `HuggingFaceBackend`): tiny random models of every supported
architecture are saved as HF checkpoints, loaded here (from the safetensors directory
and from the in-memory state dict), and their last-position logits and greedy tokens
compared with transformers' own forward and `generate` on the CPU in fp32.  RoPE
scaling (linear, Llama 3, YaRN) is checked against transformers' frequency rules."""
import math

import pytest
import torch

T = pytest.importorskip("transformers")

from vramancer_b200 import LLM, SamplingParams, ops  # noqa: E402
from vramancer_b200.engine.runner import PrefillItem  # noqa: E402
from vramancer_b200.models.config import ModelConfig  # noqa: E402
from vramancer_b200.models.weights import weights_from_state_dict  # noqa: E402

V = 512


def _hf_model(kind, **rope):
    common = dict(vocab_size=V, hidden_size=128, num_hidden_layers=2, num_attention_heads=4,
                  max_position_embeddings=256)
    if kind == "qwen2":
        m = T.Qwen2ForCausalLM(T.Qwen2Config(num_key_value_heads=2, intermediate_size=256, rope_theta=1e6,
                                             tie_word_embeddings=False, **common))
    elif kind == "llama":
        m = T.LlamaForCausalLM(T.LlamaConfig(num_key_value_heads=2, intermediate_size=256, tie_word_embeddings=True,
                                             **rope, **common))
    elif kind == "mistral":
        m = T.MistralForCausalLM(T.MistralConfig(num_key_value_heads=1, intermediate_size=256, sliding_window=None,
                                                 **common))
    elif kind == "gpt2":
        m = T.GPT2LMHeadModel(T.GPT2Config(vocab_size=V, n_embd=128, n_layer=2, n_head=4, n_positions=256))
    elif kind == "qwen3":
        m = T.Qwen3ForCausalLM(T.Qwen3Config(num_key_value_heads=2, intermediate_size=256, head_dim=64,
                                             tie_word_embeddings=False, **common))
    elif kind == "qwen3_moe":
        m = T.Qwen3MoeForCausalLM(T.Qwen3MoeConfig(num_key_value_heads=2, intermediate_size=256, head_dim=64,
                                                   moe_intermediate_size=64, num_experts=8, num_experts_per_tok=2,
                                                   norm_topk_prob=True, decoder_sparse_step=1, mlp_only_layers=[],
                                                   **common))
    elif kind == "mixtral":
        m = T.MixtralForCausalLM(T.MixtralConfig(num_key_value_heads=2, intermediate_size=64, num_local_experts=8,
                                                 num_experts_per_tok=2, **common))
    elif kind == "qwen2_moe":
        m = T.Qwen2MoeForCausalLM(T.Qwen2MoeConfig(num_key_value_heads=2, intermediate_size=256,
                                                   moe_intermediate_size=64, shared_expert_intermediate_size=128,
                                                   num_experts=8, num_experts_per_tok=2, decoder_sparse_step=1,
                                                   mlp_only_layers=[], **common))
    else:
        raise ValueError(kind)
    g = torch.Generator().manual_seed(hash(kind) % 1000)
    with torch.no_grad():                  # larger weights than HF's init: logits far from uniform
        for name, p in m.named_parameters():
            if p.dim() > 1:
                p.copy_(torch.randn(p.shape, generator=g) * 0.15)
            elif "norm" in name or name.endswith("ln_1.weight") or name.endswith("ln_2.weight") \
                    or name.endswith("ln_f.weight"):
                p.copy_(1.0 + torch.randn(p.shape, generator=g) * 0.1)
            else:
                p.copy_(torch.randn(p.shape, generator=g) * 0.05)
    return m.eval()


def _llm(src, cfg=None, weights=None):
    return LLM(cfg if cfg is not None else src, device="cpu", dtype=torch.float32, kv_cache_dtype="fp32",
               kv_pages=64, max_model_len=256, use_cuda_graph=False, fold_norms=False, weights=weights)


def _last_logits(llm, ids):
    eng = llm.engine
    kv = eng.kv
    kv.allocate("parity", len(ids))
    try:
        it = PrefillItem(ids, 0, kv.slots_for("parity", 0, len(ids)), kv.block_table("parity"), len(ids), True)
        return eng.runner.prefill_logits([it])[-1].float()
    finally:
        kv.free("parity")


def _compare(m, llm, n_prompt=20, n_new=8, seed=0):
    ids = torch.randint(0, V, (1, n_prompt), generator=torch.Generator().manual_seed(seed))
    with torch.no_grad():
        ref = m(ids).logits[0, -1].float()
        want = m.generate(ids, attention_mask=torch.ones_like(ids), max_new_tokens=n_new, do_sample=False,
                          pad_token_id=0)[0, n_prompt:].tolist()
    got = _last_logits(llm, ids[0].tolist())
    scale = ref.abs().max().item()
    assert (got - ref).abs().max().item() <= 2e-4 * max(scale, 1.0), ((got - ref).abs().max().item(), scale)
    out = llm.generate([ids[0].tolist()], SamplingParams(max_tokens=n_new, ignore_eos=True))[0].output_ids
    assert out == want, (out, want)


@pytest.mark.parametrize("kind", ["qwen2", "llama", "mistral", "gpt2", "qwen2_moe", "qwen3", "qwen3_moe", "mixtral"])
def test_checkpoint_dir_matches_transformers(kind, tmp_path):
    torch.manual_seed(0)
    m = _hf_model(kind)
    m.save_pretrained(tmp_path)
    llm = _llm(str(tmp_path))
    assert llm.cfg.arch == ("qwen2_moe" if kind.endswith("moe") or kind == "mixtral" else kind)
    assert llm.cfg.qk_norm == kind.startswith("qwen3")
    _compare(m, llm)


@pytest.mark.parametrize("kind", ["qwen2", "gpt2", "qwen2_moe", "qwen3_moe", "mixtral"])
def test_state_dict_matches_transformers(kind):
    m = _hf_model(kind)
    cfg = ModelConfig.from_hf_config(m.config.to_dict())
    w = weights_from_state_dict(cfg, m.state_dict(), dtype=torch.float32)
    _compare(m, _llm(None, cfg, w), seed=1)


ROPE_CASES = {
    "linear": {"rope_type": "linear", "factor": 4.0},
    "llama3": {"rope_type": "llama3", "factor": 8.0, "low_freq_factor": 1.0, "high_freq_factor": 4.0,
               "original_max_position_embeddings": 16},
    "yarn": {"rope_type": "yarn", "factor": 4.0, "original_max_position_embeddings": 16},
    "yarn_mscale": {"rope_type": "yarn", "factor": 8.0, "original_max_position_embeddings": 32, "mscale": 0.707,
                    "mscale_all_dim": 1.0, "beta_fast": 16.0, "beta_slow": 2.0},
}


@pytest.mark.parametrize("case", sorted(ROPE_CASES))
def test_rope_frequencies_match_transformers(case):
    from transformers.modeling_rope_utils import ROPE_INIT_FUNCTIONS
    params = dict(ROPE_CASES[case], rope_theta=50000.0)
    hc = T.LlamaConfig(hidden_size=256, num_attention_heads=2, max_position_embeddings=128, rope_parameters=params)
    inv_ref, att_ref = ROPE_INIT_FUNCTIONS[params["rope_type"]](hc, "cpu")
    cfg = ModelConfig.from_hf_config(hc.to_dict())
    assert cfg.rope_scaling is not None and cfg.rope_theta == 50000.0
    inv, att = ops.rope_inv_freq(cfg.rot_dim, cfg.rope_theta, cfg.rope_scaling, cfg.max_position)
    torch.testing.assert_close(inv.float(), inv_ref.float(), rtol=1e-5, atol=0)
    assert math.isclose(att, float(att_ref), rel_tol=1e-6)


@pytest.mark.parametrize("case", ["llama3", "yarn"])
def test_scaled_rope_model_matches_transformers(case, tmp_path):
    params = dict(ROPE_CASES[case], rope_theta=10000.0)
    m = _hf_model("llama", rope_parameters=params)
    m.save_pretrained(tmp_path)
    llm = _llm(str(tmp_path))
    assert dict(llm.cfg.rope_scaling)["rope_type"] == case
    _compare(m, llm, n_prompt=40, n_new=6, seed=2)        # positions past the original context


def test_rope_scaling_round_trips_through_hf_config():
    cfg = ModelConfig.from_hf_config({"model_type": "llama", "hidden_size": 64, "num_attention_heads": 4,
                                      "num_hidden_layers": 1, "vocab_size": 10, "rope_theta": 5e5,
                                      "rope_scaling": {"type": "linear", "factor": 2.0}})
    assert cfg.rope_theta == 5e5 and dict(cfg.rope_scaling) == {"rope_type": "linear", "factor": 2.0}
    again = ModelConfig.from_hf_config(cfg.to_hf_config())
    assert again.rope_scaling == cfg.rope_scaling
    with pytest.raises(ValueError):
        ops.rope_inv_freq(64, 1e4, {"rope_type": "longrope"})


def test_unsupported_architectures_are_refused():
    """Model types, activations or layouts the native engine does not implement raise,
    so the backend factory serves them through another backend instead of running a
    wrong model."""
    from vramancer_b200.backends import native_supports
    from vramancer_b200.models.config import UnsupportedArchitecture
    base = {"hidden_size": 64, "num_attention_heads": 4, "num_hidden_layers": 1, "vocab_size": 10}
    for extra in ({"model_type": "gemma"}, {"model_type": "phi3"}, {"model_type": "llama", "hidden_act": "gelu"},
                  {"model_type": "llama", "mlp_bias": True},
                  {"model_type": "qwen2_moe", "num_experts": 4, "mlp_only_layers": [0]}):
        with pytest.raises(UnsupportedArchitecture):
            ModelConfig.from_hf_config(dict(base, **extra))
    assert ModelConfig.from_hf_config(dict(base, model_type="qwen3")).qk_norm
    # sliding-window attention: the context is capped at the window
    mc = ModelConfig.from_hf_config(dict(base, model_type="mistral", sliding_window=4096,
                                         max_position_embeddings=32768))
    assert mc.max_position == 4096


def test_native_supports_checks_the_checkpoint(tmp_path):
    import json

    from vramancer_b200.backends import native_supports
    d = tmp_path / "m"
    d.mkdir()
    (d / "config.json").write_text(json.dumps({"model_type": "gemma2", "hidden_size": 64, "num_attention_heads": 4,
                                               "num_hidden_layers": 1, "vocab_size": 10}))
    assert not native_supports(str(d))
    (d / "config.json").write_text(json.dumps({"model_type": "qwen3", "hidden_size": 64, "num_attention_heads": 4,
                                               "num_hidden_layers": 1, "vocab_size": 10}))
    assert native_supports(str(d))


@pytest.mark.gpu
@pytest.mark.parametrize("D", [64, 128])
def test_qk_rmsnorm_kernel_matches_fp32(D, cuda_errors_clean):
    torch.manual_seed(D)
    Tn, Hq, KH = 37, 8, 2
    qkv = (torch.randn(Tn, (Hq + 2 * KH) * D, device="cuda") * 3).bfloat16()
    wq = (1 + 0.2 * torch.randn(D, device="cuda")).bfloat16()
    wk = (1 + 0.2 * torch.randn(D, device="cuda")).bfloat16()
    ref = qkv.float().view(Tn, Hq + 2 * KH, D).clone()
    for sl, w in ((slice(0, Hq), wq), (slice(Hq, Hq + KH), wk)):
        h = ref[:, sl]
        ref[:, sl] = h * torch.rsqrt(h.pow(2).mean(-1, keepdim=True) + 1e-6) * w.float()
    out = qkv.clone()
    ops.qk_rmsnorm(out, wq, wk, Hq, KH, D, 1e-6)
    torch.cuda.synchronize()
    got = out.float().view(Tn, Hq + 2 * KH, D)
    torch.testing.assert_close(got, ref, rtol=1e-2, atol=1e-2)
    assert torch.equal(out.view(Tn, Hq + 2 * KH, D)[:, Hq + KH:], qkv.view(Tn, Hq + 2 * KH, D)[:, Hq + KH:])


@pytest.mark.gpu
def test_qwen3_model_on_gpu_follows_transformers(tmp_path, cuda_errors_clean):
    """A Qwen3 checkpoint on the GPU kernels (bf16) against transformers in fp32."""
    m = T.Qwen3ForCausalLM(T.Qwen3Config(vocab_size=V, hidden_size=256, num_hidden_layers=2, num_attention_heads=4,
                                         num_key_value_heads=2, head_dim=64, intermediate_size=512,
                                         max_position_embeddings=512, tie_word_embeddings=False))
    g = torch.Generator().manual_seed(5)
    with torch.no_grad():
        for n, p in m.named_parameters():
            p.copy_(torch.randn(p.shape, generator=g) * (0.1 if p.dim() > 1 else 0.05) + (1.0 if "norm" in n else 0.0))
    m.eval().save_pretrained(tmp_path)
    llm = LLM(str(tmp_path), device="cuda", max_model_len=256, kv_pages=64, max_batch=4)
    ids = list(range(3, 40))
    got = _last_logits(llm, ids).cpu()
    with torch.no_grad():
        ref = m(torch.tensor([ids])).logits[0, -1].float()
    assert torch.nn.functional.cosine_similarity(got, ref, dim=0).item() > 0.99


def test_family_presets_have_published_sizes():
    from vramancer_b200.models.config import get_config
    for name, billions in (("qwen3-8b", 8.19), ("qwen3-30b-a3b", 30.5), ("llama-3.1-8b", 8.03),
                           ("mixtral-8x7b", 46.7), ("Qwen/Qwen3-30B-A3B", 30.5)):
        assert abs(get_config(name).num_params() / 1e9 - billions) < 0.1, name
    assert get_config("qwen3-30b-a3b").qk_norm and dict(get_config("llama-3.1-8b").rope_scaling)["factor"] == 8.0


def test_hub_reports_native_support(tmp_path, capsys):
    import json as _json

    from vramancer_b200.cli import main
    for mt, native in (("qwen3", True), ("gemma2", False)):
        d = tmp_path / mt
        d.mkdir()
        (d / "config.json").write_text(_json.dumps({"model_type": mt, "hidden_size": 64, "num_attention_heads": 4,
                                                    "num_hidden_layers": 1, "vocab_size": 10}))
        assert main(["hub", str(d)]) == 0
        out = _json.loads(capsys.readouterr().out)
        assert out["native_engine"] is native
