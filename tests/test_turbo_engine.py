"""The reference's `TurboEngine` API (core/turbo_engine.py) over this framework's engine:
a loaded Hugging Face model is converted and served; greedy outputs must equal
transformers' `generate` on the same model (CPU, fp32), through the single-device,
layer-pipelined and speculative engines."""
import pytest
import torch

T = pytest.importorskip("transformers")

import vramancer_b200 as vrm  # noqa: E402

V = 256


class CharTokenizer:
    """Test tokenizer with the HF calling conventions: one character per id."""
    eos_token_id = None

    def __call__(self, text, return_tensors=None):
        ids = [ord(c) % V for c in text]
        return {"input_ids": torch.tensor([ids]) if return_tensors == "pt" else ids}

    def decode(self, ids, skip_special_tokens=False):
        return "".join(chr(0x100 + int(i)) for i in ids)


class ByteTokenizer(CharTokenizer):
    """UTF-8 bytes: a character may span several ids."""

    def __call__(self, text, return_tensors=None):
        ids = list(text.encode("utf-8"))
        return {"input_ids": torch.tensor([ids]) if return_tensors == "pt" else ids}

    def decode(self, ids, skip_special_tokens=False):
        return bytes(int(i) for i in ids).decode("utf-8", errors="replace")


@pytest.fixture(scope="module")
def hf_model():
    torch.manual_seed(0)
    m = T.Qwen2ForCausalLM(T.Qwen2Config(vocab_size=V, hidden_size=128, num_hidden_layers=3, num_attention_heads=4,
                                         num_key_value_heads=2, intermediate_size=256, max_position_embeddings=256,
                                         rope_theta=1e4, tie_word_embeddings=False))
    with torch.no_grad():
        for n, p in m.named_parameters():
            p.copy_(torch.randn(p.shape) * (0.15 if p.dim() > 1 else 0.05) + (1.0 if "norm" in n else 0.0))
    return m.eval()


def _hf_greedy(m, ids, n):
    x = torch.tensor([ids])
    with torch.no_grad():
        return m.generate(x, attention_mask=torch.ones_like(x), max_new_tokens=n, do_sample=False,
                          pad_token_id=0)[0].tolist()


def test_turbo_engine_generate_ids_matches_transformers(hf_model):
    eng = vrm.TurboEngine(hf_model, CharTokenizer(), device="cpu", max_seq_len=128)
    assert eng.n_layers == 3 and eng.vocab_size == V and eng.dtype == torch.float32
    ids = list(range(5, 25))
    out = eng.generate_ids(torch.tensor([ids]), max_new_tokens=10)
    assert out.shape == (1, 30)
    assert out[0].tolist() == _hf_greedy(hf_model, ids, 10)


def test_turbo_engine_text_and_stream(hf_model):
    tok = CharTokenizer()
    eng = vrm.TurboEngine(hf_model, tok, device="cpu", max_seq_len=128)
    eng.warmup(prompt="warm", n_tokens=3, rounds=1)
    prompt = "hello world"
    ids = tok(prompt)["input_ids"]
    want = _hf_greedy(hf_model, ids, 12)[len(ids):]
    assert eng.generate(prompt, max_new_tokens=12, temperature=0.3) == tok.decode(want)   # do_sample=False: greedy
    pieces = list(eng.generate_stream(prompt, max_new_tokens=12))
    assert "".join(pieces) == tok.decode(want)
    # sampling runs and stays inside the vocabulary
    s = eng.generate_ids(torch.tensor([ids]), max_new_tokens=6, do_sample=True, temperature=0.8, top_k=20, top_p=0.9)
    assert s.shape == (1, len(ids) + 6) and int(s.max()) < V
    with pytest.raises(ValueError):
        eng.generate("x" * 200)


def test_multi_device_turbo_engine_matches_transformers(hf_model):
    eng = vrm.MultiGPUTurboEngine(hf_model, CharTokenizer(), layer_devices={0: "cpu", 1: "cpu", 2: "cpu"},
                                  max_seq_len=128)
    ids = list(range(40, 58))
    assert eng.generate_ids(ids, max_new_tokens=8)[0].tolist() == _hf_greedy(hf_model, ids, 8)


def test_layer_devices_become_contiguous_blocks():
    from vramancer_b200.engine.turbo import _blocks_from_layer_devices
    b = _blocks_from_layer_devices({0: "cuda:0", 1: "cuda:0", 2: "cuda:1", 3: "cuda:1", 4: "cuda:0"}, 5)
    assert [(x.start, x.end, x.device) for x in b] == [(0, 2, "cuda:0"), (2, 4, "cuda:1"), (4, 5, "cuda:0")]
    with pytest.raises(ValueError):
        _blocks_from_layer_devices({0: "cuda:0"}, 2)


def test_speculative_turbo_engine_greedy_is_exact(hf_model):
    tok = CharTokenizer()
    eng = vrm.SpeculativeTurboEngine(hf_model, hf_model, tok, device="cpu", gamma=4, max_seq_len=128)
    prompt = "speculate"
    ids = tok(prompt)["input_ids"]
    want = _hf_greedy(hf_model, ids, 16)[len(ids):]
    assert eng.generate(prompt, max_new_tokens=16) == tok.decode(want)
    st = eng.stats()
    assert st["drafted"] > 0 and st["acceptance_rate"] == 1.0          # the draft is the target
    assert st["effective_tokens_per_round"] > 2.0
    assert set(st) == {"drafted", "accepted", "rounds", "acceptance_rate", "effective_tokens_per_round"}


def test_create_turbo_engine_picks_single_device(hf_model):
    eng = vrm.create_turbo_engine(hf_model, CharTokenizer(), max_seq_len=64)
    assert isinstance(eng, vrm.TurboEngine) and eng.device.type == "cpu"


def test_stream_holds_back_partial_characters(hf_model):
    """A multi-byte character split over tokens comes out whole, and the pieces join
    to the full text."""
    tok = ByteTokenizer()
    eng = vrm.TurboEngine(hf_model, tok, device="cpu", max_seq_len=128)
    core = eng.llm.engine
    text = "é€"                                     # 2 + 3 UTF-8 bytes
    script = list(text.encode("utf-8"))

    def step():                                     # emit the scripted bytes, one per step
        for r in list(core.running) + list(core.waiting):
            core.waiting.clear()
            if r not in core.running:
                core.running.append(r)
            core._emit(r, script[len(r.output_ids)])
        return []
    core.step = step
    pieces = list(eng.generate_stream("a", max_new_tokens=len(script)))
    assert "".join(pieces) == text
    assert all("\ufffd" not in p for p in pieces) and pieces == ["é", "€"]


@pytest.mark.gpu
def test_turbo_engine_on_gpu_follows_transformers(cuda_errors_clean):
    """The converted model on the GPU kernels (bf16, CUDA-graph decode) against
    transformers in fp32 on the host: last-position logits agree in direction."""
    torch.manual_seed(3)
    m = T.Qwen2ForCausalLM(T.Qwen2Config(vocab_size=512, hidden_size=256, num_hidden_layers=2, num_attention_heads=4,
                                         num_key_value_heads=2, intermediate_size=512, max_position_embeddings=512,
                                         rope_theta=1e4, tie_word_embeddings=False)).eval()
    with torch.no_grad():
        for n, p in m.named_parameters():
            p.copy_(torch.randn(p.shape) * (0.1 if p.dim() > 1 else 0.05) + (1.0 if "norm" in n else 0.0))
    eng = vrm.TurboEngine(m, None, device="cuda:0", max_seq_len=256)
    eng.warmup(prompt=[1, 2, 3], n_tokens=4, rounds=1)
    ids = list(range(7, 47))
    from vramancer_b200.engine.runner import PrefillItem
    kv = eng.llm.engine.kv
    kv.allocate("gpu-parity", len(ids))
    it = PrefillItem(ids, 0, kv.slots_for("gpu-parity", 0, len(ids)), kv.block_table("gpu-parity"), len(ids), True)
    got = eng.llm.engine.runner.prefill_logits([it])[-1].float().cpu()
    kv.free("gpu-parity")
    with torch.no_grad():
        ref = m(torch.tensor([ids])).logits[0, -1].float()
    cos = torch.nn.functional.cosine_similarity(got, ref, dim=0).item()
    assert cos > 0.99, cos
    out = eng.generate_ids(ids, max_new_tokens=8)
    assert out.shape == (1, len(ids) + 8) and out.device.type == "cuda"
