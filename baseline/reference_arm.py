"""Reference arm of bench.py: the unmodified reference (installed into baseline/_ref)
measured through its own public API on the same metric and config.

What runs, all of it reference code:
  bs1 + TTFT  core.turbo_engine.create_turbo_engine(model, tokenizer) -> warmup() ->
              generate_ids(), the engine core/inference_pipeline.py:927 creates.  On a
              compute-capability >= 10 GPU without torchao that engine cannot run: it
              moves lm_head to the host to quantise it to FP4 (core/turbo_engine.py:
              314-328), the quantiser needs torchao, and the caught ImportError leaves
              lm_head on the host.  The arm then measures the reference's path with
              VRM_DISABLE_TURBO: core.backends.HuggingFaceBackend.generate (HF generate
              with KV cache, core/backends.py:1868-1934), and says so in "notes".
  bs32        core.continuous_batcher.ContinuousBatcher(model, tokenizer, 32).submit()
              x 32 -> start() -> futures, when it can run on the installed transformers:
              its per-request cache split (_unbatch_kv_cache, core/continuous_batcher.py:
              869-891) reads DynamicCache.key_cache, which transformers 5 removed (caches
              keep per-layer objects in .layers), so every batched-prefill request fails
              there.  The arm then measures the reference's batched generation call,
              core.backends.HuggingFaceBackend.generate_batch (core/backends.py:2113-2171:
              left-padded prompts, one HF generate with KV cache), and says so in "notes".
The model's parameters are frozen (requires_grad False), as for any inference load: the
batcher's worker thread runs its forwards without torch.no_grad, and with trainable
parameters autograd keeps every activation of the batched prefill alive (about 150 GB
for 32 x 512 tokens of the 14B model), which is what ran the GPU out of memory.
The model is transformers' Qwen2ForCausalLM built from the Qwen2.5-14B configuration with
random N(0, 0.02) bf16 weights directly on the GPU: there are no checkpoints offline, and
the reference's own loader (core/backends.py:1185-1390) passes a device_map to
from_pretrained, which needs `accelerate` (not installed).  A 14B bf16 model fits one
B200, so the reference's single-GPU bypass (core/backends.py _try_single_gpu_placement)
places it on one GPU whatever the GPU count: under torchrun rank 0 measures, the other
ranks only wait.

Decode rates exclude prefill: each is the difference between two runs of different
lengths (1 + W + K and 1 + W new tokens), timed with CUDA events around the public call
(its decode loop synchronises with the host every token).
"""
from __future__ import annotations

import json
import os
import statistics
import sys
import time
import zlib

HERE = os.path.dirname(os.path.abspath(__file__))
REF = os.path.join(HERE, "_ref")

QWEN25_14B = dict(hidden_size=5120, intermediate_size=13824, num_hidden_layers=48, num_attention_heads=40,
                  num_key_value_heads=8, vocab_size=152064, max_position_embeddings=32768, rope_theta=1e6,
                  rms_norm_eps=1e-6, tie_word_embeddings=False, initializer_range=0.02)


class IdTokenizer:
    """Tokenizer stand-in (no tokenizer files offline): a prompt is space-separated
    token ids; other words hash to an id.  No EOS, so every request runs to its
    max_new_tokens, as the benchmark requires."""
    eos_token_id = None
    pad_token_id = 0
    pad_token = "0"
    padding_side = "right"

    def __init__(self, vocab: int):
        self.vocab = vocab

    def _ids(self, s):
        return [int(t) % self.vocab if t.isdigit() else zlib.crc32(t.encode()) % self.vocab for t in s.split()] or [0]

    def __call__(self, text, return_tensors="pt", padding=False, **kw):
        import torch
        texts = [text] if isinstance(text, str) else list(text)
        ids = [self._ids(s) for s in texts]
        n = max(len(x) for x in ids)
        inp = torch.zeros(len(ids), n, dtype=torch.long)
        mask = torch.zeros_like(inp)
        for i, x in enumerate(ids):
            sl = slice(n - len(x), n) if self.padding_side == "left" else slice(0, len(x))
            inp[i, sl] = torch.tensor(x)
            mask[i, sl] = 1
        from transformers import BatchEncoding
        return BatchEncoding({"input_ids": inp, "attention_mask": mask})

    def encode(self, text, **kw):
        return self._ids(text)

    def decode(self, ids, skip_special_tokens=True, **kw):
        return " ".join(str(int(t)) for t in ids)


def _build_model(dev):
    import torch
    from transformers import Qwen2Config, Qwen2ForCausalLM
    cfg = Qwen2Config(**QWEN25_14B)
    torch.manual_seed(1234)
    prev = torch.get_default_dtype()
    torch.set_default_dtype(torch.bfloat16)
    try:
        with torch.device(dev):
            model = Qwen2ForCausalLM(cfg)
    finally:
        torch.set_default_dtype(prev)
    # some parameters (lm_head) can still be created on the host: move everything
    model = model.to(device=dev, dtype=torch.bfloat16).eval()
    model.requires_grad_(False)
    return model


def _timed(fn):
    import torch
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    out = fn()
    b.record()
    torch.cuda.synchronize()
    return a.elapsed_time(b), out


def _turbo_usable(dev) -> str:
    """'' when the reference TurboEngine can run here, else why not."""
    import importlib.util
    import torch
    if torch.cuda.get_device_capability(dev)[0] >= 10 and importlib.util.find_spec("torchao") is None:
        return ("TurboEngine unusable: on cc>=10 it moves lm_head to the host for FP4 quantisation, which needs "
                "torchao (not installed); the caught ImportError leaves lm_head on the host "
                "(core/turbo_engine.py:314-328)")
    return ""


def _bs1_turbo(model, tok, text, ids, steps, warm, ttft_runs):
    from core.turbo_engine import create_turbo_engine
    eng = create_turbo_engine(model, tok, max_seq_len=2048)
    # warmup() with the benchmark prompt: the stock default "Hello" is a 1-token prefill,
    # which cuDNN SDPA (the only backend the engine leaves enabled for GQA models,
    # core/turbo_engine.py:72-93) rejects on this stack ("Invalid backend")
    eng.warmup(prompt=text, n_tokens=4, rounds=2)
    eng.generate_ids(ids, max_new_tokens=1 + warm)
    t_short, _ = _timed(lambda: eng.generate_ids(ids, max_new_tokens=1 + warm))
    t_long, out = _timed(lambda: eng.generate_ids(ids, max_new_tokens=1 + warm + steps))
    produced = out.shape[1] - ids.shape[1] - (1 + warm)
    ttfts = [_timed(lambda: eng.generate_ids(ids, max_new_tokens=1))[0] for _ in range(ttft_runs)]
    return (t_long - t_short) / max(1, produced), ttfts, "TurboEngine.generate_ids"


def _bs1_backend(model, tok, text, steps, warm, ttft_runs):
    from core.backends import HuggingFaceBackend
    be = HuggingFaceBackend("qwen2.5-14b-random-init")
    be.model, be.tokenizer = model, tok

    def gen(n):
        return be.generate(text, max_new_tokens=n, min_new_tokens=n, do_sample=False)
    gen(1 + warm)
    t_short, _ = _timed(lambda: gen(1 + warm))
    t_long, _ = _timed(lambda: gen(1 + warm + steps))
    ttfts = [_timed(lambda: gen(1))[0] for _ in range(ttft_runs)]
    return (t_long - t_short) / steps, ttfts, "HuggingFaceBackend.generate (VRM_DISABLE_TURBO path)"


def _bs1(model, tok, prompt_ids, steps, warm, ttft_runs, notes, dev):
    import torch
    text = " ".join(str(t) for t in prompt_ids)
    why = _turbo_usable(dev)
    if not why:
        try:
            ids = torch.tensor([prompt_ids], dtype=torch.long)
            ms, ttfts, api = _bs1_turbo(model, tok, text, ids, steps, warm, ttft_runs)
            return {"tok_s": round(1000.0 / ms, 2), "ms_per_step": round(ms, 3), "api": api}, \
                statistics.median(ttfts)
        except Exception as e:   # the pipeline falls back the same way (core/inference_pipeline.py:939)
            why = f"TurboEngine failed: {type(e).__name__}: {str(e)[:160]}"
            model.to(dev)
    notes.append(why)
    os.environ["VRM_DISABLE_TURBO"] = "1"
    ms, ttfts, api = _bs1_backend(model, tok, text, steps, warm, ttft_runs)
    return {"tok_s": round(1000.0 / ms, 2), "ms_per_step": round(ms, 3), "api": api}, statistics.median(ttfts)


def _batcher_usable() -> str:
    """'' when the stock ContinuousBatcher can split a batched cache here, else why not."""
    try:
        from transformers import DynamicCache
    except ImportError:
        return ""
    if not hasattr(DynamicCache(), "key_cache"):
        import transformers
        return (f"ContinuousBatcher unusable on transformers {transformers.__version__}: _unbatch_kv_cache reads "
                "DynamicCache.key_cache (core/continuous_batcher.py:869-891), which this version no longer has, "
                "so every batched-prefill request fails; bs32 measured with HuggingFaceBackend.generate_batch")
    return ""


def _bs32_generate_batch(model, tok, prompts, steps, warm, dev):
    """bs32 through the reference's batched generation call: one left-padded HF
    generate with KV cache over all prompts (core/backends.py:2113-2171)."""
    from core.backends import HuggingFaceBackend
    be = HuggingFaceBackend("qwen2.5-14b-random-init")
    be.model, be.tokenizer = model, tok
    be.block_devices = [int(str(dev).split(":")[-1])]

    def gen(n):
        return be.generate_batch(prompts, max_new_tokens=n, min_new_tokens=n, do_sample=False)
    gen(2)                                                    # warm-up
    t_short, _ = _timed(lambda: gen(1 + warm))
    t_long, outs = _timed(lambda: gen(1 + warm + steps))
    ms_step = (t_long - t_short) / steps
    n_tok = sum(len(o.split()) for o in outs)
    return {"tok_s": round(len(prompts) * 1000.0 / ms_step, 2), "ms_per_step": round(ms_step, 3),
            "api": "HuggingFaceBackend.generate_batch", "tokens_returned": n_tok}


def _bs32(model, tok, prompts, steps, warm, dev, notes):
    why = _batcher_usable()
    if why:
        notes.append(why)
        return _bs32_generate_batch(model, tok, prompts, steps, warm, dev)
    from core.continuous_batcher import ContinuousBatcher

    def run(n_new):
        b = ContinuousBatcher(model, tok, max_batch_size=len(prompts), device=dev, verbose=False)
        futs = [b.submit(p, max_new_tokens=n_new, temperature=1.0, top_k=1) for p in prompts]

        def go():
            b.start()
            return [f.result(timeout=900) for f in futs]
        try:
            return _timed(go)
        finally:
            b.stop()

    run(2)                                                    # warm-up
    t_short, _ = run(1 + warm)
    t_long, outs = run(1 + warm + steps)
    ms_step = (t_long - t_short) / steps
    return {"tok_s": round(len(prompts) * 1000.0 / ms_step, 2), "ms_per_step": round(ms_step, 3),
            "api": "ContinuousBatcher.submit"}


def run(args, metric):
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if not os.path.isdir(os.path.join(REF, "core")):
        if rank == 0:
            print(json.dumps({"impl": "reference", "unavailable": "baseline/_ref not installed"}), flush=True)
        return
    if rank != 0:
        return                       # single-GPU placement: only rank 0's GPU is used
    import torch
    if not torch.cuda.is_available():
        print(json.dumps({"impl": "reference", "unavailable": "no CUDA device"}), flush=True)
        return
    sys.path.insert(0, REF)
    os.environ.setdefault("VRM_LOG_LEVEL", "WARNING")
    dev = f"cuda:{int(os.environ.get('LOCAL_RANK', '0'))}"
    torch.cuda.set_device(dev)
    import random
    rng = random.Random(42)
    P, B = args.prompt_len, args.batch
    steps, warm = args.steps, max(3, args.warmup)
    vocab = QWEN25_14B["vocab_size"]
    tok = IdTokenizer(vocab)
    notes = []
    t0 = time.time()
    model = _build_model(dev)
    prompt_ids = [rng.randrange(vocab) for _ in range(P)]
    from bench import ClockSampler
    clocks = ClockSampler(torch.cuda.current_device())
    clocks.start()
    bs1, ttft = _bs1(model, tok, prompt_ids, steps, warm, args.ttft_runs, notes, dev)
    try:
        prompts = [" ".join(str(rng.randrange(vocab)) for _ in range(P)) for _ in range(B)]
        bs32 = _bs32(model, tok, prompts, steps, warm, dev, notes)
        value = bs32["tok_s"]
    except Exception as e:
        bs32, value = None, None
        notes.append(f"ContinuousBatcher failed: {type(e).__name__}: {str(e)[:200]}")
    clk = clocks.stop()
    res = {
        "metric": metric,
        "value": value,
        "unit": "tok/s",
        "n_gpus": world,
        "steps": steps,
        "warmup": warm,
        "ms_per_step": bs32["ms_per_step"] if bs32 else None,
        "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": "bf16",
        "data": "synthetic: uniform random token ids, random-init N(0,0.02) bf16 weights (HF from_config)",
        "config": {"model": "Qwen2.5-14B architecture", "global_batch": B, "seq_len": P,
                   "parallelism": "single GPU (reference single-GPU bypass)",
                   "l2": "inputs larger than L2 (all weights streamed each step)"},
        "bs1": bs1,
        "ttft_p50_ms": round(ttft, 3),
        "ttft_prompt_tokens": P,
        # end to end: prompts go in as host strings and results come back as host
        # strings through the public call; per decode step the host copies in nothing
        # new and HF generate's stopping check reads one flag per sequence back
        "e2e": {"value": value, "unit": "tok/s", "api": bs32["api"] if bs32 else None,
                "h2d_bytes_per_step": round(B * P * 8 / (1 + warm + steps)) if bs32 else None,
                "d2h_bytes_per_step": B if bs32 else None,
                "note": "prompt ids (int64) copied once per call, amortised over its decode steps"},
        "clocks": clk,
        "setup_s": round(time.time() - t0, 1),
        "notes": notes,
        "impl": "reference",
    }
    if value is None:
        res["value_unavailable"] = "bs32: " + (notes[-1] if notes else "ContinuousBatcher failed") + \
            "; bs1 and TTFT are measured"
    print(json.dumps(res), flush=True)
