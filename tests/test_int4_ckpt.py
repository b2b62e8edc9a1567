"""GPTQ / AWQ checkpoints: code unpacking against packers written from the format
description, the dequantisation rule against element-wise loops, and whole checkpoints
(a tiny Qwen2 quantised in both layouts, act-order GPTQ included) loading to the same
model as their dense dequantised weights, checked against transformers."""
import json

import pytest
import torch

from vramancer_b200.quant import int4_ckpt

AWQ_ORDER = [0, 2, 4, 6, 1, 3, 5, 7]


def pack_rows_ref(codes, bits):
    """codes [K, N] -> int32 [K / per, N]: code j of word (r, n) is row r * per + j."""
    per = 32 // bits
    K, N = codes.shape
    out = torch.zeros(K // per, N, dtype=torch.int64)
    for r in range(K // per):
        for j in range(per):
            out[r] |= codes[r * per + j].to(torch.int64) << (bits * j)
    return (out - ((out >> 31) << 32)).to(torch.int32)        # wrap to signed 32-bit


def pack_cols_ref(codes, bits, order=None):
    """codes [R, N] -> int32 [R, N / per]: code j of word (r, c) is column c * per + order[j]."""
    per = 32 // bits
    order = order or list(range(per))
    R, N = codes.shape
    out = torch.zeros(R, N // per, dtype=torch.int64)
    for c in range(N // per):
        for j in range(per):
            out[:, c] |= codes[:, c * per + order[j]].to(torch.int64) << (bits * j)
    return (out - ((out >> 31) << 32)).to(torch.int32)


@pytest.mark.parametrize("bits", [2, 4, 8])
def test_gptq_unpack_round_trip(bits):
    g = torch.Generator().manual_seed(bits)
    codes = torch.randint(0, 1 << bits, (64, 48), generator=g)
    assert torch.equal(int4_ckpt.unpack_rows(pack_rows_ref(codes, bits), bits), codes)
    assert torch.equal(int4_ckpt.unpack_cols(pack_cols_ref(codes, bits), bits), codes)


def test_awq_unpack_round_trip():
    codes = torch.randint(0, 16, (16, 32), generator=torch.Generator().manual_seed(1))
    assert torch.equal(int4_ckpt.unpack_cols(pack_cols_ref(codes, 4, AWQ_ORDER), 4, AWQ_ORDER), codes)
    assert not torch.equal(int4_ckpt.unpack_cols(pack_cols_ref(codes, 4, AWQ_ORDER), 4), codes)


def _gptq_tensors(W, group, bits=4, act_order=False, sym=True, gen=None):
    """Quantise W [N, K] the GPTQ way: per-group scale / zero per output, optional
    act-order (a row permutation recorded in g_idx)."""
    N, K = W.shape
    maxq = (1 << bits) - 1
    perm = torch.randperm(K, generator=gen) if act_order else torch.arange(K)
    g_idx = torch.empty(K, dtype=torch.int32)
    g_idx[perm] = (torch.arange(K) // group).to(torch.int32)   # groups over the permuted order
    G = K // group
    scales = torch.empty(G, N)
    zeros = torch.empty(G, N, dtype=torch.int64)
    for gi in range(G):
        cols = perm[gi * group:(gi + 1) * group]
        blk = W[:, cols]
        if sym:
            s = blk.abs().amax(1).clamp_min(1e-8) * 2 / maxq
            z = torch.full((N,), (maxq + 1) // 2, dtype=torch.int64)
        else:
            lo, hi = blk.amin(1), blk.amax(1)
            s = ((hi - lo) / maxq).clamp_min(1e-8)
            z = torch.round(-lo / s).to(torch.int64).clamp(0, maxq)
        scales[gi], zeros[gi] = s, z
    scales = scales.half()
    q = torch.empty(K, N, dtype=torch.int64)
    for k in range(K):
        gi = int(g_idx[k])
        q[k] = torch.clamp(torch.round(W[:, k] / scales[gi].float()) + zeros[gi], 0, maxq).to(torch.int64)
    return {"qweight": pack_rows_ref(q, bits), "qzeros": pack_cols_ref(zeros - 1, bits),   # v1: zeros - 1
            "scales": scales, "g_idx": g_idx}, q, zeros


def test_gptq_dequantize_matches_elementwise_rule():
    gen = torch.Generator().manual_seed(0)
    W = torch.randn(16, 64, generator=gen)
    t, q, z = _gptq_tensors(W, 16, act_order=True, sym=False, gen=gen)
    got = int4_ckpt.gptq_dequantize(t["qweight"], t["qzeros"], t["scales"], t["g_idx"], group_size=16)
    want = torch.empty(16, 64)
    for n in range(16):
        for k in range(64):
            gi = int(t["g_idx"][k])
            want[n, k] = float(t["scales"][gi, n]) * (int(q[k, n]) - int(z[gi, n]))
    torch.testing.assert_close(got, want, rtol=0, atol=1e-6)
    assert (got - W).abs().max() < 0.5 * t["scales"].float().max() + 1e-6     # within half a step


def test_awq_dequantize_matches_elementwise_rule():
    gen = torch.Generator().manual_seed(1)
    K, N, group = 64, 32, 16
    q = torch.randint(0, 16, (K, N), generator=gen)
    z = torch.randint(0, 16, (K // group, N), generator=gen)
    s = (torch.rand(K // group, N, generator=gen) * 0.1 + 0.01).half()
    got = int4_ckpt.awq_dequantize(pack_cols_ref(q, 4, AWQ_ORDER), pack_cols_ref(z, 4, AWQ_ORDER), s, group_size=group)
    want = torch.empty(N, K)
    for n in range(N):
        for k in range(K):
            want[n, k] = float(s[k // group, n]) * (int(q[k, n]) - int(z[k // group, n]))
    torch.testing.assert_close(got, want, rtol=0, atol=1e-6)


def test_unsupported_layouts_are_refused():
    for qc in ({"quant_method": "gptq", "checkpoint_format": "marlin"}, {"quant_method": "gptq", "bits": 3},
               {"quant_method": "awq", "version": "gemv"}, {"quant_method": "bitsandbytes"}):
        with pytest.raises(int4_ckpt.UnsupportedQuantization):
            int4_ckpt.check_config(qc)


@pytest.mark.parametrize("method", ["gptq", "gptq_act_order", "awq"])
def test_quantised_checkpoint_loads_as_its_dequantised_model(method, tmp_path):
    T = pytest.importorskip("transformers")
    from safetensors.torch import save_file

    from vramancer_b200 import LLM
    from vramancer_b200.engine.runner import PrefillItem
    gen = torch.Generator().manual_seed(7)
    hf = T.Qwen2ForCausalLM(T.Qwen2Config(vocab_size=256, hidden_size=128, num_hidden_layers=2, num_attention_heads=4,
                                          num_key_value_heads=2, intermediate_size=256, max_position_embeddings=256,
                                          tie_word_embeddings=False)).eval()
    with torch.no_grad():
        for n, p in hf.named_parameters():
            p.copy_(torch.randn(p.shape, generator=gen) * (0.15 if p.dim() > 1 else 0.05) + (1.0 if "norm" in n else 0))
    group = 32
    sd, dense = {}, {}
    for name, t in hf.state_dict().items():
        mod = name.rsplit(".", 1)[0]
        if name.endswith(".weight") and t.dim() == 2 and ".layers." in name:
            if method.startswith("gptq"):
                tens, _, _ = _gptq_tensors(t.float(), group, act_order=method.endswith("act_order"), sym=True, gen=gen)
                if not method.endswith("act_order"):
                    tens.pop("g_idx")
                qc = {"quant_method": "gptq", "bits": 4, "group_size": group, "desc_act": method.endswith("order"),
                      "sym": True, "checkpoint_format": "gptq"}
                w = int4_ckpt.gptq_dequantize(tens["qweight"], tens["qzeros"], tens["scales"], tens.get("g_idx"),
                                              group_size=group)
            else:
                Nn, Kk = t.shape
                lo, hi = t.float().view(Nn, Kk // group, group).amin(2), t.float().view(Nn, Kk // group, group).amax(2)
                s = ((hi - lo) / 15).clamp_min(1e-8).t().half()                      # [G, N]
                z = torch.round(-lo.t() / s.float()).clamp(0, 15).to(torch.int64)   # [G, N]
                g = torch.arange(Kk) // group
                q = torch.clamp(torch.round(t.float().t() / s.float()[g]) + z[g], 0, 15).to(torch.int64)  # [K, N]
                tens = {"qweight": pack_cols_ref(q, 4, AWQ_ORDER), "qzeros": pack_cols_ref(z, 4, AWQ_ORDER),
                        "scales": s}
                qc = {"quant_method": "awq", "bits": 4, "group_size": group, "version": "gemm", "zero_point": True}
                w = int4_ckpt.awq_dequantize(tens["qweight"], tens["qzeros"], tens["scales"], group_size=group)
            for leaf, v in tens.items():
                sd[f"{mod}.{leaf}"] = v.contiguous()
            dense[name] = w
        else:
            sd[name] = t.contiguous()
            dense[name] = t
    save_file(sd, str(tmp_path / "model.safetensors"))
    cfg = hf.config.to_dict()
    cfg["quantization_config"] = qc
    (tmp_path / "config.json").write_text(json.dumps(cfg))
    kw = dict(device="cpu", dtype=torch.float32, kv_cache_dtype="fp32", kv_pages=32, max_model_len=128,
              use_cuda_graph=False, fold_norms=False)
    llm = LLM(str(tmp_path), **kw)
    hf.load_state_dict(dense)                         # transformers with the dequantised weights
    ids = list(range(3, 23))
    kv = llm.engine.kv
    kv.allocate("q", len(ids))
    got = llm.engine.runner.prefill_logits([PrefillItem(ids, 0, kv.slots_for("q", 0, len(ids)), kv.block_table("q"),
                                                        len(ids), True)])[-1]
    with torch.no_grad():
        ref = hf(torch.tensor([ids])).logits[0, -1]
    assert (got - ref).abs().max() <= 2e-4 * max(ref.abs().max().item(), 1.0)
