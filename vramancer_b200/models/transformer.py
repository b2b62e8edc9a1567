"""Decoder forward pass over the paged KV pool, for one pipeline stage / TP rank.

The residual stream `r` is a [T, H] buffer that every layer updates in place:
  TP = 1   the o_proj and down_proj GEMMs add their product into `r` in the GEMM
           epilogue (no separate residual kernel), then a plain RMSNorm reads `r`;
  TP > 1   row-parallel partial sums are all-reduced first (fused kernel or NCCL)
           and added by the residual-fused RMSNorm / an add kernel.
Per dense layer at TP=1: RMSNorm, QKV GEMM(+bias), RoPE+KV-page write, paged
attention, O GEMM(+residual), RMSNorm, gate/up GEMM(+SiLU*up), down GEMM(+residual):
eight launches, all of them sm_100a kernels of this package.

Reference parity: the reference runs HF modules (core/backends.py:1629-1852 manual
path, core/turbo_engine.py:194-254 TurboForward) and its own TP layer in
core/tensor_parallel.py:172-445 (no KV cache there); this module owns the forward.
"""
from __future__ import annotations

import math
import os
from dataclasses import dataclass, field
from typing import Callable, List, Optional

import torch

from .. import ops
from ..kv.pool import KVPool
from .config import ModelConfig
from .weights import Weights


@dataclass
class ForwardBatch:
    """Device-side metadata of one forward.

    decode:  T == B tokens, one per sequence; context_lens include the new token.
    prefill: tokens of B sequences concatenated; cu_q [B+1] delimits them;
             context_lens = cached prefix + new tokens; logits_rows selects the rows
             whose logits are needed (last token of each finished prompt).
    """
    input_ids: torch.Tensor
    positions: torch.Tensor
    slot_mapping: torch.Tensor
    block_tables: torch.Tensor
    context_lens: torch.Tensor
    is_decode: bool
    cu_q: Optional[torch.Tensor] = None
    max_q_len: int = 1
    logits_rows: Optional[torch.Tensor] = None
    attn_splits: int = 0

    @property
    def num_tokens(self) -> int:
        return self.input_ids.shape[0]


class TPContext:
    """What a tensor-parallel rank needs from the communication layer."""

    def __init__(self, rank: int, size: int, all_reduce: Callable[[torch.Tensor], torch.Tensor],
                 all_gather_last: Callable[[torch.Tensor], torch.Tensor], fused_ar=None,
                 all_gather_stack: Optional[Callable[[torch.Tensor], torch.Tensor]] = None):
        self.rank, self.size = rank, size
        self.all_reduce = all_reduce
        self.all_gather_last = all_gather_last
        # optional FusedAllReduce: row-parallel GEMM with the all-reduce in its epilogue
        self.fused_ar = fused_ar
        # x [...] -> [ranks, ...] (every rank's x): the candidate exchange of
        # vocabulary-parallel sampling; None keeps full-logit gathers
        self.all_gather_stack = all_gather_stack


# Returned in place of a normalised activation when the next GEMM applies the RMSNorm
# itself (decode with folded norms): it reads the residual stream and the per-token
# sums of squares the previous GEMM stored.
_FOLDED = object()
FOLD_MAX_TOKENS = int(os.environ.get("VRM_FOLD_MAX_TOKENS", "16"))
# Under tensor parallelism the folded norm replaces the reduce kernel altogether (the
# row-parallel GEMM reduces and stores the norm sums itself): every fused decode batch.
FOLD_MAX_TOKENS_TP = int(os.environ.get("VRM_FOLD_MAX_TOKENS_TP", "128"))


class DecoderModel:
    def __init__(self, cfg: ModelConfig, weights: Weights, *, device="cpu", dtype=torch.bfloat16,
                 first_layer: int = 0, last_layer: Optional[int] = None, tp: Optional[TPContext] = None,
                 ep=None):
        self.cfg = cfg
        self.ep = ep                  # parallel.expert_parallel.ExpertParallel (experts sharded) or None
        self.w = weights
        self.device = torch.device(device)
        self.dtype = dtype
        self.first_layer = first_layer
        self.last_layer = cfg.num_layers if last_layer is None else last_layer
        self.has_embed = first_layer == 0
        self.has_head = self.last_layer == cfg.num_layers
        self.tp = tp
        tps = tp.size if tp else 1
        self.tp_size = tps
        self.hq = cfg.num_heads // tps
        self.kvh = max(1, cfg.num_kv_heads // tps)
        self.D = cfg.head_dim
        self.sm_scale = 1.0 / math.sqrt(cfg.head_dim)
        self._rope_dummy = None      # one-page bf16 pool for RoPE without a KV write (TurboQuant pages)
        self.cos_sin = (ops.rope_cos_sin(cfg.max_position, cfg.rot_dim, cfg.rope_theta, self.device,
                                          scaling=cfg.rope_scaling)
                        if cfg.rot_dim > 0 else None)
        # decode attention does RoPE + the KV write itself when rotation covers the whole
        # head (or there is none); VRM_FUSED_ROPE=0 keeps the separate kernel
        self.fused_rope = (cfg.rot_dim in (0, cfg.head_dim) and cfg.head_dim in (64, 128)
                           and os.environ.get("VRM_FUSED_ROPE", "1") != "0")
        # folded RMSNorm (fold_norms): weights already folded by another model over the
        # same tensors are detected, so every model on them normalises without weight
        self._ssq = None
        self._ssq_parts = 0
        self._fold_active = False
        first_qkv = self.lw(self.first_layer, "qkv_w") if self.last_layer > self.first_layer else None
        self.folded = getattr(first_qkv, "_vrm_norm_w", None) is not None
        self._ones = (torch.ones(cfg.hidden_size, dtype=dtype, device=self.device) if self.folded else None)

    @property
    def num_local_layers(self) -> int:
        return self.last_layer - self.first_layer

    def lw(self, i: int, name: str) -> Optional[torch.Tensor]:
        return self.w.get(f"layers.{i}.{name}")

    # ------------------------------------------------------------------ pieces
    def embed(self, batch: ForwardBatch) -> torch.Tensor:
        cfg = self.cfg
        if cfg.is_gpt2:
            return ops.embedding(batch.input_ids, self.w["embed"], positions=batch.positions,
                                 pos_table=self.w["pos_embed"])
        return ops.embedding(batch.input_ids, self.w["embed"])

    def fold_norms(self) -> bool:
        """Folds each layer's input and post-attention RMSNorm weight into the columns of
        the GEMM that consumes the normalised activation (qkv_w, gate_up_w: W' = W
        diag(w_norm), in place, marked on the tensor), so that small decode batches run
        the norms inside the GEMMs: the GEMM that adds into the residual stream stores
        per-token sums of squares of its output, the next GEMM reads the residual stream
        and scales by rsqrt(mean + eps) (two launches fewer per layer).  Prefill and
        larger batches normalise without weight and use W'.  Dense RMSNorm models at
        TP = 1 with resident bf16 CUDA weights; returns whether the weights are folded."""
        cfg = self.cfg
        if self.folded:
            return self._alloc_fold()
        if (self.device.type != "cuda" or not self._fold_capable() or cfg.is_gpt2 or cfg.is_moe
                or self.dtype != torch.bfloat16 or cfg.hidden_size > 64 * 128 or self.last_layer <= self.first_layer):
            return False
        pairs = []
        for i in range(self.first_layer, self.last_layer):
            for wk, nk in (("qkv_w", "in_norm_w"), ("gate_up_w", "post_norm_w")):
                W, nw = self.lw(i, wk), self.lw(i, nk)
                if (not isinstance(W, torch.Tensor) or getattr(W, "_vrm_quant", None) is not None or nw is None
                        or W.dtype != torch.bfloat16 or W.device.type != "cuda" or W.shape[1] != nw.numel()
                        or (self.device.index is not None and W.device.index != self.device.index)):
                    return False
                pairs.append((W, nw))
        for W, nw in pairs:
            W.mul_(nw.to(W.dtype).view(1, -1))
            W._vrm_norm_w = nw.detach().clone()
        self.folded = True
        self._ones = torch.ones(cfg.hidden_size, dtype=self.dtype, device=self.device)
        return self._alloc_fold()

    def _fold_capable(self) -> bool:
        """One GPU, or tensor parallelism with the fused all-reduce (whose row-parallel
        GEMM stores the norm sums of the reduced residual)."""
        return self.tp_size == 1 or (self.tp is not None and self.tp.fused_ar is not None)

    def _alloc_fold(self) -> bool:
        if self.device.type == "cuda" and self._fold_capable() and self._ssq is None:
            self._ssq_parts = (self.cfg.hidden_size + 127) // 128
            self._ssq = torch.zeros(self._ssq_parts, 128, dtype=torch.float32, device=self.device)
        return self.folded

    def _in_proj(self, x, r: torch.Tensor, w, b, epilogue: int = 0) -> torch.Tensor:
        """The GEMM that consumes a normalised activation (or, folded, the residual stream)."""
        if x is _FOLDED:
            return ops.linear(r, w, b, epilogue=epilogue, ssq_in=self._ssq, ssq_parts=self._ssq_parts,
                              norm_eps=self.cfg.norm_eps)
        return ops.linear(x, w, b, epilogue=epilogue)

    def _norm(self, x, i_or_name, which: str, residual=None):
        cfg = self.cfg
        if isinstance(i_or_name, int):
            w = self.lw(i_or_name, f"{which}_w")
            b = self.lw(i_or_name, f"{which}_b")
            if self.folded and which in ("in_norm", "post_norm"):
                w = self._ones          # the weight lives in the next GEMM's columns
        else:
            w, b = self.w["final_norm_w"], self.w.get("final_norm_b")
        if cfg.is_gpt2:
            return ops.layernorm(x, w, b, cfg.norm_eps, residual=residual)
        return ops.rmsnorm(x, w, cfg.norm_eps, residual=residual)

    def _attention(self, i: int, x, batch: ForwardBatch, pool: KVPool, r: Optional[torch.Tensor] = None) -> torch.Tensor:
        cfg = self.cfg
        hq, kvh, D = self.hq, self.kvh, self.D
        qkv = self._in_proj(x, r, self.lw(i, "qkv_w"), self.lw(i, "qkv_b"))
        if cfg.qk_norm:          # Qwen3: per-head RMSNorm of q and k before RoPE
            ops.qk_rmsnorm(qkv, self.lw(i, "q_norm_w"), self.lw(i, "k_norm_w"), hq, kvh, D, cfg.norm_eps)
        li = i - self.first_layer
        if getattr(pool, "is_tq", False):
            return self._attention_tq(qkv, batch, pool, li)
        # decode attention leaves HBM bandwidth spare at short contexts: it prefetches the
        # o_proj weights into L2 for the GEMM that follows it
        pf = self._o_prefetch(i) if batch.is_decode and qkv.is_cuda else None
        if batch.is_decode and self.fused_rope and qkv.is_cuda:
            # RoPE + KV-page write inside the decode attention kernel (one launch fewer)
            return ops.paged_attention_decode(qkv, pool.cache, li, batch.block_tables, batch.context_lens,
                                              pool.kv_scale, self.sm_scale, hq, num_splits=batch.attn_splits,
                                              positions=batch.positions, cos_sin=self.cos_sin,
                                              slot_mapping=batch.slot_mapping, l2_prefetch=pf)
        ops.rope_kv_write(qkv, batch.positions, self.cos_sin, pool.cache, batch.slot_mapping, pool.kv_scale,
                          li, hq, kvh, D)
        if batch.is_decode:
            return ops.paged_attention_decode(qkv, pool.cache, li, batch.block_tables, batch.context_lens,
                                              pool.kv_scale, self.sm_scale, hq, num_splits=batch.attn_splits,
                                              l2_prefetch=pf)
        return ops.paged_attention_prefill(qkv, pool.cache, li, batch.block_tables, batch.cu_q,
                                           batch.context_lens, pool.kv_scale, self.sm_scale, hq,
                                           batch.max_q_len)

    def _o_prefetch(self, i: int) -> Optional[torch.Tensor]:
        """The tensor holding layer i's o_proj weights (bf16 / fp8 matrix, or NVFP4
        codes), for the decode attention kernel's L2 prefetch; None when there is none."""
        w = self.lw(i, "o_w")
        if isinstance(w, torch.Tensor):
            return w if w.is_contiguous() else None
        codes = getattr(w, "q", None)             # NVFP4Weight / FP8Weight codes
        return codes if isinstance(codes, torch.Tensor) and codes.is_contiguous() else None

    def _attention_tq(self, qkv: torch.Tensor, batch: ForwardBatch, pool: KVPool, li: int) -> torch.Tensor:
        """Attention over TurboQuant KV pages: RoPE in place, the step's k / v written as
        records, decode scored from the records; prefill decodes the batch's pages of this
        layer to bf16 and runs the regular prefill kernel on them."""
        hq, kvh, D = self.hq, self.kvh, self.D
        if self._rope_dummy is None:
            # RoPE without a KV write goes through the same kernel with a one-page bf16 pool
            self._rope_dummy = torch.zeros(1, 1, 2, kvh, 16, D, dtype=torch.bfloat16, device=qkv.device)
        ops.rope_kv_write(qkv, batch.positions, self.cos_sin, self._rope_dummy, None, None, 0, hq, kvh, D)
        ops.tq_kv_write(qkv, batch.slot_mapping, pool.cache, li, hq, kvh, pool.tq)
        if batch.is_decode:
            return ops.tq_paged_decode(qkv, pool.cache, li, batch.block_tables, batch.context_lens, pool.tq,
                                       self.sm_scale, hq)
        bt = batch.block_tables
        pages = bt.reshape(-1)
        mini = ops.tq_decompress_pool(pool.cache, li, pages, pool.tq)
        bt_mini = torch.arange(pages.numel(), dtype=torch.int32, device=bt.device).view(bt.shape)
        return ops.paged_attention_prefill(qkv, mini, 0, bt_mini, batch.cu_q, batch.context_lens, None,
                                           self.sm_scale, hq, batch.max_q_len)

    def _row_parallel(self, x: torch.Tensor, w: torch.Tensor, b: Optional[torch.Tensor], r: torch.Tensor,
                      nxt: Optional[tuple]) -> Optional[torch.Tensor]:
        """r += x @ w.T (+ b) across the TP group; returns norm(r) when `nxt` names the
        norm that follows ((layer, "post_norm" | "in_norm") or (None, "final"))."""
        if self.tp_size == 1:
            if self._fold_active and nxt and nxt[0] is not None:
                # the next GEMM normalises: store the per-token sums of squares instead
                ops.linear(x, w, b, residual=r, out=r, ssq_out=self._ssq)
                return _FOLDED
            ops.linear(x, w, b, residual=r, out=r)
            return self._norm(r, nxt[0] if nxt[0] is not None else "final", nxt[1]) if nxt else None
        far = self.tp.fused_ar
        if far is not None and x.is_cuda and self._fold_active and far.supports_reduce(x.shape[0], w):
            # one kernel: GEMM, push to every rank, reduce + bias into the residual stream
            # and the norm sums the next GEMM normalises from
            last = not nxt or nxt[0] is None
            far.push_reduce(x, w, residual=r, bias=b, ssq_out=None if last else self._ssq)
            if not nxt:
                return None
            return _FOLDED if not last else self._norm(r, "final", "final")
        if far is not None and x.is_cuda and far.supports_weight(x.shape[0], w):
            # push the partial to every rank (bf16, fp8 or NVFP4 weights), then one
            # kernel: reduce + bias + residual + norm
            T, H = x.shape[0], w.shape[0]
            far.push_weight(x, w)
            if not nxt:
                far.reduce(T, H, bias=b, residual=r)
                return None
            nw, nb = self._norm_params(*nxt)
            out = torch.empty_like(r)
            far.reduce(T, H, bias=b, residual=r, out=out, norm_w=nw, norm_b=nb, eps=self.cfg.norm_eps,
                       layernorm=self.cfg.is_gpt2)
            return out
        y = ops.linear(x, w)
        y = self.tp.all_reduce(y)
        if b is not None:
            ops.add_(y, b.expand_as(y).contiguous())
        if nxt:
            return self._norm(y, nxt[0] if nxt[0] is not None else "final", nxt[1], residual=r)
        ops.add_(r, y)
        return None

    def _norm_params(self, i: Optional[int], which: str):
        if i is None:
            return self.w["final_norm_w"], self.w.get("final_norm_b")
        if self.folded and which in ("in_norm", "post_norm"):
            return self._ones, None          # the weight lives in the next GEMM's columns
        return self.lw(i, f"{which}_w"), self.lw(i, f"{which}_b")

    def _mlp(self, i: int, x: torch.Tensor, r: torch.Tensor, nxt: Optional[tuple]) -> Optional[torch.Tensor]:
        """MLP of layer i into r; returns the next norm's output when `nxt` is given and
        it could be fused into the MLP's output projection."""
        cfg = self.cfg
        if cfg.is_gpt2:
            h = ops.linear(x, self.lw(i, "fc_w"), self.lw(i, "fc_b"))
            ops.gelu_tanh_(h)
            return self._row_parallel(h, self.lw(i, "proj_w"), self.lw(i, "proj_b"), r, nxt)
        if cfg.is_moe:
            # residual add (and the next layer's input norm) fused into the combine
            return self._moe(i, x, r, self._norm_params(*nxt)[0] if nxt else None)
        a = self._in_proj(x, r, self.lw(i, "gate_up_w"), None, ops.EPI_SILU_MUL)
        return self._row_parallel(a, self.lw(i, "down_w"), None, r, nxt)

    def _moe(self, i: int, x: torch.Tensor, r: torch.Tensor, norm_w: Optional[torch.Tensor]) -> Optional[torch.Tensor]:
        """Top-k softmax routing over SwiGLU experts (device-scheduled grouped GEMM on
        CUDA, parallel/moe.py); r += MoE(x); returns RMSNorm(r) * norm_w when given."""
        from ..parallel.moe import expert_mlp, moe_forward
        if self.ep is not None:
            add = None
            sgu = self.lw(i, "shared_gate_up_w")
            if sgu is not None:
                ys = expert_mlp(x, sgu, self.lw(i, "shared_down_w"))
                sg = self.lw(i, "shared_gate_w")
                if sg is not None:
                    ys = (ys.float() * torch.sigmoid(ops.linear(x, sg).float())).to(x.dtype)
                add = ys.contiguous()
            return self.ep.forward(x, self.lw(i, "router_w"), self.lw(i, "experts_gate_up_w"),
                                   self.lw(i, "experts_down_w"), add=add, residual=r, norm_w=norm_w)
        return moe_forward(self.cfg, x, self.lw(i, "router_w"), self.lw(i, "experts_gate_up_w"),
                           self.lw(i, "experts_down_w"), shared_gate_up=self.lw(i, "shared_gate_up_w"),
                           shared_down=self.lw(i, "shared_down_w"), shared_gate=self.lw(i, "shared_gate_w"),
                           residual=r, norm_w=norm_w)

    def layer(self, i: int, r: torch.Tensor, batch: ForwardBatch, pool: KVPool,
              x: Optional[torch.Tensor] = None) -> Optional[torch.Tensor]:
        """Runs layer i on the residual stream r.  `x` is in_norm(r) when the previous
        layer already produced it; returns the next layer's in_norm(r) when it could be
        fused into this layer's last projection, else None."""
        if x is None:
            x = self._norm(r, i, "in_norm")
        attn = self._attention(i, x, batch, pool, r)
        x = self._row_parallel(attn, self.lw(i, "o_w"), self.lw(i, "o_b"), r, (i, "post_norm"))
        nxt = (i + 1, "in_norm") if i + 1 < self.last_layer else None
        return self._mlp(i, x, r, nxt)

    def logits(self, r: torch.Tensor, rows: Optional[torch.Tensor] = None) -> torch.Tensor:
        h = r if rows is None else r.index_select(0, rows)
        x = self._norm(h.contiguous(), "final", "final")
        lg = ops.linear(x, self.w["lm_head"])
        if self.tp_size > 1 and not self.vp_logits:
            lg = self.tp.all_gather_last(lg)[:, : self.cfg.vocab_size]
        return lg

    # ------------------------------------------------------------------ vocabulary-parallel sampling
    vp_logits = False   # set by the runner around a forward whose sampling is vocabulary-parallel

    @property
    def vocab_parallel(self) -> bool:
        """Decode sampling can run on this rank's logits shard (candidates exchanged
        between ranks instead of full logits): TP > 1 on CUDA with a candidate gather."""
        return (self.tp_size > 1 and self.has_head and self.device.type == "cuda"
                and getattr(self.tp, "all_gather_stack", None) is not None
                and os.environ.get("VRM_VP_SAMPLE", "1") != "0")

    def set_vp_logits(self, on: bool) -> None:
        self.vp_logits = bool(on)

    def sample_vocab_parallel(self, logits, temperature, top_k, top_p, seed, steps, out):
        """Samples from this rank's logits shard [B, V / tp]; every rank gets the same ids."""
        return ops.sample_vocab_parallel(logits, self.tp.rank * self.w["lm_head"].shape[0], self.cfg.vocab_size,
                                         temperature, top_k, top_p, seed, steps, self.tp.all_gather_stack, out=out)

    # ------------------------------------------------------------------ entry points
    def forward(self, batch: ForwardBatch, pool: KVPool, hidden: Optional[torch.Tensor] = None) -> torch.Tensor:
        """Runs this stage's layers.  The first stage embeds `batch.input_ids`; later
        stages take `hidden` (the residual stream from the previous stage).  The last
        stage returns logits of `batch.logits_rows` (all rows if None); other stages
        return the residual stream."""
        r = self.embed(batch) if self.has_embed else hidden
        if r is None:
            raise ValueError("non-first pipeline stage needs the hidden state")
        # small decode batches run the folded norms inside the GEMMs.  Measured on B200
        # (Qwen2.5-14B, graph-replayed step): batch 1 6.38 -> 6.26 ms, but batch 32 7.58 ->
        # 8.36 ms (the norm-sum epilogue and the per-token rsqrt cost more than the norm
        # launches they replace there), so batches above 16 keep the norm kernels.
        if self.tp_size == 1:
            limit = FOLD_MAX_TOKENS
        else:
            far = self.tp.fused_ar
            limit = min(FOLD_MAX_TOKENS_TP, far.max_tokens) if far is not None else 0
        self._fold_active = (self._ssq is not None and batch.is_decode and r.is_cuda and r.shape[0] <= limit)
        x = None
        for i in range(self.first_layer, self.last_layer):
            x = self.layer(i, r, batch, pool, x)
        if self.has_head:
            return self.logits(r, batch.logits_rows)
        return r
