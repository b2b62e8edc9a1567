"""Model runner: builds forward batches from host metadata and executes them, with
decode steps replayed from CUDA graphs.

Decode inputs live in one device staging buffer that is filled by a single
host->device copy per step from pinned memory (token ids, positions, cache slots,
context lengths, block tables, sampling parameters); the captured graph reads views
of it and writes the sampled token ids into a device buffer that is copied back to
pinned memory.  One graph per batch-size bucket (1, 2, 4, 8, 16, 32, ... max_batch);
padded rows have context length 0 and slot -1, so they neither read nor write KV.

Reference parity: core/cuda_graph_decode.py:59-257 (per-batch-size graph cache,
single device, rejects dynamic caches) and core/turbo_engine.py:432-603 (graph with
argmax inside, zero-sync greedy loop).  Here the graph covers the whole paged decode
step including sampling, at any batch bucket.
"""
from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Dict, List, Optional, Sequence

import numpy as np
import torch

from .. import ops
from ..kv.pool import KVPool
from ..models.transformer import DecoderModel, ForwardBatch

DEFAULT_BUCKETS = (1, 2, 4, 8, 16, 32, 48, 64, 96, 128, 192, 256)


@dataclass
class PrefillItem:
    token_ids: Sequence[int]      # new tokens of this chunk
    start_pos: int                # absolute position of token_ids[0]
    slots: Sequence[int]          # cache slot per new token
    block_table: Sequence[int]
    context_len: int              # start_pos + len(token_ids)
    want_logits: bool


class _Stage:
    """One pinned staging area (decode inputs + sampled ids) and the event recorded
    after the last copies that read or write it."""

    def __init__(self, n_i32: int, n_f32: int, B: int, pin: bool):
        self.h_i32 = torch.zeros(n_i32, dtype=torch.int32, pin_memory=pin)
        self.h_f32 = torch.zeros(n_f32, dtype=torch.float32, pin_memory=pin)
        self.h_out = torch.zeros(B, dtype=torch.int32, pin_memory=pin)
        self.event = torch.cuda.Event() if pin else None
        self.pending = False

    def record(self) -> None:
        self.event.record()
        self.pending = True

    def wait(self) -> None:
        if self.pending:
            self.event.synchronize()
            self.pending = False


class PendingDecode:
    """A launched decode step whose sampled ids have not been read yet."""

    def __init__(self, stage: _Stage, n: int):
        self.stage, self.n = stage, n


class ModelRunner:
    def __init__(self, model: DecoderModel, pool: KVPool, *, max_batch: int = 256, max_model_len: int = 4096,
                 use_cuda_graph: bool = True, buckets: Sequence[int] = DEFAULT_BUCKETS, seed: int = 0):
        self.model = model
        self.pool = pool
        self.device = model.device
        self.max_batch = max_batch
        self.max_model_len = max_model_len
        ref_pool = pool if pool is not None else model.pools[0]   # pipelines own one pool per stage
        self.page_size = ref_pool.spec.page_size
        self.max_pages = (max_model_len + self.page_size - 1) // self.page_size
        self.use_graph = use_cuda_graph and self.device.type == "cuda"
        self.buckets = sorted(b for b in buckets if b <= max_batch) or [max_batch]
        if self.buckets[-1] < max_batch:
            self.buckets.append(max_batch)
        self.seed = seed
        self._graphs: Dict[int, torch.cuda.CUDAGraph] = {}
        # vocabulary-parallel sampling (TP): the decode graph samples from this rank's
        # logits shard; steps with a row that needs the whole distribution (top-p without
        # top-k) replay a second graph that gathers full logits (_graphs_alt)
        self._vp_model = bool(getattr(model, "vocab_parallel", False))
        self._vp_step = self._vp_model
        self._graphs_alt: Dict[int, torch.cuda.CUDAGraph] = {}
        self._graph_pool = None
        self._alloc_decode_buffers()
        self.launches_per_decode = None
        # graph-replayed speculative verify: (batch bucket, tokens per sequence) ->
        # (graph, static buffers)
        self._verify: Dict[tuple, tuple] = {}

    # ------------------------------------------------------------------ buffers
    def _alloc_decode_buffers(self):
        B, P = self.max_batch, self.max_pages
        # int32 section: ids, pos, slots, ctx, topk, steps (6*B) + block tables (B*P)
        self._n_i32 = 6 * B + B * P
        self._n_f32 = 2 * B
        pin = self.device.type == "cuda"
        # two pinned staging areas: step n+1 is staged while step n's copies are in flight
        self._stages = [_Stage(self._n_i32, self._n_f32, B, pin) for _ in range(2)]
        self._stage_idx = 0
        self.d_i32 = torch.zeros(self._n_i32, dtype=torch.int32, device=self.device)
        self.d_f32 = torch.zeros(self._n_f32, dtype=torch.float32, device=self.device)
        d = self.d_i32
        self.d_ids, self.d_pos, self.d_slots = d[0:B], d[B:2 * B], d[2 * B:3 * B]
        self.d_ctx, self.d_topk, self.d_steps = d[3 * B:4 * B], d[4 * B:5 * B], d[5 * B:6 * B]
        self.d_bt = d[6 * B:].view(B, P)
        self.d_temp, self.d_topp = self.d_f32[0:B], self.d_f32[B:2 * B]
        self.d_out = torch.zeros(B, dtype=torch.int32, device=self.device)
        self._use_stage(0)

    def _use_stage(self, i: int) -> None:
        """Points the staging views (h_i32, h_f32, h_out, hn_*) at staging area i."""
        st = self._stages[i]
        B = self.max_batch
        self.h_i32, self.h_f32, self.h_out = st.h_i32, st.h_f32, st.h_out
        hn = self.h_i32.numpy()
        self.hn_ids, self.hn_pos, self.hn_slots = hn[0:B], hn[B:2 * B], hn[2 * B:3 * B]
        self.hn_ctx, self.hn_topk, self.hn_steps = hn[3 * B:4 * B], hn[4 * B:5 * B], hn[5 * B:6 * B]
        self.hn_bt = hn[6 * B:].reshape(B, self.max_pages)
        hf = self.h_f32.numpy()
        self.hn_temp, self.hn_topp = hf[0:B], hf[B:2 * B]

    def bucket_for(self, n: int) -> int:
        for b in self.buckets:
            if b >= n:
                return b
        raise ValueError(f"batch {n} exceeds max_batch {self.max_batch}")

    # ------------------------------------------------------------------ decode
    def _decode_batch(self, B: int) -> ForwardBatch:
        splits = ops.decode_attention_splits(B, self.model.kvh, self.max_pages) if self.device.type == "cuda" else 0
        return ForwardBatch(input_ids=self.d_ids[:B], positions=self.d_pos[:B], slot_mapping=self.d_slots[:B],
                            block_tables=self.d_bt[:B], context_lens=self.d_ctx[:B], is_decode=True,
                            attn_splits=splits)

    def _decode_body(self, B: int) -> None:
        batch = self._decode_batch(B)
        vp = self._vp_step
        if vp:
            self.model.set_vp_logits(True)
        try:
            logits = self.model.forward(batch, self.pool)
        finally:
            if vp:
                self.model.set_vp_logits(False)
        if logits is not None and vp:             # this rank's vocabulary shard
            self.model.sample_vocab_parallel(logits, self.d_temp[:B], self.d_topk[:B], self.d_topp[:B], self.seed,
                                             self.d_steps[:B], out=self.d_out[:B])
        elif logits is not None:                  # None: a pipeline stage before the last
            if logits.device != self.device:      # in-process pipeline: last stage on another GPU
                logits = logits.to(self.device)
            ops.sample(logits, self.d_temp[:B], self.d_topk[:B], self.d_topp[:B], self.seed, self.d_steps[:B],
                       out=self.d_out[:B])
        share = getattr(self.model, "share_sampled", None)
        if share is not None:                     # multi-process pipeline: every rank gets the ids
            share(self.d_out[:B])

    def stage_decode_inputs(self, ids, positions, slots, ctx, block_tables: List[Sequence[int]],
                            temperature, top_k, top_p, steps) -> int:
        """Fills the pinned staging buffers for n live rows; returns the bucket size."""
        n = len(ids)
        B = self.bucket_for(n) if self.use_graph else n
        self.hn_ids[:B] = 0
        self.hn_pos[:B] = 0
        self.hn_slots[:B] = -1
        self.hn_ctx[:B] = 0
        self.hn_ids[:n] = ids
        self.hn_pos[:n] = positions
        self.hn_slots[:n] = slots
        self.hn_ctx[:n] = ctx
        self.hn_topk[:n] = top_k
        self.hn_steps[:n] = steps
        self.hn_temp[:n] = temperature
        self.hn_topp[:n] = top_p
        for r, bt in enumerate(block_tables):
            self.hn_bt[r, :len(bt)] = bt
        self._vp_step = self._vp_model and ops.vp_sampling_ok(temperature, top_k, top_p, self.model.cfg.vocab_size)
        return B

    def upload_decode_inputs(self) -> None:
        """One H2D copy of every decode input (the whole staging area)."""
        self.d_i32.copy_(self.h_i32, non_blocking=True)
        self.d_f32.copy_(self.h_f32, non_blocking=True)

    @property
    def h2d_bytes_per_decode(self) -> int:
        return self.h_i32.numel() * 4 + self.h_f32.numel() * 4

    def decode(self, B: int) -> torch.Tensor:
        """Runs one decode step for bucket B on the uploaded inputs; returns d_out[:B]."""
        if self.use_graph:
            g = (self._graphs if self._vp_step == self._vp_model else self._graphs_alt).get(B)
            if g is None:
                g = self.capture(B)
            g.replay()
        else:
            self._decode_body(B)
        return self.d_out[:B]

    def launch_decode(self, ids, positions, slots, ctx, block_tables, temperature, top_k, top_p, steps, *,
                      ids_on_device: bool = False) -> "PendingDecode":
        """Stages, uploads and launches one decode step without waiting for it; the
        sampled ids are copied into pinned memory behind it (collect_decode reads them).
        With ids_on_device the token fed to row r is row r of the previous step's
        sampled output, still on the device: the host launches step n+1 before it has
        read step n's tokens, so its scheduling overlaps the GPU's work."""
        n = len(positions)
        st = self._stages[self._stage_idx]
        st.wait()                               # this area's previous copies have run
        self._use_stage(self._stage_idx)
        B = self.stage_decode_inputs(ids if not ids_on_device else [0] * n, positions, slots, ctx, block_tables,
                                     temperature, top_k, top_p, steps)
        self.upload_decode_inputs()
        if ids_on_device:
            self.d_ids[:n].copy_(self.d_out[:n], non_blocking=True)
        out = self.decode(B)
        if self.device.type == "cuda":
            st.h_out[:B].copy_(out, non_blocking=True)
            st.record()
        else:
            st.h_out[:B].copy_(out)
        self._stage_idx ^= 1
        return PendingDecode(st, n)

    def collect_decode(self, p: "PendingDecode") -> List[int]:
        """Waits for a launched decode step and returns its sampled ids."""
        p.stage.wait()
        return p.stage.h_out[:p.n].tolist()

    def decode_step(self, ids, positions, slots, ctx, block_tables, temperature, top_k, top_p, steps) -> List[int]:
        """Host-to-host decode step: stage, upload, run, read back the sampled ids."""
        return self.collect_decode(self.launch_decode(ids, positions, slots, ctx, block_tables, temperature,
                                                      top_k, top_p, steps))

    def capture(self, B: int) -> torch.cuda.CUDAGraph:
        """Warm up (allocates split workspaces) and capture the decode graph of bucket B."""
        # warm-up on zeroed inputs: slot -1 / ctx 0 rows touch no KV
        saved_i, saved_f = self.d_i32.clone(), self.d_f32.clone()
        self.d_ids[:B].zero_()
        self.d_slots[:B].fill_(-1)
        self.d_ctx[:B].zero_()
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            self._decode_body(B)
        torch.cuda.current_stream().wait_stream(s)
        torch.cuda.synchronize()
        self.d_i32.copy_(saved_i)
        self.d_f32.copy_(saved_f)
        g = torch.cuda.CUDAGraph()
        if self._graph_pool is None:
            self._graph_pool = torch.cuda.graph_pool_handle()
        with torch.cuda.graph(g, pool=self._graph_pool):
            self._decode_body(B)
        torch.cuda.synchronize()
        (self._graphs if self._vp_step == self._vp_model else self._graphs_alt)[B] = g
        return g

    def capture_all(self, sizes: Optional[Sequence[int]] = None) -> None:
        if not self.use_graph:
            return
        step_vp, self._vp_step = self._vp_step, self._vp_model    # the default variant
        try:
            for B in sorted(sizes or self.buckets, reverse=True):
                if B not in self._graphs:
                    self.capture(B)
        finally:
            self._vp_step = step_vp

    def copy_pages(self, pairs) -> None:
        """Copy-on-write page copies (src, dst) in every KV pool this runner drives."""
        if hasattr(self.model, "copy_pages"):
            self.model.copy_pages(pairs)
            return
        for src, dst in pairs:
            self.pool.cache[dst].copy_(self.pool.cache[src])

    def release_graphs(self) -> None:
        self._graphs.clear()
        self._graphs_alt.clear()
        self._verify.clear()
        self._graph_pool = None

    # ------------------------------------------------------------------ prefill
    def prefill(self, items: List[PrefillItem], temperature, top_k, top_p, steps) -> List[Optional[int]]:
        """Runs one (chunked) prefill forward over several sequences; returns the
        sampled next token for items with want_logits (None for the others)."""
        dev = self.device
        ids, pos, slots, cu, ctx = [], [], [], [0], []
        maxp = 1
        for it in items:
            n = len(it.token_ids)
            ids.extend(it.token_ids)
            pos.extend(range(it.start_pos, it.start_pos + n))
            slots.extend(it.slots)
            cu.append(cu[-1] + n)
            ctx.append(it.context_len)
            maxp = max(maxp, len(it.block_table))
        B = len(items)
        bt = np.zeros((B, maxp), dtype=np.int32)
        for r, it in enumerate(items):
            bt[r, :len(it.block_table)] = it.block_table
        rows = [cu[r + 1] - 1 for r, it in enumerate(items) if it.want_logits]
        meta = np.concatenate([np.asarray(ids, np.int32), np.asarray(pos, np.int32), np.asarray(slots, np.int32),
                               np.asarray(cu, np.int32), np.asarray(ctx, np.int32), bt.reshape(-1),
                               np.asarray(rows, np.int32)])
        h = torch.from_numpy(meta)
        if dev.type == "cuda":
            h = h.pin_memory()
        d = h.to(dev, non_blocking=True)
        T = len(ids)
        o = 0
        d_ids = d[o:o + T]; o += T
        d_pos = d[o:o + T]; o += T
        d_slots = d[o:o + T]; o += T
        d_cu = d[o:o + B + 1]; o += B + 1
        d_ctx = d[o:o + B]; o += B
        d_bt = d[o:o + B * maxp].view(B, maxp); o += B * maxp
        d_rows = d[o:o + len(rows)].long()
        batch = ForwardBatch(input_ids=d_ids, positions=d_pos, slot_mapping=d_slots, block_tables=d_bt,
                             context_lens=d_ctx, is_decode=False, cu_q=d_cu,
                             max_q_len=max(len(it.token_ids) for it in items), logits_rows=d_rows)
        if not rows:
            # no logits wanted: still run all layers (KV must be written)
            batch.logits_rows = d_rows
        logits = self.model.forward(batch, self.pool)
        if not rows:
            return [None] * B
        sel = [r for r, it in enumerate(items) if it.want_logits]
        if logits is not None:
            if logits.device != dev:
                logits = logits.to(dev)
            tt = torch.tensor([temperature[r] for r in sel], dtype=torch.float32)
            tk = torch.tensor([top_k[r] for r in sel], dtype=torch.int32)
            tp = torch.tensor([top_p[r] for r in sel], dtype=torch.float32)
            st = torch.tensor([steps[r] for r in sel], dtype=torch.int32)
            nxt_t = ops.sample(logits, tt.to(dev), tk.to(dev), tp.to(dev), self.seed, st.to(dev))
        else:                                     # a pipeline stage before the last
            nxt_t = torch.zeros(len(sel), dtype=torch.int32, device=dev)
        share = getattr(self.model, "share_sampled", None)
        if share is not None:
            share(nxt_t)
        nxt = nxt_t.cpu().tolist()
        res: List[Optional[int]] = [None] * B
        for j, r in enumerate(sel):
            res[r] = nxt[j]
        return res

    # ------------------------------------------------------------------ speculative verify
    VERIFY_TOKENS = (2, 3, 5, 9, 13, 17)     # tokens per sequence: 1 + draft length

    def _verify_buffers(self, B: int, T: int):
        P = self.max_pages
        n = 3 * B * T + B * P + B + (B + 1)
        d = torch.zeros(n, dtype=torch.int32, device=self.device)
        h = torch.zeros(n, dtype=torch.int32, pin_memory=True)
        views = {}
        o = 0
        for name, size in (("ids", B * T), ("pos", B * T), ("slots", B * T), ("bt", B * P), ("ctx", B),
                           ("cu", B + 1)):
            views[name] = (d[o:o + size], h[o:o + size])
            o += size
        out = torch.zeros(B * T, dtype=torch.int32, device=self.device)
        h_out = torch.zeros(B * T, dtype=torch.int32, pin_memory=True)
        return d, h, views, out, h_out

    def _verify_body(self, B: int, T: int, views, out) -> None:
        g = lambda k: views[k][0]   # noqa: E731
        batch = ForwardBatch(input_ids=g("ids"), positions=g("pos"), slot_mapping=g("slots"),
                             block_tables=g("bt").view(B, self.max_pages), context_lens=g("ctx"), is_decode=False,
                             cu_q=g("cu"), max_q_len=T, logits_rows=None)
        vp = self._vp_model
        if vp:
            self.model.set_vp_logits(True)
        try:
            logits = self.model.forward(batch, self.pool)
        finally:
            if vp:
                self.model.set_vp_logits(False)
        if vp:                                     # greedy over this rank's vocabulary shard
            z = torch.zeros(B * T, dtype=torch.float32, device=self.device)
            zi = torch.zeros(B * T, dtype=torch.int32, device=self.device)
            self.model.sample_vocab_parallel(logits, z, zi, z, 0, zi, out)
        else:
            ops.argmax(logits, out=out)

    def verify_greedy(self, items: List[PrefillItem]) -> Optional[List[List[int]]]:
        """The target's greedy token after every fed position of each item (a speculative
        verify step), from a CUDA graph per (batch bucket, tokens per sequence): every
        sequence feeds T tokens; positions past an item's tokens write no KV and their
        outputs are dropped.  None when it does not apply (no graphs, too many tokens)."""
        if not self.use_graph or not items:
            return None
        n = len(items)
        longest = max(len(it.token_ids) for it in items)
        T = next((t for t in self.VERIFY_TOKENS if t >= longest), None)
        if T is None or n > self.max_batch:
            return None
        B = self.bucket_for(n)
        key = (B, T)
        ent = self._verify.get(key)
        if ent is None:
            ent = self._verify_buffers(B, T)
        d, h, views, out, h_out = ent[:5]
        hn = {k: v[1].numpy() for k, v in views.items()}
        hn["ids"][:] = 0
        hn["pos"][:] = 0
        hn["slots"][:] = -1
        hn["ctx"][:] = 0
        hn["cu"][:] = [T * i for i in range(B + 1)]
        bt = hn["bt"].reshape(B, self.max_pages)
        maxpos = self.model.cfg.max_position - 1
        for r, it in enumerate(items):
            m = len(it.token_ids)
            ids = list(it.token_ids) + [it.token_ids[-1]] * (T - m)
            hn["ids"][r * T:(r + 1) * T] = ids
            hn["pos"][r * T:(r + 1) * T] = [min(it.start_pos + j, maxpos) for j in range(T)]
            hn["slots"][r * T:r * T + m] = list(it.slots)
            hn["ctx"][r] = it.start_pos + T
            bt[r, :] = 0
            bt[r, :len(it.block_table)] = it.block_table
        d.copy_(h, non_blocking=True)
        if len(ent) == 5:
            # warm-up on these inputs (writes only the items' own KV slots), then capture
            s = torch.cuda.Stream()
            s.wait_stream(torch.cuda.current_stream())
            with torch.cuda.stream(s):
                self._verify_body(B, T, views, out)
            torch.cuda.current_stream().wait_stream(s)
            torch.cuda.synchronize()
            graph = torch.cuda.CUDAGraph()
            if self._graph_pool is None:
                self._graph_pool = torch.cuda.graph_pool_handle()
            with torch.cuda.graph(graph, pool=self._graph_pool):
                self._verify_body(B, T, views, out)
            ent = ent + (graph,)
            self._verify[key] = ent
        ent[5].replay()
        h_out.copy_(out, non_blocking=True)
        torch.cuda.current_stream().synchronize()
        o = h_out.numpy()
        return [o[r * T:r * T + len(it.token_ids)].tolist() for r, it in enumerate(items)]

    def prefill_logits(self, items: List[PrefillItem]) -> torch.Tensor:
        """Prefill returning the raw logits rows (for scoring / speculative verify)."""
        dev = self.device
        ids, pos, slots, cu, ctx = [], [], [], [0], []
        maxp = max(len(it.block_table) for it in items)
        for it in items:
            n = len(it.token_ids)
            ids.extend(it.token_ids)
            pos.extend(range(it.start_pos, it.start_pos + n))
            slots.extend(it.slots)
            cu.append(cu[-1] + n)
            ctx.append(it.context_len)
        bt = torch.zeros(len(items), maxp, dtype=torch.int32)
        for r, it in enumerate(items):
            bt[r, :len(it.block_table)] = torch.tensor(it.block_table, dtype=torch.int32)
        i32 = lambda v: torch.tensor(v, dtype=torch.int32, device=dev)
        batch = ForwardBatch(input_ids=i32(ids), positions=i32(pos), slot_mapping=i32(slots),
                             block_tables=bt.to(dev), context_lens=i32(ctx), is_decode=False, cu_q=i32(cu),
                             max_q_len=max(len(it.token_ids) for it in items), logits_rows=None)
        return self.model.forward(batch, self.pool)
