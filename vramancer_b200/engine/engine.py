"""Continuous-batching LLM engine over the paged KV cache.

Each `step()`:
  1. admits waiting requests while the batch and the KV pool have room (prefix-cache
     hits skip the cached part of the prompt),
  2. runs one chunked-prefill forward over up to `max_prefill_tokens` prompt tokens of
     admitted requests (a request whose prompt completes gets its first token),
  3. runs one decode step (CUDA graph) for every request that is generating,
  4. applies stop conditions, streams tokens to callbacks, frees finished requests.
Requests join and leave at step granularity (iteration-level scheduling).  The KV of
a request stays in its pages for its whole life: nothing is concatenated or padded
per step.

Reference parity: ContinuousBatcher, core/continuous_batcher.py:106-1065 (waiting
queue, admission, chunked prefill at VRM_PREFILL_CHUNK, batched decode, per-request
sampling, streaming callback, futures) — which re-concatenates HF caches every step
(:828-891); here decode reads pages in place.
"""
from __future__ import annotations

import itertools
import os
import threading
import time
from collections import deque
from concurrent.futures import Future
from dataclasses import dataclass, field
from typing import Callable, Deque, Dict, List, Optional, Sequence

import torch

from ..kv.paged import OutOfPages, PagedKVCacheManager
from .runner import ModelRunner, PrefillItem


@dataclass
class SamplingParams:
    max_tokens: int = 16
    temperature: float = 0.0
    top_k: int = 0
    top_p: float = 1.0
    stop_token_ids: Sequence[int] = ()
    ignore_eos: bool = False

    @property
    def greedy(self) -> bool:
        return self.temperature <= 0.0


_ids = itertools.count()


@dataclass
class Request:
    prompt_ids: List[int]
    params: SamplingParams
    request_id: object = field(default_factory=lambda: f"req-{next(_ids)}")
    on_token: Optional[Callable[["Request", int], None]] = None
    output_ids: List[int] = field(default_factory=list)
    num_computed: int = 0          # tokens of prefill_ids whose KV is written
    cached_tokens: int = 0
    resumed: bool = False          # preempted after producing tokens: re-prefill, then keep decoding
    retries: int = 0               # re-runs after failed engine steps
    finished: bool = False
    finish_reason: Optional[str] = None
    arrival: float = field(default_factory=time.perf_counter)
    first_token_time: Optional[float] = None
    finish_time: Optional[float] = None
    future: Optional[Future] = None

    @property
    def prefill_ids(self) -> List[int]:
        """Tokens whose KV a prefill writes: the prompt, or after a preemption the prompt
        and every generated token but the last (which the next decode step feeds)."""
        if self.resumed and self.output_ids:
            return self.prompt_ids + self.output_ids[:-1]
        return self.prompt_ids

    @property
    def prefill_done(self) -> bool:
        return self.num_computed >= len(self.prefill_ids)

    @property
    def ttft(self) -> Optional[float]:
        return None if self.first_token_time is None else self.first_token_time - self.arrival

    @property
    def total_len(self) -> int:
        return len(self.prompt_ids) + len(self.output_ids)


class LLMEngine:
    def __init__(self, runner: ModelRunner, manager: PagedKVCacheManager, *, max_batch: Optional[int] = None,
                 max_prefill_tokens: int = 8192, eos_token_id: Optional[int] = None, spec_num_draft: int = 0,
                 spec_ngram: int = 3, ep_sync: Optional["EPSync"] = None, lookahead: bool = True):
        if ep_sync is not None and spec_num_draft > 0:
            raise ValueError("speculative decoding is not supported with expert parallelism")
        self.ep_sync = ep_sync
        self.runner = runner
        self.kv = manager
        self.max_batch = max_batch or runner.max_batch
        self.max_prefill_tokens = max_prefill_tokens
        self.max_model_len = runner.max_model_len
        self.eos_token_id = eos_token_id
        self.waiting: Deque[Request] = deque()
        self.running: List[Request] = []
        self._lock = threading.RLock()
        self.stats = {"steps": 0, "prefill_tokens": 0, "decode_tokens": 0, "finished": 0, "preempted": 0}
        # prompt-lookup speculative decoding inside continuous batching (0 = off)
        self.spec_num_draft = spec_num_draft
        self.spec_ngram = spec_ngram
        from .speculative import SpecStats
        self.spec_stats = SpecStats()
        # per-request incremental n-gram indexes (native), and an optional override that
        # supplies each request's draft (e.g. a known continuation: forced acceptance)
        self._ngram: Dict[object, object] = {}
        self.draft_provider: Optional[Callable[[Request], List[int]]] = None
        # benchmarks only: keep every greedy draft whatever the target predicts, so the
        # verify cost can be timed at a chosen acceptance (outputs are then not the target's)
        self.spec_force_accept = False
        # overlapped decode: step n+1 is launched (fed from the device) before step n's
        # tokens are read back, so host scheduling hides behind the GPU's work
        self.lookahead = lookahead and ep_sync is None and os.environ.get("VRM_LOOKAHEAD", "1") != "0"
        self._pending = None          # (requests, PendingDecode) of the step in flight

    # ------------------------------------------------------------------ API
    def add_request(self, prompt_ids: Sequence[int], params: Optional[SamplingParams] = None, *,
                    request_id=None, on_token=None) -> Request:
        params = params or SamplingParams()
        if len(prompt_ids) == 0:
            raise ValueError("empty prompt")
        if len(prompt_ids) + 1 > self.max_model_len:
            raise ValueError(f"prompt of {len(prompt_ids)} tokens exceeds max_model_len {self.max_model_len}")
        req = Request(list(int(t) for t in prompt_ids), params, on_token=on_token)
        if request_id is not None:
            req.request_id = request_id
        req.future = Future()
        with self._lock:
            self.waiting.append(req)
        return req

    def recover(self, max_retries: int = 2) -> List[Request]:
        """After a failed step: the running requests give their KV pages back and wait
        again at the front of the queue; on re-admission they prefill their prompt and
        the tokens they already have, then continue (request-level resume).  A request
        that already failed `max_retries` times is returned instead (out of the running
        set, pages freed, not yet finished: the caller reports the error and finishes it
        with reason "error")."""
        with self._lock:
            self._pending = None               # the in-flight step's tokens are lost
            failed: List[Request] = []
            back: List[Request] = []
            for r in list(self.running):
                if r.finished:
                    continue
                self.running.remove(r)
                self.kv.free(r.request_id)
                r.retries += 1
                if r.retries > max_retries:
                    failed.append(r)
                    continue
                r.num_computed = 0
                r.cached_tokens = 0
                r.resumed = bool(r.output_ids)
                back.append(r)
            for r in reversed(back):
                self.waiting.appendleft(r)
            return failed

    def flush(self) -> List[Request]:
        """Reads the decode step still in flight (overlapped decode), emitting its
        tokens; returns the requests that finished."""
        with self._lock:
            done: List[Request] = []
            self._drain(done)
            return done

    def has_unfinished(self) -> bool:
        with self._lock:
            return bool(self.waiting or self.running)

    def abort(self, request_id) -> bool:
        with self._lock:
            for q in (self.waiting, self.running):
                for r in list(q):
                    if r.request_id == request_id:
                        self._finish(r, "abort")
                        return True
        return False

    def generate(self, prompts: Sequence[Sequence[int]], params: Optional[SamplingParams] = None) -> List[Request]:
        reqs = [self.add_request(p, params) for p in prompts]
        if self.ep_sync is not None:
            # every expert-parallel rank keeps stepping until all ranks are done
            while self.ep_sync.any_rank(any(not r.finished for r in reqs)):
                self.step()
            return reqs
        while any(not r.finished for r in reqs):
            self.step()
        return reqs

    # ------------------------------------------------------------------ scheduling
    def _admit(self) -> None:
        while self.waiting and len(self.running) < self.max_batch:
            req = self.waiting[0]
            ids = req.prefill_ids
            need = len(ids) + 1
            if req.resumed:
                # a preempted sequence comes back only with a page of headroom for every
                # running one, or it would be preempted again at the next page boundary
                need += self.kv.page_size * len(self.running)
            if not self.kv.can_allocate(need):
                break
            try:
                cached = self.kv.allocate(req.request_id, len(ids), ids)
            except OutOfPages:
                break
            self.waiting.popleft()
            req.num_computed = cached
            req.cached_tokens = cached
            self.running.append(req)

    def _draft(self, r: Request) -> List[int]:
        """Prompt-lookup draft of a running request (native n-gram index, extended by the
        tokens generated since its last draft; the Python scan without the runtime)."""
        if self.draft_provider is not None:
            return list(self.draft_provider(r))[:self.spec_num_draft]
        from .speculative import find_draft, ngram_index
        ix = self._ngram.get(r.request_id)
        if ix is None:
            ix = ngram_index(self.spec_ngram)
            if ix is None:
                return find_draft(r.prompt_ids + r.output_ids, self.spec_ngram, self.spec_num_draft)
            ix.extend(list(r.prompt_ids))
            self._ngram[r.request_id] = ix
        have = len(ix) - len(r.prompt_ids)
        if have < len(r.output_ids):
            ix.extend(list(r.output_ids[have:]))
        return ix.draft(self.spec_num_draft)

    def _finish(self, req: Request, reason: str) -> None:
        if req.finished:
            return
        req.finished = True
        req.finish_reason = reason
        req.finish_time = time.perf_counter()
        if req in self.running:
            self.running.remove(req)
        elif req in self.waiting:
            self.waiting.remove(req)
        self.kv.free(req.request_id)
        self._ngram.pop(req.request_id, None)
        self.stats["finished"] += 1
        if req.future is not None and not req.future.done():
            req.future.set_result(req)

    def _emit(self, req: Request, tok: int) -> None:
        req.output_ids.append(tok)
        if req.first_token_time is None:
            req.first_token_time = time.perf_counter()
        if req.on_token is not None:
            req.on_token(req, tok)
        p = req.params
        stop = set(p.stop_token_ids)
        if self.eos_token_id is not None and not p.ignore_eos:
            stop.add(self.eos_token_id)
        if tok in stop:
            self._finish(req, "stop")
        elif len(req.output_ids) >= p.max_tokens:
            self._finish(req, "length")
        elif req.total_len >= self.max_model_len:
            self._finish(req, "length")

    def step(self) -> List[Request]:
        """One scheduler iteration; returns requests that finished during it."""
        with self._lock:
            before = self.stats["finished"]
            done: List[Request] = []
            pool = getattr(self.runner, "pool", None)
            if getattr(pool, "reclaim_requested", False):
                # a lender wants its memory back: borrowed KV pages move home between
                # steps, after the step in flight has been read
                self._drain(done)
                pool.reclaim(self.kv)
            self._admit()
            if self.ep_sync is None:
                self._prefill_chunk(done)
                self._decode(done)
            else:
                # the ranks' MoE layer calls must pair up: forward passes run on every
                # rank when they run on any (one-token dummies where there is no work)
                mine = any(not r.prefill_done for r in self.running)
                if self.ep_sync.any_rank(mine):
                    if mine:
                        self._prefill_chunk(done)
                    else:
                        self.ep_sync.dummy_prefill(self.runner)
                mine = any(r.prefill_done and not r.finished and r.output_ids for r in self.running)
                if self.ep_sync.any_rank(mine):
                    if mine:
                        self._decode(done)
                    else:
                        self.ep_sync.dummy_decode(self.runner)
            self.stats["steps"] += 1
            return done

    def _prefill_chunk(self, done: List[Request]) -> None:
        budget = self.max_prefill_tokens
        items, reqs = [], []
        for req in self.running:
            if req.prefill_done or budget <= 0:
                continue
            ids = req.prefill_ids
            n = min(len(ids) - req.num_computed, budget)
            s = req.num_computed
            slots = self.kv.slots_for(req.request_id, s, n)
            items.append(PrefillItem(token_ids=ids[s:s + n], start_pos=s, slots=slots,
                                     block_table=self.kv.block_table(req.request_id), context_len=s + n,
                                     want_logits=(s + n == len(ids))))
            reqs.append(req)
            budget -= n
        if not items:
            return
        toks = self.runner.prefill(items, [r.params.temperature for r in reqs], [r.params.top_k for r in reqs],
                                   [r.params.top_p for r in reqs], [0 for _ in reqs])
        for req, it, tok in zip(reqs, items, toks):
            req.num_computed += len(it.token_ids)
            self.stats["prefill_tokens"] += len(it.token_ids)
            if req.prefill_done:
                self.kv.commit_prefix(req.request_id, req.prefill_ids)
                if req.resumed:
                    # KV rebuilt up to the last generated token: decoding resumes from it
                    req.resumed = False
                    continue
                self._emit(req, int(tok))
                if req.finished:
                    done.append(req)

    def _decode(self, done: List[Request]) -> None:
        active = [r for r in self.running if r.prefill_done and not r.finished and r.output_ids]
        if self.spec_num_draft > 0 and active:
            from .speculative import speculative_decode_step
            drafts = [self._draft(r) for r in active]
            if any(drafts):
                self._drain(done)
                active = [r for r in active if not r.finished]
                drafts = [self._draft(r) for r in active]
                if not self._pages_for_verify(active, drafts):
                    drafts = []          # not enough KV pages: plain decode (with preemption)
            if drafts and any(drafts):
                outs = speculative_decode_step(self, active, self.spec_ngram, self.spec_num_draft, self.spec_stats,
                                               drafts=drafts)
                for r, toks in zip(active, outs):
                    for t in toks:
                        self.stats["decode_tokens"] += 1
                        self._emit(r, int(t))
                        if r.finished:
                            done.append(r)
                            break
                return
            # nothing to draft: an ordinary (graph-replayed) decode step
            active = [r for r in active if not r.finished]
        pend = self._pending
        if pend is not None and active and self._can_chain(pend[0], active):
            # launch step n+1 on the device-resident tokens of step n, then read step n
            nxt = self._launch(active, chained=True)
            self._pending = None
            self._consume(pend[0], pend[1], done)
            self._pending = (active, nxt)
            return
        self._drain(done)
        active = [r for r in active if not r.finished]
        active = self._ensure_pages(active, done)
        if not active:
            return
        handle = self._launch(active, chained=False)
        if self.lookahead:
            self._pending = (active, handle)
        else:
            self._consume(active, handle, done)

    def _pages_for_verify(self, active: List[Request], drafts) -> bool:
        """Whether the pool has the pages a verify step (last token + drafts per
        sequence) needs; the lending pool, when present, supplies overflow pages."""
        if getattr(self.kv, "_overflow", None) is not None:
            return True
        ps = self.kv.page_size
        need = 0
        for r, d in zip(active, drafts):
            n0 = self.kv.seq_len(r.request_id)
            need += -(-(n0 + 1 + len(d)) // ps) - (-(-n0 // ps))
        return need <= self.kv.num_free_pages()

    def _ensure_pages(self, active: List[Request], done: List[Request]) -> List[Request]:
        """Recompute preemption: when the pool cannot give every sequence of this decode
        step the page its next token starts, the most recently admitted sequences give
        their pages back and wait again; on re-admission they prefill prompt + generated
        tokens (the prefix cache keeps what it still holds) and continue where they
        stopped.  A lone sequence that outgrows the whole pool ends with reason "length"."""
        if getattr(self.kv, "_overflow", None) is not None:
            return active              # the lending pool supplies overflow pages
        ps = self.kv.page_size
        while active:
            need = sum(1 for r in active if self.kv.seq_len(r.request_id) % ps == 0)
            if need <= self.kv.num_free_pages():
                return active
            victim = active[-1]
            if len(active) == 1:
                self._finish(victim, "length")
                done.append(victim)
                return []
            active = active[:-1]
            self.kv.free(victim.request_id)
            if victim in self.running:
                self.running.remove(victim)
            victim.num_computed = 0
            victim.cached_tokens = 0
            victim.resumed = True
            self.waiting.appendleft(victim)
            self.stats["preempted"] += 1
        return active

    def _can_chain(self, prev: List[Request], active: List[Request]) -> bool:
        """Step n+1 may run before step n is read when the batch is the same requests
        in the same rows, none of them ends by length with step n's token, and the KV
        pool has a page for every sequence that starts one."""
        if not self.lookahead or len(prev) != len(active) or any(a is not b for a, b in zip(prev, active)):
            return False
        ps = self.kv.page_size
        new_pages = 0
        for r in active:
            if r.finished or len(r.output_ids) + 1 >= r.params.max_tokens or r.total_len + 1 >= self.max_model_len:
                return False
            if self.kv.seq_len(r.request_id) % ps == 0:
                new_pages += 1
        return new_pages <= self.kv.num_free_pages()

    def _launch(self, active: List[Request], chained: bool):
        """Appends one KV slot per request and launches the decode step.  Chained: the
        token fed is the one step n sampled (still on the device), one position later."""
        off = 1 if chained else 0
        ids, pos, slots, ctx, bts = [], [], [], [], []
        temp, topk, topp, steps = [], [], [], []
        for r in active:
            p = r.total_len - 1 + off               # position of the token being fed
            s = self.kv.append_slots(r.request_id, 1)[0]
            ids.append(0 if chained else r.output_ids[-1])
            pos.append(p)
            slots.append(s)
            ctx.append(p + 1)
            bts.append(self.kv.block_table(r.request_id))
            temp.append(r.params.temperature)
            topk.append(r.params.top_k)
            topp.append(r.params.top_p)
            steps.append(len(r.output_ids) + off)
        self._apply_cow()
        return self.runner.launch_decode(ids, pos, slots, ctx, bts, temp, topk, topp, steps, ids_on_device=chained)

    def _consume(self, reqs: List[Request], handle, done: List[Request]) -> None:
        """Reads a launched step's tokens and emits them (requests that finished or were
        aborted meanwhile drop theirs)."""
        toks = self.runner.collect_decode(handle)
        for r, tok in zip(reqs, toks):
            if r.finished:
                continue
            self.stats["decode_tokens"] += 1
            self._emit(r, int(tok))
            if r.finished:
                done.append(r)

    def _drain(self, done: List[Request]) -> None:
        """Reads the step still in flight, if any."""
        pend, self._pending = self._pending, None
        if pend is not None:
            self._consume(pend[0], pend[1], done)

    def _apply_cow(self) -> None:
        copies = self.kv.pop_cow_copies()
        if copies:
            self.runner.copy_pages(copies)


class EPSync:
    """Lockstep of expert-parallel ranks (each runs its own engine on its own
    sequences): a host-side OR over the ranks before every forward pass, and one-token
    dummy passes into a reserved KV page for a rank without work, so that every rank
    makes the same sequence of MoE layer calls.

    Reference parity: none (the reference has no expert parallelism)."""

    DUMMY = "__ep_dummy__"

    def __init__(self, manager: PagedKVCacheManager, group=None):
        import torch.distributed as dist
        self.dist = dist
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        manager.allocate(self.DUMMY, 1)
        self.slot = manager.slots_for(self.DUMMY, 0, 1)[0]
        self.block_table = manager.block_table(self.DUMMY)

    def any_rank(self, flag: bool) -> bool:
        if self.world == 1:
            return bool(flag)
        t = torch.tensor([1 if flag else 0], dtype=torch.int32)
        self.dist.all_reduce(t, op=self.dist.ReduceOp.MAX, group=self.group)
        return bool(t.item())

    def dummy_prefill(self, runner) -> None:
        from .runner import PrefillItem
        runner.prefill([PrefillItem(token_ids=[0], start_pos=0, slots=[self.slot], block_table=self.block_table,
                                    context_len=1, want_logits=False)], [0.0], [0], [1.0], [0])

    def dummy_decode(self, runner) -> None:
        runner.decode_step([0], [0], [self.slot], [1], [self.block_table], [0.0], [0], [1.0], [0])
