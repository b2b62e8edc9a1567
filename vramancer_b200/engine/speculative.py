"""Speculative decoding: prompt lookup (n-gram drafts) and draft-model proposals,
verified by one forward of the target over all proposals.

Verification is a chunked-prefill forward over the paged cache: every sequence
feeds [last token, d_1 .. d_k] at its next positions, the kernels attend over the
cached prefix plus the new rows, and greedy predictions p_0..p_k come back for all
rows at once (batched across sequences).  Drafts are accepted while d_i == p_{i-1};
the first mismatch contributes p_j as a bonus token; KV of rejected positions is
truncated from the block table (their slots are simply rewritten later).  Greedy
output is identical to plain decoding.

Reference parity: prompt lookup = HF `prompt_lookup_num_tokens`
(core/backends.py:1920-1925, vramancer/dropin.py wrap-generate); draft model =
core/speculative_decoding.py:95-329 (gamma-adaptive, window 10), whose stochastic
acceptance (`q > 0.5`, :268-281) is not rejection sampling and is not reproduced.
Sampled requests use speculative sampling (Leviathan et al. 2023; Chen et al. 2023)
with a deterministic draft (q = a point mass on each drafted token): draft d_i is kept
with probability p_i(d_i), where p_i is the target's filtered distribution
(temperature, top-k, top-p) at that position; at the first rejection the token comes
from p_i with d_i removed and renormalised, and when every draft is kept a bonus token
comes from p_k.  The emitted tokens are distributed exactly as plain sampling from
the target.  A draft model that samples its proposals from q uses the general rule:
keep d_i with probability min(1, p_i(d_i) / q_i(d_i)), else draw from
norm(max(0, p_i - q_i)).
"""
from __future__ import annotations

import zlib
from typing import List, Optional, Sequence, Tuple

import torch

from .. import ops
from .runner import PrefillItem


def find_draft(seq: Sequence[int], max_ngram: int = 3, num_draft: int = 8, min_ngram: int = 1) -> List[int]:
    """Continuation of the most recent earlier occurrence of the sequence's last n-gram
    (n from max_ngram down to min_ngram)."""
    L = len(seq)
    for n in range(min(max_ngram, L - 1), min_ngram - 1, -1):
        tail = list(seq[L - n:])
        # scan backwards for the latest match that has a continuation
        for s in range(L - n - 1, -1, -1):
            if list(seq[s:s + n]) == tail:
                cont = list(seq[s + n:s + n + num_draft])
                if cont:
                    return cont
    return []


def ngram_index(max_ngram: int = 3, min_ngram: int = 1):
    """A native incremental index with `find_draft`'s rule (extend(tokens), draft(k),
    len), or None when the host runtime is not built."""
    try:
        from .. import _runtime
    except ImportError:
        return None
    return _runtime.NgramIndex(max_ngram, min_ngram)


def accept_greedy(draft: Sequence[int], preds: Sequence[int]) -> Tuple[List[int], int]:
    """(accepted drafts + bonus token, number of accepted drafts)."""
    acc = []
    for i, d in enumerate(draft):
        if int(preds[i]) == int(d):
            acc.append(int(d))
        else:
            break
    return acc + [int(preds[len(acc)])], len(acc)


def filtered_probs(logits: torch.Tensor, temperature: float, top_k: int, top_p: float) -> torch.Tensor:
    """Sampling distribution of logits rows [n, V] under temperature / top-k / top-p
    (top-k first, then the smallest top-p nucleus of what is left), fp32."""
    z = logits.float() / max(float(temperature), 1e-6)
    V = z.shape[-1]
    if 0 < top_k < V:
        thr = torch.topk(z, top_k, dim=-1).values[..., -1:]
        z = z.masked_fill(z < thr, float("-inf"))
    p = torch.softmax(z, dim=-1)
    if top_p < 1.0:
        sp, si = torch.sort(p, dim=-1, descending=True)
        keep = (torch.cumsum(sp, dim=-1) - sp) < top_p
        mask = torch.zeros_like(keep).scatter(-1, si, keep)
        p = torch.where(mask, p, torch.zeros_like(p))
        p = p / p.sum(-1, keepdim=True)
    return p


def accept_sampled(draft: Sequence[int], probs: torch.Tensor, gen: torch.Generator) -> Tuple[List[int], int]:
    """Speculative sampling with a deterministic draft: probs [len(draft) + 1, V] are the
    target's distributions at the draft positions and after the last draft.  Returns
    (kept drafts + one sampled token, number of kept drafts)."""
    probs = probs.float().cpu()
    out: List[int] = []
    for i, d in enumerate(draft):
        pi = probs[i]
        u = float(torch.rand((), generator=gen))
        if u < float(pi[int(d)]):
            out.append(int(d))
            continue
        residual = pi.clone()
        residual[int(d)] = 0.0
        tot = float(residual.sum())
        if tot <= 0.0:          # p_i was a point mass on d: unreachable after a rejection
            out.append(int(d))
            continue
        out.append(int(torch.multinomial(residual / tot, 1, generator=gen)))
        return out, i
    out.append(int(torch.multinomial(probs[len(draft)], 1, generator=gen)))
    return out, len(draft)


def accept_with_draft_probs(draft: Sequence[int], probs: torch.Tensor, qprobs: torch.Tensor,
                            gen: torch.Generator) -> Tuple[List[int], int]:
    """Speculative sampling with a sampled draft: d_i was drawn from q_i (qprobs row i);
    keep it with probability min(1, p_i(d_i) / q_i(d_i)), else draw from
    norm(max(0, p_i - q_i)) and stop; after every draft is kept, draw from p_k."""
    probs = probs.float().cpu()
    qprobs = qprobs.float().cpu()
    V = probs.shape[-1]
    if qprobs.shape[-1] != V:
        # draft and target vocabularies differ in padding: the draft's mass on ids the
        # target does not have is dropped (such ids are never proposed) and q renormalised
        q2 = torch.zeros(qprobs.shape[0], V)
        n = min(V, qprobs.shape[-1])
        q2[:, :n] = qprobs[:, :n]
        qprobs = q2 / q2.sum(-1, keepdim=True).clamp_min(1e-30)
    out: List[int] = []
    for i, d in enumerate(draft):
        if int(d) >= V:
            out.append(int(torch.multinomial(probs[i], 1, generator=gen)))
            return out, i
        p, q = probs[i], qprobs[i]
        d = int(d)
        u = float(torch.rand((), generator=gen))
        if float(q[d]) > 0.0 and u < min(1.0, float(p[d]) / float(q[d])):
            out.append(d)
            continue
        residual = torch.clamp(p - q, min=0.0)
        tot = float(residual.sum())
        out.append(int(torch.multinomial(residual / tot if tot > 0 else p, 1, generator=gen)))
        return out, i
    out.append(int(torch.multinomial(probs[len(draft)], 1, generator=gen)))
    return out, len(draft)


class SpecStats:
    def __init__(self):
        self.proposed = 0
        self.accepted = 0
        self.steps = 0

    @property
    def acceptance(self) -> float:
        return self.accepted / self.proposed if self.proposed else 0.0

    def to_dict(self):
        return {"proposed": self.proposed, "accepted": self.accepted, "steps": self.steps,
                "acceptance": round(self.acceptance, 4)}


def speculative_decode_step(engine, active, ngram: int, num_draft: int, stats: SpecStats,
                            drafts: Optional[List[List[int]]] = None,
                            draft_probs: Optional[List[Optional[torch.Tensor]]] = None):
    """One verify step for `active` requests of an LLMEngine.  `draft_probs[i]`, when
    given, holds the draft model's distributions [len(draft), V] the drafts of a sampled
    request were drawn from (else the draft counts as deterministic)."""
    kv, runner = engine.kv, engine.runner
    items, feeds, starts, ds = [], [], [], []
    for i, r in enumerate(active):
        seq = r.prompt_ids + r.output_ids
        room = min(r.params.max_tokens - len(r.output_ids) - 1, engine.max_model_len - len(seq) - 1)
        if drafts is not None:
            d = list(drafts[i])
        elif num_draft > 0:
            d = find_draft(seq, ngram, num_draft)
        else:
            d = []
        d = d[:max(0, room)]
        feed = [seq[-1]] + d
        start = len(seq) - 1
        slots = kv.append_slots(r.request_id, len(feed))
        items.append(PrefillItem(feed, start, slots, kv.block_table(r.request_id), start + len(feed), True))
        feeds.append(feed)
        starts.append(start)
        ds.append(d)
    engine._apply_cow()
    if all(r.params.greedy for r in active) and getattr(runner, "verify_greedy", None) is not None:
        # greedy batch: the verify forward + argmax replay as one CUDA graph
        vg = runner.verify_greedy(items)
        if vg is not None:
            return _accept_all_greedy(engine, active, feeds, starts, ds, [t for row in vg for t in row], stats)
    logits = runner.prefill_logits(items)
    if logits.is_cuda:
        preds = ops.argmax(logits).cpu().tolist()
    else:
        preds = torch.argmax(logits.float(), -1).tolist()
    # non-greedy requests without a draft draw their token with their own temperature /
    # top-k / top-p from the logits of that position (the sampling kernel)
    rows, samp = [], []
    off = 0
    for r, feed in zip(active, feeds):
        if not r.params.greedy and len(feed) == 1:
            rows.append(off)
            samp.append(r)
        off += len(feed)
    if samp:
        dev = logits.device
        sel = logits[torch.tensor(rows, device=dev)].contiguous()
        f32 = lambda v: torch.tensor(v, dtype=torch.float32, device=dev)   # noqa: E731
        i32 = lambda v: torch.tensor(v, dtype=torch.int32, device=dev)     # noqa: E731
        drawn = ops.sample(sel, f32([r.params.temperature for r in samp]), i32([r.params.top_k for r in samp]),
                           f32([r.params.top_p for r in samp]), runner.seed,
                           i32([len(r.output_ids) for r in samp])).cpu().tolist()
        for row, tok in zip(rows, drawn):
            preds[row] = int(tok)
    out = []
    off = 0
    stats.steps += 1
    for r, feed, start, d in zip(active, feeds, starts, ds):
        p = preds[off:off + len(feed)]
        off += len(feed)
        if r.params.greedy:
            toks, na = ((list(d) + [int(p[len(d)])], len(d)) if getattr(engine, "spec_force_accept", False)
                        else accept_greedy(d, p))
        elif not d:
            toks, na = [int(p[0])], 0
        else:
            pr = filtered_probs(logits[off - len(feed):off], r.params.temperature, r.params.top_k, r.params.top_p)
            # seeded from (runner seed, request, position): the same on every rank
            gen = torch.Generator().manual_seed((runner.seed * 1000003 + zlib.crc32(str(r.request_id).encode()) * 7919
                                                 + len(r.output_ids)) & 0x7FFFFFFFFFFFFFFF)
            q = draft_probs[len(out)] if draft_probs is not None else None
            toks, na = accept_sampled(d, pr, gen) if q is None else accept_with_draft_probs(d, pr, q, gen)
        stats.proposed += len(d)
        stats.accepted += na
        kv.truncate(r.request_id, start + 1 + na)
        out.append(toks)
    return out


def _accept_all_greedy(engine, active, feeds, starts, ds, preds, stats):
    out = []
    off = 0
    stats.steps += 1
    force = getattr(engine, "spec_force_accept", False)
    for r, feed, start, d in zip(active, feeds, starts, ds):
        p = preds[off:off + len(feed)]
        off += len(feed)
        # forced acceptance (benchmarks of the verify cost): every draft is kept
        toks, na = (list(d) + [int(p[len(d)])], len(d)) if force else accept_greedy(d, p)
        stats.proposed += len(d)
        stats.accepted += na
        engine.kv.truncate(r.request_id, start + 1 + na)
        out.append(toks)
    return out


class PromptLookupDecoder:
    """Single-sequence greedy generation with prompt-lookup drafts through an LLM."""

    def __init__(self, llm, num_draft: int = 8, ngram: int = 3):
        self.llm = llm
        self.num_draft = num_draft
        self.ngram = ngram
        self.stats = SpecStats()

    def generate(self, prompt_ids: Sequence[int], max_new_tokens: int) -> List[int]:
        eng = self.llm.engine
        from .engine import SamplingParams
        with eng._lock:
            req = eng.add_request(prompt_ids, SamplingParams(max_tokens=max_new_tokens))
            eng.waiting.remove(req)
            eng.kv.allocate(req.request_id, len(req.prompt_ids))
            eng.running.append(req)
            try:
                # prefill (+ first token)
                toks = eng.runner.prefill([PrefillItem(req.prompt_ids, 0, eng.kv.slots_for(req.request_id, 0,
                                                                                          len(req.prompt_ids)),
                                                       eng.kv.block_table(req.request_id), len(req.prompt_ids),
                                                       True)], [0.0], [0], [1.0], [0])
                req.num_computed = len(req.prompt_ids)
                eng._emit(req, int(toks[0]))
                while not req.finished:
                    new = speculative_decode_step(eng, [req], self.ngram, self.num_draft, self.stats)[0]
                    for t in new:
                        eng._emit(req, t)
                        if req.finished:
                            break
            finally:
                if not req.finished:
                    eng._finish(req, "abort")
        return list(req.output_ids)


def _full_logits(llm, seq: Sequence[int]) -> torch.Tensor:
    """Last-position logits of `seq` under `llm` (a prefill into a scratch sequence)."""
    eng = llm.engine
    rid = f"draft-{id(seq)}-{len(seq)}"
    with eng._lock:
        eng.kv.allocate(rid, len(seq))
        try:
            it = PrefillItem(list(seq), 0, eng.kv.slots_for(rid, 0, len(seq)), eng.kv.block_table(rid), len(seq), True)
            return llm.runner.prefill_logits([it])[-1:].float()
        finally:
            eng.kv.free(rid)


# default small draft model per target-model family, by name prefix (the reference's
# choices; a draft must share the target's tokenizer)
DRAFT_MODEL_MAP = (
    ("Qwen/Qwen2.5-", "Qwen/Qwen2.5-0.5B-Instruct"),
    ("qwen2.5-", "qwen2.5-0.5b"),
    ("Qwen/Qwen2-", "Qwen/Qwen2-0.5B-Instruct"),
    ("meta-llama/Llama-3", "meta-llama/Llama-3.2-1B"),
    ("llama-3", "llama-3.2-1b"),
    ("meta-llama/Llama-2", "TinyLlama/TinyLlama-1.1B-Chat-v1.0"),
    ("mistralai/", "TinyLlama/TinyLlama-1.1B-Chat-v1.0"),
    ("gpt2", "distilgpt2"),
    ("openai-community/gpt2", "distilgpt2"),
)


def guess_draft_model(main_model_name: str) -> Optional[str]:
    """The default draft model for a target model name (None when no family matches,
    and never the target itself: a draft as large as the target saves nothing)."""
    name = str(main_model_name or "")
    base = name.rstrip("/").rsplit("/", 1)[-1]
    for prefix, draft in DRAFT_MODEL_MAP:
        if name.startswith(prefix) or base.startswith(prefix):
            if draft.lower() not in (name.lower(), base.lower()):
                return draft
    return None


class DraftModelDecoder:
    """Draft-model speculation: a small model proposes gamma tokens greedily, the
    target verifies them in one forward; gamma adapts to the running acceptance
    (window of recent rounds) between gamma_min and gamma_max."""

    def __init__(self, target, draft, gamma: int = 5, adaptive: bool = True, gamma_min: int = 2, gamma_max: int = 12,
                 window: int = 10):
        self.target, self.draft = target, draft
        self.gamma = gamma
        self.adaptive = adaptive
        self.gmin, self.gmax, self.window = gamma_min, gamma_max, window
        self.recent: List[float] = []
        self.stats = SpecStats()

    @property
    def target_vocab(self) -> int:
        return self.target.cfg.vocab_size

    def _draft_can_read(self, seq: Sequence[int]) -> bool:
        """A draft with a smaller vocabulary cannot embed ids beyond it: no draft then."""
        return not seq or max(seq) < self.draft.cfg.vocab_size

    def _propose(self, seq: List[int], k: int) -> List[int]:
        from .engine import SamplingParams
        if not self._draft_can_read(seq):
            return []
        r = self.draft.engine.generate([seq], SamplingParams(max_tokens=k))[0]
        out = []
        for t in r.output_ids:      # an id the target's vocabulary lacks ends the draft
            if t >= self.target_vocab:
                break
            out.append(t)
        return out

    def _propose_sampled(self, seq: List[int], k: int, params, gen: torch.Generator):
        """k draft tokens drawn from the draft model's filtered distributions (same
        temperature / top-k / top-p as the request), over the target's vocabulary (draft
        logits of ids the target lacks are masked, missing ids get none); returns
        (tokens, q rows [k, V_target])."""
        toks: List[int] = []
        rows = []
        cur = list(seq)
        V = self.target_vocab
        if not self._draft_can_read(cur):
            return toks, None
        for _ in range(k):
            if len(cur) + 1 > self.draft.engine.max_model_len:
                break
            logits = _full_logits(self.draft, cur)
            if logits.shape[-1] > V:
                logits = logits[..., :V]
            elif logits.shape[-1] < V:
                pad = torch.full((*logits.shape[:-1], V - logits.shape[-1]), float("-inf"), dtype=logits.dtype,
                                 device=logits.device)
                logits = torch.cat([logits, pad], dim=-1)
            q = filtered_probs(logits, params.temperature, params.top_k, params.top_p)[0]
            t = int(torch.multinomial(q.cpu(), 1, generator=gen))
            toks.append(t)
            rows.append(q.cpu())
            cur.append(t)
        return toks, (torch.stack(rows) if rows else None)

    def generate(self, prompt_ids: Sequence[int], max_new_tokens: int, params=None, seed: int = 0) -> List[int]:
        """Greedy by default; with sampling `params` (temperature > 0) the draft samples
        its proposals and the target accepts them by rejection sampling, so the output
        follows the target's distribution exactly."""
        eng = self.target.engine
        from .engine import SamplingParams
        sp = params if params is not None else SamplingParams(max_tokens=max_new_tokens)
        sp = SamplingParams(max_tokens=max_new_tokens, temperature=sp.temperature, top_k=sp.top_k, top_p=sp.top_p,
                            stop_token_ids=sp.stop_token_ids, ignore_eos=sp.ignore_eos)
        gen = torch.Generator().manual_seed(seed)
        with eng._lock:
            req = eng.add_request(prompt_ids, sp)
            eng.waiting.remove(req)
            eng.kv.allocate(req.request_id, len(req.prompt_ids))
            eng.running.append(req)
            toks = eng.runner.prefill([PrefillItem(req.prompt_ids, 0, eng.kv.slots_for(req.request_id, 0,
                                                                                      len(req.prompt_ids)),
                                                   eng.kv.block_table(req.request_id), len(req.prompt_ids), True)],
                                      [sp.temperature], [sp.top_k], [sp.top_p], [0])
            req.num_computed = len(req.prompt_ids)
            eng._emit(req, int(toks[0]))
            while not req.finished:
                seq = req.prompt_ids + req.output_ids
                if sp.greedy:
                    d, q = self._propose(seq, self.gamma), None
                else:
                    d, q = self._propose_sampled(seq, self.gamma, sp, gen)
                new = speculative_decode_step(eng, [req], 0, 0, self.stats, drafts=[d],
                                              draft_probs=None if q is None else [q])[0]
                if d:
                    self.recent = (self.recent + [(len(new) - 1) / len(d)])[-self.window:]
                if self.adaptive and len(self.recent) >= 3:
                    rate = sum(self.recent) / len(self.recent)
                    self.gamma = min(self.gmax, self.gamma + 1) if rate > 0.8 else (
                        max(self.gmin, self.gamma - 1) if rate < 0.4 else self.gamma)
                for t in new:
                    eng._emit(req, t)
                    if req.finished:
                        break
        return list(req.output_ids)
