"""InferencePipeline: the conductor behind the CLI and the HTTP API.

    pipe = InferencePipeline().load("qwen2.5-14b", num_gpus=1)
    text = pipe.generate("Hello", max_new_tokens=32)
    fut = pipe.submit("Hi", max_new_tokens=8)          # concurrent requests
    for delta in pipe.generate_stream("Tell me", max_new_tokens=64): ...

`load` builds one of:
  * single device (GPU, or CPU reference ops when no GPU is present),
  * an in-process pipeline over `num_gpus` GPUs (layer ranges from the splitter),
  * a tensor-parallel rank when the process runs under torchrun (WORLD_SIZE > 1;
    rank 0 drives, the other ranks follow the same scheduling in lockstep).
A background thread runs the continuous-batching engine; `submit` returns a Future,
`generate` waits on it, `generate_stream` yields text as tokens arrive.  OOM during
generation goes through the auto-heal ladder; faults are classified and counted by
the GPU fault manager; every request is recorded in metrics and the request history.

Reference parity: core/inference_pipeline.py:89-1944 (load 163-439, generate 501-689,
infer 691-740, submit 1749-1777, shutdown 1826-1906, get_pipeline/reset_pipeline).
"""
from __future__ import annotations

import os
import queue
import threading
import time
from concurrent.futures import Future
from typing import Any, Dict, Iterator, List, Optional, Sequence, Union

import torch

from .engine.engine import LLMEngine, Request, SamplingParams
from .engine.runner import PrefillItem
from .llm import LLM
from .models.config import get_config
from .serving.tokenizer import load_tokenizer
from .utils.fault import GPUFaultManager, OOMAutoHeal
from .utils.observability import METRICS, RequestHistory, get_logger, span

log = get_logger("vramancer.pipeline")


def stop_index(text: str, stop: Optional[Sequence[str]]) -> int:
    """Index of the earliest occurrence of any stop string in text, or -1."""
    best = -1
    for st in stop or ():
        i = text.find(st)
        if i >= 0 and (best < 0 or i < best):
            best = i
    return best


class InferencePipeline:
    def __init__(self, backend_name: str = "auto", enable_metrics: bool = True, enable_discovery: bool = False,
                 verbose: bool = False):
        self.backend_name = backend_name
        self.enable_metrics = enable_metrics
        self.verbose = verbose
        self.llm: Optional[LLM] = None
        self.engine: Optional[LLMEngine] = None
        self.tokenizer = None
        self.model_name: Optional[str] = None
        self.num_gpus = 0
        self.mode = "none"
        self.history = RequestHistory()
        self.autoheal = OOMAutoHeal()
        self.fault = None
        self._thread: Optional[threading.Thread] = None
        self._stop = threading.Event()
        self._wake = threading.Condition()
        self.loaded_at: Optional[float] = None
        self.lora = None
        self.spec = None
        self._draft = None            # draft-model decoder for enable_speculative (False: none)
        self._bcast = None            # TP serving: rank 0 broadcasts request events
        self._events: List = []

    # ------------------------------------------------------------------ load
    def load(self, model_name: str, num_gpus: Optional[int] = None, *, max_batch: int = 64,
             max_model_len: int = 4096, kv_cache_dtype: str = "bf16", quantization: Optional[str] = None,
             device: Optional[str] = None, num_layers: Optional[int] = None, kv_pages: Optional[int] = None,
             use_cuda_graph: Optional[bool] = None, prompt_lookup: int = 0, **kw) -> "InferencePipeline":
        cfg = get_config(model_name)
        if num_layers:
            cfg = cfg.with_(num_layers=num_layers)
        self.model_name = model_name
        has_cuda = torch.cuda.is_available() and device != "cpu"
        ngpu = torch.cuda.device_count() if has_cuda else 0
        if num_gpus is None:
            num_gpus = self._auto_num_gpus(cfg, ngpu) if has_cuda else 0
        self.num_gpus = num_gpus
        world = int(os.environ.get("WORLD_SIZE", "1"))
        dtype = torch.bfloat16 if has_cuda else torch.float32
        kvd = kv_cache_dtype if has_cuda else "fp32"
        graph = has_cuda if use_cuda_graph is None else use_cuda_graph
        with span("pipeline.load", model=model_name, num_gpus=num_gpus):
            if world > 1 and has_cuda:
                from .parallel import comm
                info = comm.init_distributed()
                tp = comm.tp_context()
                self.llm = LLM(cfg, device=f"cuda:{info.local_rank}", kv_cache_dtype=kvd, max_batch=max_batch,
                               max_model_len=max_model_len, kv_pages=kv_pages, tp=tp, use_cuda_graph=graph,
                               quantization=quantization, **kw)
                self.mode = f"tp{world}"
                from .parallel.follower import StepBroadcaster
                self._bcast = StepBroadcaster()
            elif has_cuda and num_gpus > 1:
                self.llm = self._build_pp(cfg, num_gpus, max_batch, max_model_len, kv_pages, kvd, dtype, **kw)
                self.mode = f"pp{num_gpus}"
            else:
                dev = "cuda:0" if has_cuda else "cpu"
                self.llm = LLM(cfg, device=dev, dtype=dtype, kv_cache_dtype=kvd, max_batch=max_batch,
                               max_model_len=max_model_len, kv_pages=kv_pages or (None if has_cuda else 512),
                               use_cuda_graph=graph, quantization=quantization, **kw)
                self.mode = "single-gpu" if has_cuda else "cpu"
        self.engine = self.llm.engine
        self.tokenizer = load_tokenizer(model_name if os.path.isdir(str(model_name)) else None, cfg.vocab_size)
        if getattr(self.tokenizer, "eos_token_id", None) is not None:
            self.engine.eos_token_id = self.tokenizer.eos_token_id
        if prompt_lookup:
            from .engine.speculative import PromptLookupDecoder
            self.spec = PromptLookupDecoder(self.llm, num_draft=prompt_lookup)
        self.fault = GPUFaultManager(list(range(max(ngpu, 0))))
        from .serving.lora import LoRAManager
        self.lora = LoRAManager(self.llm)
        self.loaded_at = time.time()
        self.start()
        log.info("loaded %s (%s, %d layers) in mode %s", model_name, cfg.arch, cfg.num_layers, self.mode)
        return self

    def _auto_num_gpus(self, cfg, ngpu: int) -> int:
        need = cfg.num_params() * 2 * 1.25
        free = torch.cuda.mem_get_info(0)[0] if ngpu else 0
        return 1 if need <= 0.9 * free else ngpu

    def _build_pp(self, cfg, n, max_batch, max_model_len, kv_pages, kvd, dtype, **kw) -> LLM:
        from .kv.pool import kv_dtype_from_str
        from .parallel.placement import detect_gpus, split_model_into_blocks
        devs = [f"cuda:{i}" for i in range(n)]
        blocks = split_model_into_blocks(cfg, devs, gpus=detect_gpus()[:n])
        pages = kv_pages or max_batch * ((max_model_len + 15) // 16) + 16
        return LLM.from_local_pipeline(cfg, blocks, num_pages=pages, max_batch=max_batch, max_model_len=max_model_len,
                                       dtype=dtype, kv_dtype=kv_dtype_from_str(kvd))

    # ------------------------------------------------------------------ engine loop
    def start(self) -> None:
        if self._thread and self._thread.is_alive():
            return
        self._stop.clear()
        self._thread = threading.Thread(target=self._loop, name="vrm-engine", daemon=True)
        self._thread.start()

    def _loop(self) -> None:
        while not self._stop.is_set():
            eng = self.engine
            if self._bcast is not None:
                # keep follower ranks in lockstep: same events, then the same step
                with self._wake:
                    ev, self._events = self._events, []
                if ev or (eng is not None and eng.has_unfinished()):
                    self._bcast.exchange(ev)
                else:
                    with self._wake:
                        self._wake.wait(0.02)
                    continue
            if eng is None or not eng.has_unfinished():
                with self._wake:
                    self._wake.wait(0.02)
                continue
            try:
                eng.step()
                if self.enable_metrics:
                    METRICS.batch_size.set(len(eng.running))
                    METRICS.queue_depth.set(len(eng.waiting))
                    free = eng.kv.num_free_pages()
                    dev = str(getattr(eng.runner, "device", "cpu"))
                    METRICS.kv_free_pages.labels(dev).set(free)
                    METRICS.kv_used_pages.labels(dev).set(eng.kv.num_pages - free)
            except Exception as e:   # resume the running requests (bounded), keep serving
                log.error("engine step failed: %s", e)
                if self.fault is not None and self.fault.states:
                    self.fault.handle_fault(0, e)
                if self._bcast is None:
                    # request-level resume: re-prefill from token ids, at most twice each
                    failed = eng.recover(max_retries=2)
                else:
                    # tensor-parallel ranks would have to agree on the recovery: fail fast
                    failed = [r for r in list(eng.running) + list(eng.waiting) if not r.finished]
                for r in failed:
                    if r.future is not None and not r.future.done():
                        r.future.set_exception(e)
                    eng._finish(r, "error")

    def _kick(self) -> None:
        with self._wake:
            self._wake.notify_all()

    # ------------------------------------------------------------------ requests
    def _encode(self, prompt: Union[str, Sequence[int]]) -> List[int]:
        if isinstance(prompt, str):
            ids = self.tokenizer.encode(prompt)
            return ids or [getattr(self.tokenizer, "bos_token_id", 1) or 1]
        return [int(t) for t in prompt]

    def submit(self, prompt: Union[str, Sequence[int]], max_new_tokens: int = 128, temperature: float = 0.0,
               top_p: float = 1.0, top_k: int = 0, stop_token_ids: Sequence[int] = (), on_token=None,
               request_id=None) -> Future:
        if self.engine is None:
            raise RuntimeError("no model loaded")
        ids = self._encode(prompt)
        params = SamplingParams(max_tokens=self.autoheal.scaled(max_new_tokens), temperature=temperature,
                                top_k=top_k, top_p=top_p, stop_token_ids=tuple(stop_token_ids))
        req = self.engine.add_request(ids, params, request_id=request_id, on_token=on_token)
        if self._bcast is not None:
            with self._wake:
                self._events.append(("add", (ids, {"max_tokens": params.max_tokens, "temperature": temperature,
                                                   "top_k": top_k, "top_p": top_p,
                                                   "stop_token_ids": tuple(stop_token_ids)}, req.request_id)))
        if self.enable_metrics:
            METRICS.infer_requests.labels("submit").inc()
            METRICS.prompt_tokens.inc(len(ids))
        self._kick()
        return req.future

    def generate(self, prompt: Union[str, Sequence[int]], max_new_tokens: int = 128, temperature: float = 0.0,
                 top_p: float = 1.0, top_k: int = 0, enable_speculative: bool = False, timeout: float = 600.0,
                 return_ids: bool = False, **kw) -> Union[str, List[int]]:
        t0 = time.perf_counter()
        with span("pipeline.generate", model=str(self.model_name), max_new_tokens=max_new_tokens):
            draft = self._speculator() if enable_speculative else None
            if draft is not None:
                # draft-model speculation: greedy requests exact, sampled ones by rejection
                # sampling (outputs follow the target's distribution)
                sp = SamplingParams(max_tokens=max_new_tokens, temperature=temperature, top_k=top_k, top_p=top_p)
                ids = draft.generate(self._encode(prompt), max_new_tokens, params=sp)
                out_ids, ttft, itl = ids, None, None
            elif (enable_speculative or self.spec is not None) and temperature <= 0 and self.spec is not None:
                ids = self.spec.generate(self._encode(prompt), max_new_tokens)
                out_ids, ttft, itl = ids, None, None
            else:
                req: Request = self.submit(prompt, max_new_tokens, temperature, top_p, top_k, **kw).result(timeout)
                out_ids, ttft = req.output_ids, req.ttft
                # mean inter-token latency of this request (first token to last)
                itl = None
                if len(out_ids) > 1 and req.first_token_time is not None and req.finish_time is not None:
                    itl = (req.finish_time - req.first_token_time) / (len(out_ids) - 1)
        dt = time.perf_counter() - t0
        if self.enable_metrics:
            METRICS.tokens_generated.inc(len(out_ids))
            METRICS.infer_latency.observe(dt)
            if ttft is not None:
                METRICS.ttft.observe(ttft)
            if itl is not None:
                METRICS.itl.observe(itl)
        self.history.record("generate", str(self.model_name), len(self._encode(prompt)), len(out_ids), dt, ttft)
        return out_ids if return_ids else self.tokenizer.decode(out_ids)

    def _speculator(self):
        """Draft-model decoder for `generate(enable_speculative=True)`: the draft is
        VRM_DRAFT_MODEL, else the family default of the loaded model
        (engine.speculative.DRAFT_MODEL_MAP), when it names a preset or a local
        checkpoint; None when there is none (prompt lookup, if loaded, then applies).
        Single-process serving only (tensor-parallel ranks keep the engine lockstep)."""
        if self._draft is not None or self.llm is None or self._bcast is not None:
            return self._draft or None
        from .engine.speculative import DraftModelDecoder, guess_draft_model
        from .utils.config import flags
        self._draft = False
        name = flags.VRM_DRAFT_MODEL or guess_draft_model(str(self.model_name))
        if not name:
            return None
        try:
            get_config(name)
        except Exception as e:  # noqa: BLE001 - not a preset, alias or local checkpoint
            log.warning("draft model %s not available (%s); speculative decoding off", name, e)
            return None
        dev = self.llm.device
        cuda = dev.type == "cuda"
        draft = LLM(name, device=str(dev), dtype=torch.bfloat16 if cuda else torch.float32,
                    kv_cache_dtype="bf16" if cuda else "fp32", max_batch=2,
                    max_model_len=self.engine.max_model_len, kv_pages=None if cuda else 256,
                    use_cuda_graph=self.llm.runner.use_graph)
        self._draft = DraftModelDecoder(self.llm, draft, gamma=flags.VRM_SPEC_GAMMA, adaptive=flags.VRM_SPEC_ADAPTIVE)
        log.info("speculative decoding with draft model %s", name)
        return self._draft

    def generate_stream(self, prompt: Union[str, Sequence[int]], max_new_tokens: int = 128, temperature: float = 0.0,
                        top_p: float = 1.0, top_k: int = 0, stop: Optional[Sequence[str]] = None,
                        **kw) -> Iterator[str]:
        """Text deltas as tokens arrive.  With `stop` strings the stream ends before the
        first one and the request is aborted (no further tokens are computed)."""
        q: "queue.Queue" = queue.Queue()
        holder = {}

        def on_tok(req, tok):
            holder["id"] = req.request_id
            q.put(tok)

        fut = self.submit(prompt, max_new_tokens, temperature, top_p, top_k, on_token=on_tok, **kw)
        ids: List[int] = []
        prev = ""
        while True:
            try:
                tok = q.get(timeout=0.05)
            except queue.Empty:
                if fut.done() and q.empty():
                    break
                continue
            ids.append(tok)
            text = self.tokenizer.decode(ids)
            cut = stop_index(text, stop) if stop else -1
            if cut >= 0:
                if cut > len(prev):
                    yield text[len(prev):cut]
                self.abort(holder.get("id"))
                break
            if len(text) > len(prev):
                yield text[len(prev):]
                prev = text
        fut.result()

    def abort(self, request_id) -> bool:
        """Ends a request early (its tokens so far stay in its result)."""
        if request_id is None or self.engine is None:
            return False
        if self._bcast is not None:
            with self._wake:
                self._events.append(("abort", request_id))
        return self.engine.abort(request_id)

    def stop_watcher(self, stop: Sequence[str]):
        """on_token callback that aborts a request once its text contains a stop string
        (single-process serving; under tensor parallelism the text is cut afterwards)."""
        if not stop or self._bcast is not None:
            return None
        ids: List[int] = []
        # a stop string of n UTF-8 bytes spans at most n tokens that each decode to at
        # least one byte; byte-level BPE can also emit tokens that decode to nothing on
        # their own (a partial multi-byte character), so allow up to 4 tokens per byte.
        # Checking the text of that many last tokens at every token finds the stop
        # string as soon as it is complete, at a cost independent of the output length
        # (this runs inside the engine step)
        window = 4 * max(len(x.encode("utf-8")) for x in stop) + 4

        def on_tok(req, tok):
            ids.append(tok)
            if stop_index(self.tokenizer.decode(ids[-window:]), stop) >= 0:
                self.engine.abort(req.request_id)
        return on_tok

    def infer(self, input_ids: Union[torch.Tensor, Sequence[int]]) -> torch.Tensor:
        """Last-position logits of one sequence (no generation)."""
        ids = input_ids.flatten().tolist() if isinstance(input_ids, torch.Tensor) else list(input_ids)
        kv = self.engine.kv
        rid = f"infer-{time.time_ns()}"
        with self.engine._lock:
            kv.allocate(rid, len(ids))
            try:
                it = PrefillItem(ids, 0, kv.slots_for(rid, 0, len(ids)), kv.block_table(rid), len(ids), True)
                logits = self.engine.runner.prefill_logits([it])[-1]
            finally:
                kv.free(rid)
        return logits.float().cpu()

    def generate_batch(self, prompts: Sequence[Union[str, Sequence[int]]], max_new_tokens: int = 128,
                       **kw) -> List[str]:
        futs = [self.submit(p, max_new_tokens, **kw) for p in prompts]
        return [self.tokenizer.decode(f.result().output_ids) for f in futs]

    # ------------------------------------------------------------------ status
    def status(self) -> Dict[str, Any]:
        st: Dict[str, Any] = {"loaded": self.engine is not None, "model": self.model_name, "mode": self.mode,
                              "num_gpus": self.num_gpus, "uptime_s": (time.time() - self.loaded_at)
                              if self.loaded_at else 0}
        if self.llm is not None:
            st["config"] = self.llm.cfg.to_dict()
            st["engine"] = dict(self.engine.stats)
            st["running"] = len(self.engine.running)
            st["waiting"] = len(self.engine.waiting)
            st["kv"] = self.engine.kv.stats()
        if self.fault is not None:
            st["gpu_health"] = self.fault.status()
        st["autoheal_scale"] = self.autoheal.scale
        return st

    def benchmark(self, prompt_len: int = 128, max_new_tokens: int = 64, batch: int = 1) -> Dict[str, float]:
        g = torch.Generator().manual_seed(0)
        V = self.llm.cfg.vocab_size
        prompts = [torch.randint(0, V, (prompt_len,), generator=g).tolist() for _ in range(batch)]
        t0 = time.perf_counter()
        futs = [self.submit(p, max_new_tokens) for p in prompts]
        reqs = [f.result() for f in futs]
        dt = time.perf_counter() - t0
        toks = sum(len(r.output_ids) for r in reqs)
        ttfts = sorted(r.ttft for r in reqs if r.ttft is not None)
        return {"tokens": toks, "seconds": dt, "tok_s": toks / dt, "ttft_p50_ms": 1000 * ttfts[len(ttfts) // 2]}

    def shutdown(self) -> None:
        if self._bcast is not None:
            try:
                self._bcast.exchange("stop")
            except Exception:
                pass
        self._stop.set()
        self._kick()
        if self._thread is not None:
            self._thread.join(timeout=5)
        if self.llm is not None:
            self.llm.runner.release_graphs()
        self.llm = self.engine = None


_pipeline: Optional[InferencePipeline] = None
_plock = threading.Lock()


def get_pipeline() -> InferencePipeline:
    global _pipeline
    with _plock:
        if _pipeline is None:
            _pipeline = InferencePipeline()
        return _pipeline


def reset_pipeline() -> None:
    global _pipeline
    with _plock:
        if _pipeline is not None:
            _pipeline.shutdown()
        _pipeline = None
